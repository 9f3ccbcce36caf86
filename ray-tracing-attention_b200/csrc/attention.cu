// attention.cu -- GQA causal decode attention, split-K over history.
//
// Reference: the S_t/R_t detector, resident_ray.comp:97-117 (legacy op 3) and
// resident_detector_ordered_{scores,normalize,value}.comp: s_j = q.k_j/sqrt(hd)
// over the visible ring window, online running max m and normaliser Z,
// U = sum_j exp(s_j - m) v_j, out = U / max(Z, 1e-30) * sigmoid(gate),
// physical = (m + 20, Z).  The reference walks 256-position tiles newest
// first on one workgroup per head; here the window is split across CTAs and
// the per-split (m, Z, U) records are merged exactly like its grouped receipts
// (resident_attention_runtime.inl:603-645, verify_attention_receipts.py:117-203).
//
// B200 design: one CTA per (sequence, KV head, split).  Each warp owns two of
// eight 16-position stages; K and V rows (hd fp16 each) arrive by per-row
// cp.async.bulk into rows padded to hd*2+16 bytes (conflict-free ldmatrix).
// The four query heads that share the KV head are the N columns of an
// m16n8k16 f16 MMA: columns 0-3 hold fp16(q) and columns 4-7 the fp16
// residual q - fp16(q), so scores carry ~22 significant bits; P is split the
// same way for the P*V MMA.  Accumulation is fp32 throughout.
#include <atomic>
#include <mutex>
#include <string>

#include <cuda.h>

#include "../../include/rta.h"
#include "rta_internal.h"
#include "attention.h"
#include "packets.cuh"

namespace rta {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = 128;
constexpr int kTileMany = 16;   // positions per stage, several waves of splits
constexpr int kTileOne = 16;    // positions per stage, one wave (32 measured slower: 37.1 vs 34.6 us at L 32768)
constexpr int kStages = 12;     // one wave of splits (a long history): a ring shared by kWarpsOne warps
constexpr int kWarpsOne = 8;
constexpr int kStagesMany = 4;  // several waves of splits: one per warp of kWarps, three CTAs per SM
constexpr int kHD = 256;       // head dimension handled by this kernel
constexpr int kRowBytes = kHD * 2 + 16;
constexpr int kGroup = 4;      // query heads per KV head (GQA 16/4)

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __halves2half2(__float2half_rn(lo), __float2half_rn(hi));
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Visible window of sequence z at absolute time t: ages [lo, t].
__device__ __forceinline__ void window(const AttnParams& p, uint32_t z, uint32_t& t, uint32_t& lo, uint32_t& n) {
  t = p.pos ? p.pos[z * p.ctrl_step] : p.t;
  const uint32_t cap = p.capacity;
  lo = t + 1u >= cap ? t + 1u - cap : 0u;
  if (lo < p.history_start) lo = p.history_start;
  n = t >= lo ? t - lo + 1u : 0u;
}

// Splits sequence z uses out of the launch's nsplit (see split_by_length).
__device__ __forceinline__ uint32_t used_splits(const AttnParams& p, uint32_t n, uint32_t nsplit) {
  if (!p.split_by_length || p.packets || p.group_block) return nsplit;
  const uint32_t want = static_cast<uint32_t>((static_cast<uint64_t>(n) * nsplit + p.capacity - 1u) / p.capacity);
  return want < 1u ? 1u : want > nsplit ? nsplit : want;
}

// WARPS x 32 threads and a ring of STAGES stages of TILE positions (16 or
// 32: one or two 16-row MMA blocks).  Warp w takes tiles w, w + WARPS, ...;
// tile t lands in stage t % STAGES, and the warp that consumes tile t issues
// tile t + STAGES into the stage it frees, so the ring stays full whichever
// warp is ahead.  One wave of CTAs (a long history): eight warps over twelve
// 16-position stages (198 KB in flight per SM, two warps per scheduler);
// several waves (many sequences): four warps over four 16-position stages and
// three CTAs per SM.  Softmax in base 2: the scores carry log2(e) / sqrt(d), the
// split records' maxima go out in natural units.
template <int WARPS, int STAGES, int TILE>
__global__ void __launch_bounds__(WARPS * 32) attention_split_kernel(const AttnParams p) {
  static_assert(STAGES <= 16 && (TILE == 16 || TILE == 32), "16 barriers at most; one or two row blocks");
  constexpr int kStages = STAGES, kWarps = WARPS, kThreads = WARPS * 32, kTile = TILE, kNB = TILE / 16;
  constexpr int kStageBytes = 2 * kTile * kRowBytes;  // K rows then V rows
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint32_t* issued = reinterpret_cast<uint32_t*>(smem + kStages * kStageBytes + 128);  // copies per stage
  __half* pbuf = reinterpret_cast<__half*>(smem + kStages * kStageBytes + 256);  // [warp][8 cols][TILE pos]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = static_cast<uint32_t>(lane) >> 2, t4 = static_cast<uint32_t>(lane) & 3u;
  const uint32_t split = blockIdx.x, kv = blockIdx.y, z = blockIdx.z;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[s], 1);
      issued[s] = 0u;
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t run = p.running ? p.running[blockIdx.z * p.ctrl_step] : 1u;  // same round trip as the position
  uint32_t t, lo, n;
  window(p, z, t, lo, n);
  if (run == 0u) return;
  const uint32_t nsplit = used_splits(p, n, gridDim.x);
  if (split >= nsplit) return;  // not used by this sequence: no record, the merge skips it
  uint32_t chunk = (n + nsplit - 1u) / nsplit;
  chunk = (chunk + 63u) / 64u * 64u;
  if (chunk < 64u) chunk = 64u;
  const uint32_t first = lo + split * chunk;
  const uint32_t last = min(t + 1u, first + chunk);  // exclusive
  const uint32_t count = first < last ? last - first : 0u;
  const uint32_t ntiles = (count + kTile - 1u) / kTile;

  const __half* kbase = p.k + static_cast<size_t>(z) * p.seq_stride + static_cast<size_t>(kv) * p.kv_stride;
  const __half* vbase = p.v + static_cast<size_t>(z) * p.seq_stride + static_cast<size_t>(kv) * p.kv_stride;

  auto issue = [&](uint32_t tile) {  // called by one full warp
    const uint32_t s = tile % kStages;
    uint8_t* st = smem + s * kStageBytes;
    if (lane == 0) {
      mbar_expect_tx(&bars[s], 2u * kTile * kHD * 2u);
      __threadfence_block();
      atomicAdd(&issued[s], 1u);  // the consumer's go-ahead (see the main loop)
    }
    __syncwarp();
    // one row copy per lane and kind: 16-position tiles split the lanes
    // between K and V rows, 32-position tiles give each lane its K and V row
#pragma unroll
    for (int c = 0; c < kNB; ++c) {
      const uint32_t row = kTile == 32 ? static_cast<uint32_t>(lane) : static_cast<uint32_t>(lane) & 15u;
      const bool is_v = kTile == 32 ? c == 1 : lane >= 16;
      uint32_t pos = first + tile * kTile + row;
      if (pos >= last) pos = last - 1u;  // finite filler for masked rows
      const size_t at = static_cast<size_t>(pos % p.capacity) * p.pos_stride;
      const __half* src = is_v ? vbase + at : kbase + at;
      uint8_t* dst = st + (is_v ? kTile * kRowBytes : 0) + row * kRowBytes;
      bulk_g2s(dst, src, kHD * 2u, &bars[s]);
    }
  };
  // the ring's first tiles: tile t < STAGES by warp t % WARPS
  for (uint32_t tile = warp; tile < ntiles && tile < static_cast<uint32_t>(kStages); tile += kWarps) issue(tile);

  // Query fragments (B operand, "col" layout): column g<4 -> hi(q[head g]),
  // g>=4 -> lo residual of head g-4; k = dim.
  const uint32_t head = kv * kGroup + (g & 3u);
  const float* qh = p.q + static_cast<size_t>(z) * p.q_seq_stride + static_cast<size_t>(head) * kHD;
  uint32_t qb[16][2];
#pragma unroll
  for (int kk = 0; kk < 16; ++kk) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const uint32_t d = kk * 16 + r * 8 + 2 * t4;
      const float x0 = qh[d], x1 = qh[d + 1];
      if (g < 4u) {
        qb[kk][r] = pack_half2(x0, x1);
      } else {
        const float h0 = __half2float(__float2half_rn(x0)), h1 = __half2float(__float2half_rn(x1));
        qb[kk][r] = pack_half2(x0 - h0, x1 - h1);
      }
    }
  }

  constexpr float kLog2e = 1.4426950408889634f;
  const float inv_scale = kLog2e / sqrtf(static_cast<float>(kHD));  // scores in log2 units
  float o[16][4];
#pragma unroll
  for (int mt = 0; mt < 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, z_run[2] = {0.f, 0.f};
  bool failed = false;
  __half* pw = pbuf + warp * 8 * kTile;

  for (uint32_t tile = warp; tile < ntiles; tile += kWarps) {
    const uint32_t s = tile % kStages;
    if (kStages != kWarps) {
      // Shared ring (a stage serves several warps): the stage's barrier may
      // still be a phase short of this tile (the tile before it in the stage
      // not consumed yet), and a parity wait cannot tell phase k from k + 2.
      // Wait (boundedly) until this tile's copy has been issued, then for its
      // phase.  With one stage per warp the warp itself orders the phases.
      const uint32_t need = tile / kStages + 1u;
      if (*reinterpret_cast<volatile uint32_t*>(&issued[s]) < need) {  // rare: the clock is read only here
        const uint64_t start = globaltimer();
        for (uint32_t spin = 0; *reinterpret_cast<volatile uint32_t*>(&issued[s]) < need; ++spin) {
          if ((spin & 63u) == 63u && globaltimer() - start > RTA_WAIT_NS) {
            if (p.err) atomicOr(p.err, RTA_DEVERR_TIMEOUT);
            failed = true;
            break;
          }
          __nanosleep(32);
        }
        if (failed) break;
      }
    }
    if (!mbar_wait(&bars[s], (tile / kStages) & 1u, p.err)) {
      failed = true;
      break;
    }
    const uint32_t st = smem_u32(smem + s * kStageBytes);
    // S^T[pos][col] = K[pos] . Q[col], one 16-row block per b; four
    // independent accumulators per block break the 16-deep MMA chain
    float sc[kNB][4];
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      float sp[4][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        const uint32_t addr = st + (b * 16 + (lane & 15)) * kRowBytes + (kk * 16 + (lane >> 4) * 8) * 2;
        ldsm_x4(addr, a0, a1, a2, a3);
        mma_f16(sp[kk & 3], a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
      // hi + lo columns -> full score; lanes t4 and t4^2 end up with the same values.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float sacc = (sp[0][i] + sp[1][i]) + (sp[2][i] + sp[3][i]);
        sc[b][i] = (sacc + __shfl_xor_sync(0xffffffffu, sacc, 2)) * inv_scale;
      }
      const uint32_t pos0 = tile * kTile + b * 16 + g, pos1 = pos0 + 8u;
      if (pos0 >= count) sc[b][0] = sc[b][1] = -INFINITY;
      if (pos1 >= count) sc[b][2] = sc[b][3] = -INFINITY;
    }
    float pr[kNB][4], rescale[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {  // the two heads of this lane: 2*(t4&1)+hh
      float mx = -INFINITY;
#pragma unroll
      for (int b = 0; b < kNB; ++b) mx = fmaxf(mx, fmaxf(sc[b][hh], sc[b][2 + hh]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m_run[hh], mx);
      const float scale = m_new == -INFINITY ? 1.f : exp2f(m_run[hh] - m_new);
      float ps = 0.f;
#pragma unroll
      for (int b = 0; b < kNB; ++b) {
        const float p0 = m_new == -INFINITY ? 0.f : exp2f(sc[b][hh] - m_new);
        const float p1 = m_new == -INFINITY ? 0.f : exp2f(sc[b][2 + hh] - m_new);
        ps += p0 + p1;
        pr[b][hh] = p0;
        pr[b][2 + hh] = p1;
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      z_run[hh] = z_run[hh] * scale + ps;
      m_run[hh] = m_new;
      rescale[hh] = scale;
    }
    // the value accumulators follow a new maximum; a scale of exactly 1 (the
    // maximum did not move, the common case) changes nothing and is skipped
    if (__any_sync(0xffffffffu, (rescale[0] != 1.f) | (rescale[1] != 1.f))) {
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        o[mt][0] *= rescale[0];
        o[mt][2] *= rescale[0];
        o[mt][1] *= rescale[1];
        o[mt][3] *= rescale[1];
      }
    }
    // P (split hi/lo) -> shared [col][pos] for the B operand of P*V.
    {
      const uint32_t hA = 2u * (t4 & 1u);
      const bool hi = t4 < 2u;
#pragma unroll
      for (int b = 0; b < kNB; ++b)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t col = (hi ? 0u : 4u) + hA + hh;
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const float pv = pr[b][2 * r + hh];
            const __half ph = __float2half_rn(pv);
            pw[col * kTile + b * 16 + g + 8u * r] = hi ? ph : __float2half_rn(pv - __half2float(ph));
          }
        }
    }
    __syncwarp();
    const uint32_t vst = st + kTile * kRowBytes;
#pragma unroll
    for (int b = 0; b < kNB; ++b) {
      const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(pw + g * kTile + b * 16 + 2u * t4);
      const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(pw + g * kTile + b * 16 + 2u * t4 + 8u);
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        uint32_t a0, a1, a2, a3;
        const uint32_t mi = static_cast<uint32_t>(lane) >> 3, rr = static_cast<uint32_t>(lane) & 7u;
        const uint32_t prow = b * 16 + rr + ((mi >> 1) << 3), dcol = mt * 16 + (mi & 1u) * 8;
        ldsm_x4_t(vst + prow * kRowBytes + dcol * 2, a0, a1, a2, a3);
        mma_f16(o[mt], a0, a1, a2, a3, pb0, pb1);
      }
    }
    __syncwarp();
    if (tile + kStages < ntiles) issue(tile + kStages);
  }

  // ---- combine the warps of this CTA through shared memory ----------------
  const size_t rec = (static_cast<size_t>(z) * p.kvh + kv) * gridDim.x + split;  // record index
  if (__syncthreads_or(failed ? 1 : 0)) {
    // A stage never arrived: publish an empty record (the host sees the
    // timeout bit).  Copies issued into the ring and not consumed may still be
    // in flight: wait once more, boundedly, for the last copy into every stage,
    // so that no bulk copy lands in shared memory after this CTA has left the SM.
    if (threadIdx.x == 0)
      for (int s2 = 0; s2 < kStages; ++s2) {
        const uint32_t n_issued = issued[s2];
        if (n_issued) (void)mbar_wait(&bars[s2], (n_issued - 1u) & 1u, nullptr);
      }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < kGroup * kHD; i += kThreads) {
      p.part_o[(rec * kGroup + i / kHD) * kHD + i % kHD] = 0.f;
      if (i % kHD == 0) {
        p.part_m[rec * kGroup + i / kHD] = -INFINITY;
        p.part_z[rec * kGroup + i / kHD] = 0.f;
      }
    }
    return;
  }
  float* cm = reinterpret_cast<float*>(smem);          // [warp][4] m
  float* cz = cm + kWarps * 4;                          // [warp][4] Z
  float* co = cz + kWarps * 4;                          // [warp][8][kHD]
  {
    if (lane < 4) {  // lanes 0..3 hold heads 2*(t4&1)+hh for t4 = lane
      const uint32_t hA = 2u * (t4 & 1u);
      if (t4 < 2u) {
        cm[warp * 4 + hA] = m_run[0];
        cm[warp * 4 + hA + 1] = m_run[1];
        cz[warp * 4 + hA] = z_run[0];
        cz[warp * 4 + hA + 1] = z_run[1];
      }
    }
#pragma unroll
    for (int mt = 0; mt < 16; ++mt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t d = mt * 16 + g + ((r >> 1) << 3), col = 2u * t4 + (r & 1);
        co[(warp * 8 + col) * kHD + d] = o[mt][r];
      }
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < kGroup * kHD; i += kThreads) {
    const uint32_t h = i / kHD, d = i % kHD;
    float m = -INFINITY;
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, cm[w * 4 + h]);
    float zs = 0.f, os = 0.f;
    if (m != -INFINITY)
      for (int w = 0; w < kWarps; ++w) {
        const float e = cm[w * 4 + h] == -INFINITY ? 0.f : exp2f(cm[w * 4 + h] - m);
        zs += cz[w * 4 + h] * e;
        os += (co[(w * 8 + h) * kHD + d] + co[(w * 8 + 4 + h) * kHD + d]) * e;
      }
    p.part_o[(rec * kGroup + h) * kHD + d] = os;
    if (d == 0) {
      p.part_m[rec * kGroup + h] = m * (1.0f / kLog2e);  // natural units, as the merge expects
      p.part_z[rec * kGroup + h] = zs;
    }
  }
}


// ------------------------------------------------------------ packet history
// The same split-K detector over the reference's own history format: K as
// Q4_K and V as Q6_K blocks per (position, KV head).  Every K/V value is
// decoded exactly as ggufValue does ((d*sc)*q - dmin*m, (d*scale)*(q6-32);
// resident_quant.glsl:10-19) and all arithmetic is fp32 on the CUDA cores:
// at 4 query heads per KV head the 1416-byte packet rows, not the FMAs, bound
// the kernel.
//
// Lanes own dimensions.  Scores: lane l decodes the 4 code bytes 16+4l..19+4l
// of a key block (dims 64p+4(l%8)+j and 64p+32+4(l%8)+j, p = l/8), so a warp
// reads each key block with one coalesced 128-byte load; eight positions' 4-head
// partial dots are folded across the warp by a 31-step transpose-reduction
// after which lane L holds (position L/4, head L%4).  Values: lane l owns dims
// 32k+l (ql bytes l, 32+l, 64+l, 96+l; qh bytes 128+l, 160+l).
__device__ __forceinline__ void q4k_group_scale(const uint8_t* hb, uint32_t grp, float d, float dmin, float& dsc,
                                                float& dmm) {
  uint32_t sc, mn;
  if (grp < 4u) {
    sc = hb[4 + grp] & 63u;
    mn = hb[8 + grp] & 63u;
  } else {
    const uint32_t u = grp - 4u, mixed = hb[12 + u];
    sc = (mixed & 15u) | ((static_cast<uint32_t>(hb[4 + u]) >> 6) << 4);
    mn = (mixed >> 4) | ((static_cast<uint32_t>(hb[8 + u]) >> 6) << 4);
  }
  dsc = d * static_cast<float>(sc);    // exact (11 + 6 bits)
  dmm = dmin * static_cast<float>(mn);
}

__global__ void __launch_bounds__(kThreads) attention_packet_split_kernel(const AttnParams p) {
  __shared__ float cm[kWarps][kGroup], cz[kWarps][kGroup];
  __shared__ float co[kWarps][kGroup][kHD];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t split = blockIdx.x, kv = blockIdx.y, z = blockIdx.z;
  pdl_wait();
  pdl_launch_dependents();
  if (p.running && p.running[z * p.ctrl_step] == 0u) return;

  uint32_t t, lo, n;
  window(p, z, t, lo, n);
  uint32_t first, last;  // ages [first, last)
  if (p.group_block) {   // newest-first groups of group_block positions
    const uint64_t top = static_cast<uint64_t>(t) + 1u, off = static_cast<uint64_t>(split) * p.group_block;
    last = top > off ? static_cast<uint32_t>(top - off) : 0u;
    if (last < lo) last = lo;
    first = last > lo + p.group_block ? last - p.group_block : lo;
  } else {
    uint32_t chunk = (n + gridDim.x - 1u) / gridDim.x;
    chunk = (chunk + 63u) / 64u * 64u;
    if (chunk < 64u) chunk = 64u;
    first = lo + split * chunk;
    last = min(t + 1u, first + chunk);
    if (first > last) first = last;
  }
  const uint8_t* rows = p.packets + static_cast<size_t>(z) * p.packet_seq_stride;
  const uint32_t vbase = p.kvh * kPacketKeyBytes + kv * kPacketValueBytes;

  // this lane's query values in the key layout: qk[h][j] dims 64p+4(l%8)+j, qk[h][4+j] = +32
  const uint32_t pk = lane / 8u, kcol = 4u * (lane % 8u);
  float qk[kGroup][8];
#pragma unroll
  for (uint32_t h = 0; h < kGroup; ++h) {
    const float* qh = p.q + static_cast<size_t>(z) * p.q_seq_stride + static_cast<size_t>(kv * kGroup + h) * kHD;
#pragma unroll
    for (uint32_t j = 0; j < 4u; ++j) {
      qk[h][j] = qh[64u * pk + kcol + j];
      qk[h][4u + j] = qh[64u * pk + 32u + kcol + j];
    }
  }
  float o[kGroup][8];
#pragma unroll
  for (uint32_t h = 0; h < kGroup; ++h)
#pragma unroll
    for (uint32_t k = 0; k < 8u; ++k) o[h][k] = 0.f;
  float m_run[kGroup], z_run[kGroup];
#pragma unroll
  for (uint32_t h = 0; h < kGroup; ++h) {
    m_run[h] = -INFINITY;
    z_run[h] = 0.f;
  }
  const float inv_scale = 1.0f / 16.0f;  // 1/sqrt(256), applied after the dot like the reference

  for (uint32_t g0 = first + 8u * warp; g0 < last; g0 += 8u * kWarps) {
    // ---- scores of positions g0..g0+7 (partial over this lane's 8 dims)
    float part[32];
#pragma unroll
    for (uint32_t pi = 0; pi < 8u; ++pi) {
      const uint32_t age = g0 + pi < last ? g0 + pi : last - 1u;  // finite filler, masked below
      const uint8_t* kb = rows + static_cast<size_t>((age - p.packet_base) % p.capacity) * p.packet_stride +
                          kv * kPacketKeyBytes;
      const uint32_t hd0 = *reinterpret_cast<const uint32_t*>(kb);
      const uint32_t code = *reinterpret_cast<const uint32_t*>(kb + 16u + 4u * lane);
      const float d = half_bits_to_float(hd0 & 0xffffu), dmin = half_bits_to_float(hd0 >> 16);
      float dsc0, dmm0, dsc1, dmm1;
      q4k_group_scale(kb, 2u * pk, d, dmin, dsc0, dmm0);
      q4k_group_scale(kb, 2u * pk + 1u, d, dmin, dsc1, dmm1);
      float kval[8];
#pragma unroll
      for (uint32_t j = 0; j < 4u; ++j) {
        kval[j] = fmaf(dsc0, static_cast<float>((code >> (8u * j)) & 15u), -dmm0);
        kval[4u + j] = fmaf(dsc1, static_cast<float>((code >> (8u * j + 4u)) & 15u), -dmm1);
      }
#pragma unroll
      for (uint32_t h = 0; h < kGroup; ++h) {
        float acc = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < 8u; ++j) acc = fmaf(qk[h][j], kval[j], acc);
        part[pi * 4u + h] = acc;
      }
    }
    // transpose-reduction: lane L ends with the full dot of (position L/4, head L%4)
#pragma unroll
    for (uint32_t w = 16u, cnt = 16u; w >= 1u; w >>= 1, cnt >>= 1) {
      const bool upper = (lane & w) != 0u;
#pragma unroll
      for (uint32_t i = 0; i < cnt; ++i) {
        const float keep = upper ? part[i + cnt] : part[i];
        const float send = upper ? part[i] : part[i + cnt];
        part[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
      }
    }
    const uint32_t my_pos = lane >> 2, my_head = lane & 3u;
    const float sc = g0 + my_pos < last ? part[0] * inv_scale : -INFINITY;
    // ---- online max / normaliser per head (lanes with equal lane%4 share a head)
    float mx = sc;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    float m_new[kGroup], keep[kGroup];
#pragma unroll
    for (uint32_t h = 0; h < kGroup; ++h) {
      m_new[h] = fmaxf(m_run[h], __shfl_sync(0xffffffffu, mx, h));
      keep[h] = m_new[h] == -INFINITY ? 1.f : expf(m_run[h] - m_new[h]);
    }
    const float m_sel = my_head == 0u ? m_new[0] : my_head == 1u ? m_new[1] : my_head == 2u ? m_new[2] : m_new[3];
    const float pr = (sc == -INFINITY || m_sel == -INFINITY) ? 0.f : expf(sc - m_sel);
    float ps = pr;
    ps += __shfl_xor_sync(0xffffffffu, ps, 4);
    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
#pragma unroll
    for (uint32_t h = 0; h < kGroup; ++h) {
      z_run[h] = z_run[h] * keep[h] + __shfl_sync(0xffffffffu, ps, h);
      m_run[h] = m_new[h];
#pragma unroll
      for (uint32_t k = 0; k < 8u; ++k) o[h][k] *= keep[h];
    }
    // ---- weighted values
#pragma unroll
    for (uint32_t pi = 0; pi < 8u; ++pi) {
      if (g0 + pi >= last) break;  // uniform across the warp
      float w[kGroup];
#pragma unroll
      for (uint32_t h = 0; h < kGroup; ++h) w[h] = __shfl_sync(0xffffffffu, pr, pi * 4u + h);
      const uint8_t* vb =
          rows + static_cast<size_t>((g0 + pi - p.packet_base) % p.capacity) * p.packet_stride + vbase;
      const float d = half_bits_to_float(vb[208] | (vb[209] << 8));
      const uint32_t ql[4] = {vb[lane], vb[32u + lane], vb[64u + lane], vb[96u + lane]};
      const uint32_t qh[2] = {vb[128u + lane], vb[160u + lane]};
#pragma unroll
      for (uint32_t k = 0; k < 8u; ++k) {  // dim 32k + lane: part k/4, ql byte 64(k/4) + 32(k%2) + l
        const uint32_t part_ = k / 4u;
        const uint32_t lo4 = (ql[2u * part_ + (k % 2u)] >> (4u * ((k % 4u) / 2u))) & 15u;
        const uint32_t hi2 = (qh[part_] >> (2u * (k % 4u))) & 3u;
        const int scale = static_cast<int>(static_cast<int8_t>(vb[192u + 2u * k + (lane >> 4)]));
        const float v = (d * static_cast<float>(scale)) * static_cast<float>(static_cast<int>(lo4 | (hi2 << 4)) - 32);
#pragma unroll
        for (uint32_t h = 0; h < kGroup; ++h) o[h][k] = fmaf(w[h], v, o[h][k]);
      }
    }
  }

  // ---- combine the four warps and publish this split's record
  if (lane == 0) {
#pragma unroll
    for (uint32_t h = 0; h < kGroup; ++h) {
      cm[warp][h] = m_run[h];
      cz[warp][h] = z_run[h];
    }
  }
#pragma unroll
  for (uint32_t h = 0; h < kGroup; ++h)
#pragma unroll
    for (uint32_t k = 0; k < 8u; ++k) co[warp][h][32u * k + lane] = o[h][k];
  __syncthreads();
  const size_t rec = (static_cast<size_t>(z) * p.kvh + kv) * gridDim.x + split;
  for (uint32_t i = threadIdx.x; i < kGroup * kHD; i += kThreads) {
    const uint32_t h = i / kHD, dd = i % kHD;
    float m = -INFINITY;
    for (uint32_t w = 0; w < kWarps; ++w) m = fmaxf(m, cm[w][h]);
    float zs = 0.f, os = 0.f;
    if (m != -INFINITY)
      for (uint32_t w = 0; w < kWarps; ++w) {
        const float e = cm[w][h] == -INFINITY ? 0.f : expf(cm[w][h] - m);
        zs += cz[w][h] * e;
        os += co[w][h][dd] * e;
      }
    p.part_o[(rec * kGroup + h) * kHD + dd] = os;
    if (dd == 0) {
      p.part_m[rec * kGroup + h] = m;
      p.part_z[rec * kGroup + h] = zs;
    }
  }
}

// Merge the split records of every (sequence, head): m = max m_s,
// Z = sum Z_s e^(m_s-m), U = sum U_s e^(m_s-m), out = U/max(Z,1e-30)*gate.
// Every load goes out in one round: each thread's split maxima and sums, and
// the value rows -- with at most eight splits (many sequences) each thread
// takes its own dimension of every row; with more (one long history) warp w
// takes splits w, w+8, ... (its first kMergeRows of them at once; lane l holds
// dimensions 8l..8l+7) and the eight warps' partial rows are added in warp
// order.  The weights e^(m_s-m) follow once the maxima are in.
// Launched with programmatic dependent launch: its CTAs are resident and
// waiting when the split grid finishes.
constexpr uint32_t kMaxMergeSplits = 1024;
constexpr uint32_t kMergeWarps = kHD / 32u;
constexpr uint32_t kMergeRows = 8;  // value rows per warp requested before the weights are known
template <bool FEW>  // FEW: at most kMergeWarps splits in the launch (the path is fixed at compile time: registers)
__global__ void __launch_bounds__(kHD) attention_merge_kernel(const AttnParams p, uint32_t nsplit) {
  __shared__ float es[kMaxMergeSplits];
  __shared__ float red[kMergeWarps];
  __shared__ __align__(16) float rows[FEW ? 1 : kMergeWarps][kHD];
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t head = blockIdx.x, z = blockIdx.y, d = threadIdx.x;
  const uint32_t lane = d & 31u, warp = d >> 5;
  const uint32_t run = p.running ? p.running[z * p.ctrl_step] : 1u;  // checked once the maxima are in
  const uint32_t kv = head / kGroup, h = head % kGroup;
  const size_t rec0 = (static_cast<size_t>(z) * p.kvh + kv) * nsplit;
  if (p.split_by_length) {  // only the records this sequence's splits wrote
    uint32_t t, lo, n;
    window(p, z, t, lo, n);
    nsplit = used_splits(p, n, nsplit);
  }
  constexpr uint32_t kOwn = kMaxMergeSplits / kHD;
  float mloc = -INFINITY, zown[kOwn];
#pragma unroll
  for (uint32_t i = 0; i < kOwn; ++i) {
    const uint32_t s = d + i * kHD;
    zown[i] = 0.f;
    if (s < nsplit) {
      const float ms = p.part_m[(rec0 + s) * kGroup + h];
      zown[i] = p.part_z[(rec0 + s) * kGroup + h];
      es[s] = ms;
      mloc = fmaxf(mloc, ms);
    }
  }
  const float* po = p.part_o + (rec0 * kGroup + h) * kHD + 8u * lane;
  constexpr size_t kRecStride = static_cast<size_t>(kGroup) * kHD;  // floats between two splits' rows
  float ov[FEW ? kMergeWarps : 1];                         // few splits: dimension d of every row
  float4 va[FEW ? 1 : kMergeRows], vb[FEW ? 1 : kMergeRows];  // otherwise: this warp's first rows
  if constexpr (FEW) {
    const float* pd = p.part_o + (rec0 * kGroup + h) * kHD + d;
#pragma unroll
    for (uint32_t j = 0; j < kMergeWarps; ++j) ov[j] = j < nsplit ? pd[j * kRecStride] : 0.f;
  } else {
#pragma unroll
    for (uint32_t j = 0; j < (FEW ? 1u : kMergeRows); ++j) {
      const uint32_t s = warp + j * kMergeWarps;
      va[j] = vb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (s < nsplit) {
        va[j] = *reinterpret_cast<const float4*>(po + s * kRecStride);
        vb[j] = *reinterpret_cast<const float4*>(po + s * kRecStride + 4u);
      }
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
  if (lane == 0) red[warp] = mloc;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (uint32_t w = 1; w < kMergeWarps; ++w) m = fmaxf(m, red[w]);
  if (run == 0u) return;
  float zloc = 0.f;
#pragma unroll
  for (uint32_t i = 0; i < kOwn; ++i) {  // this thread's own entries of es
    const uint32_t s = d + i * kHD;
    if (s < nsplit) {
      const float ms = es[s];
      const float e = (ms == -INFINITY || m == -INFINITY) ? 0.f : expf(ms - m);
      es[s] = e;
      if (e != 0.f) zloc += zown[i] * e;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) zloc += __shfl_xor_sync(0xffffffffu, zloc, o);
  __syncthreads();  // maxima read by every thread before red is reused; weights visible
  if (lane == 0) red[warp] = zloc;
  float os = 0.f;
  if constexpr (FEW) {
#pragma unroll
    for (uint32_t j = 0; j < kMergeWarps; ++j)
      if (j < nsplit && es[j] != 0.f) os += ov[j] * es[j];
    __syncthreads();  // the sums in red
  } else {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    auto add_row = [&](const float4& a, const float4& b, float e) {
      if (e != 0.f) {
        acc[0] += a.x * e;
        acc[1] += a.y * e;
        acc[2] += a.z * e;
        acc[3] += a.w * e;
        acc[4] += b.x * e;
        acc[5] += b.y * e;
        acc[6] += b.z * e;
        acc[7] += b.w * e;
      }
    };
#pragma unroll
    for (uint32_t j = 0; j < (FEW ? 1u : kMergeRows); ++j) {
      const uint32_t s = warp + j * kMergeWarps;
      if (s < nsplit) add_row(va[j], vb[j], es[s]);
    }
#pragma unroll 4
    for (uint32_t s = warp + (FEW ? 1u : kMergeRows) * kMergeWarps; s < nsplit; s += kMergeWarps)  // long lists
      add_row(*reinterpret_cast<const float4*>(po + s * kRecStride),
              *reinterpret_cast<const float4*>(po + s * kRecStride + 4u), es[s]);
    *reinterpret_cast<float4*>(&rows[FEW ? 0 : warp][8u * lane]) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(&rows[FEW ? 0 : warp][8u * lane + 4u]) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    __syncthreads();
#pragma unroll
    for (uint32_t w = 0; w < (FEW ? 1u : kMergeWarps); ++w) os += rows[w][d];
  }
  float zs = 0.f;
#pragma unroll
  for (uint32_t w = 0; w < kMergeWarps; ++w) zs += red[w];
  float v = os / fmaxf(zs, 1e-30f);
  if (p.gate) v *= detector_sigmoid(p.gate[static_cast<size_t>(z) * p.gate_seq_stride + static_cast<size_t>(head) * kHD + d]);
  uint32_t od = d;
  if (p.rotary_out && d < p.rotary_out) od = (d % 2u) * (p.rotary_out / 2u) + d / 2u;  // original axis order
  p.out[static_cast<size_t>(z) * p.out_seq_stride + static_cast<size_t>(head) * kHD + od] = v;
  if (p.phys && d == 0) {
    p.phys[(static_cast<size_t>(z) * p.heads + head) * 2] = m + 20.0f;
    p.phys[(static_cast<size_t>(z) * p.heads + head) * 2 + 1] = zs;
  }
  if (!isfinite(v) && p.err) atomicOr(p.err, RTA_DEVERR_DETECTOR);
}

}  // namespace

size_t attention_smem_bytes(int stages, int warps, int tile) {
  return static_cast<size_t>(stages) * 2 * tile * kRowBytes + 256 + warps * 8 * tile * 2;
}

cudaError_t launch_attention_merge(const AttnParams& p, uint32_t nsplit, uint32_t nseq, bool pdl, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.heads, nseq);
  cfg.blockDim = dim3(kHD);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return nsplit <= kMergeWarps ? cudaLaunchKernelEx(&cfg, attention_merge_kernel<true>, p, nsplit)
                               : cudaLaunchKernelEx(&cfg, attention_merge_kernel<false>, p, nsplit);
}

cudaError_t launch_attention(const AttnParams& p, uint32_t nsplit, uint32_t nseq, bool pdl, cudaStream_t s) {
  if (p.hd != kHD || p.heads != p.kvh * kGroup || !p.q || !p.out || !p.part_m || !p.part_z || !p.part_o ||
      nsplit == 0 || nsplit > kMaxMergeSplits || nseq == 0 || p.capacity == 0)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(p.part_o) % 16u) return cudaErrorMisalignedAddress;  // the merge reads float4 rows
  if (p.packets) {  // the reference's packet history
    if (p.packet_stride != packet_bytes(p.kvh) || p.packet_stride % 8 || p.packet_seq_stride % 8 ||
        reinterpret_cast<uintptr_t>(p.packets) % 8)
      return cudaErrorMisalignedAddress;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(nsplit, p.kvh, nseq);
    cfg.blockDim = dim3(kThreads);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, attention_packet_split_kernel, p);
    if (e != cudaSuccess) return e;
    return launch_attention_merge(p, nsplit, nseq, true, s);
  }
  if (!p.k || !p.v) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(p.k) % 16 || reinterpret_cast<uintptr_t>(p.v) % 16 || p.pos_stride % 8 ||
      p.kv_stride % 8 || p.seq_stride % 8)
    return cudaErrorMisalignedAddress;
  // One-time per-device kernel setup, off the per-launch path.  Host threads
  // may make their first call on one device at the same time: the setup runs
  // under a lock and publishes the SM count with release order, so the fast
  // path (an acquire load) never reads a half-initialised entry.
  static std::mutex setup_mutex;
  static std::atomic<int> sms_of[64];
  cudaError_t e = cudaSuccess;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  int sms = sms_of[dev].load(std::memory_order_acquire);
  if (sms == 0) {
    std::lock_guard<std::mutex> lock(setup_mutex);
    sms = sms_of[dev].load(std::memory_order_relaxed);
    if (sms == 0) {
      e = cudaFuncSetAttribute(attention_split_kernel<kWarpsOne, kStages, kTileOne>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(attention_smem_bytes(kStages, kWarpsOne, kTileOne)));
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(attention_split_kernel<kWarps, kStagesMany, kTileMany>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(attention_smem_bytes(kStagesMany, kWarps, kTileMany)));
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      if (sms <= 0) return cudaErrorInvalidDevice;
      sms_of[dev].store(sms, std::memory_order_release);
    }
  }
  const bool many = static_cast<uint64_t>(nsplit) * p.kvh * nseq > static_cast<uint64_t>(sms);
  const size_t smem = many ? attention_smem_bytes(kStagesMany, kWarps, kTileMany)
                            : attention_smem_bytes(kStages, kWarpsOne, kTileOne);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, p.kvh, nseq);
  cfg.blockDim = dim3(many ? kThreads : kWarpsOne * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = many ? cudaLaunchKernelEx(&cfg, attention_split_kernel<kWarps, kStagesMany, kTileMany>, p)
           : cudaLaunchKernelEx(&cfg, attention_split_kernel<kWarpsOne, kStages, kTileOne>, p);
  if (e != cudaSuccess) return e;
  return launch_attention_merge(p, nsplit, nseq, true, s);  // resident early, waits for the split grid
}

uint32_t attention_default_splits(uint32_t history, uint32_t kvh, int sms) {
  // enough CTAs to fill the GPU once, but at least 64 positions per split
  uint32_t want = static_cast<uint32_t>(sms) / (kvh ? kvh : 1u);
  const uint32_t by_len = (history + 63u) / 64u;
  if (want > by_len) want = by_len;
  return want ? want : 1u;
}

}  // namespace rta

// ---------------------------------------------------------------------------
// Allocation-free variant of the decode attention.
//
// Some callers cannot allocate device memory at the moment they decode: a
// serving loop that runs under another framework's caching allocator (which
// owns every byte of the GPU and forbids a foreign cudaMalloc), code that must
// not trigger cudaMalloc's implicit device synchronisation on a latency-critical
// path, or an embedding that has no place to keep a per-call workspace.  For
// them the split records live in one fixed array in this library's device
// image instead of a caller workspace: every GPU that loads the library keeps
// it (about 1 MiB) until the process exits, and every call shares it.
namespace rta {
namespace {
constexpr uint32_t kStaticRecords = 1024;  // (query heads) x (splits) records at most
constexpr size_t kStaticFloats = kStaticRecords * (2 + kHD);
static __device__ __align__(256) float g_attention_scratch[kStaticFloats];
std::mutex g_scratch_mutex;
// Device address of the array per device ordinal, valid in the CUDA context it
// was looked up in (identified by the driver's context id, which is never
// reused within a process): a caller that resets the device or makes another
// context current on it gets a fresh lookup instead of a stale address.
struct ScratchAddr {
  unsigned long long ctx_id = 0;
  float* addr = nullptr;
};
ScratchAddr g_scratch_addr[64];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Id of the calling thread's current context (0 when there is none or the
// driver cannot tell); the driver entry points are resolved through the
// runtime, so the library needs no link against the driver library.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag resolved;
  std::call_once(resolved, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(fn);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}
}  // namespace
}  // namespace rta

extern "C" rta_status rta_attention_decode_f16_noalloc(const float* q, const void* k, const void* v, uint32_t time,
                                                       uint32_t capacity, uint32_t heads, uint32_t kv_heads,
                                                       uint32_t head_dim, uint32_t pos_stride, uint32_t kv_stride,
                                                       const float* gate, float* out, float* phys, uint32_t splits,
                                                       uint32_t* device_error, void* stream) {
  using namespace rta;
  if (!q || !k || !v || !out || head_dim != kHD || kv_heads == 0 || heads != 4 * kv_heads || capacity == 0 ||
      splits == 0) {
    set_last_error("rta_attention_decode_f16_noalloc: head_dim 256, heads == 4*kv_heads, capacity and splits > 0");
    return RTA_E_ARG;
  }
  if (static_cast<size_t>(heads) * splits > kStaticRecords) {
    set_last_error("rta_attention_decode_f16_noalloc: heads * splits = " +
                   std::to_string(static_cast<size_t>(heads) * splits) + " exceeds the static scratch limit of " +
                   std::to_string(kStaticRecords) + " records");
    return RTA_E_ARG;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    set_last_error("rta_attention_decode_f16_noalloc: no current CUDA device");
    return RTA_E_CUDA;
  }
  // strides count head_dim-wide rows, so only the base pointers can break the 16-byte row copies
  if (reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16) {
    set_last_error("rta_attention_decode_f16_noalloc: k and v must be 16-byte aligned (rows are copied in 16-byte "
                   "units)");
    return RTA_E_ARG;
  }
  float* scratch = nullptr;
  {
    // Set-up per device (and per context on it), with that device current:
    // the array's name is only a host-side stand-in, the kernel needs its
    // device address.  The first call on a device does this lookup.
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchAddr& slot = g_scratch_addr[dev];
    unsigned long long ctx = current_context_id();
    if (!slot.addr || ctx == 0 || slot.ctx_id != ctx) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_attention_scratch);
      if (e != cudaSuccess || !addr) {
        set_last_error(std::string("rta_attention_decode_f16_noalloc: cudaGetSymbolAddress: ") +
                       cudaGetErrorString(e));
        return RTA_E_CUDA;
      }
      if (ctx == 0) ctx = current_context_id();  // the lookup made the primary context current
      slot.addr = static_cast<float*>(addr);
      slot.ctx_id = ctx;
    }
    scratch = slot.addr;
  }
  const size_t recs = static_cast<size_t>(heads) * splits;
  AttnParams p;
  p.q = q;
  p.q_seq_stride = static_cast<size_t>(heads) * head_dim;
  p.k = static_cast<const __half*>(k);
  p.v = static_cast<const __half*>(v);
  p.kv_stride = static_cast<size_t>(kv_stride) * head_dim;
  p.pos_stride = static_cast<size_t>(pos_stride) * head_dim;
  p.heads = heads;
  p.kvh = kv_heads;
  p.hd = head_dim;
  p.capacity = capacity;
  p.t = time;
  p.gate = gate;
  p.out = out;
  p.out_seq_stride = static_cast<size_t>(heads) * head_dim;
  p.phys = phys;
  p.err = device_error;
  p.part_m = scratch;
  p.part_z = scratch + recs;
  p.part_o = scratch + 2 * recs;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (device_error) {
    e = cudaMemsetAsync(device_error, 0, 4, s);
    if (e != cudaSuccess) {
      set_last_error(std::string("rta_attention_decode_f16_noalloc: ") + cudaGetErrorString(e));
      return RTA_E_CUDA;
    }
  }
  e = launch_attention(p, splits, 1, false, s);
  if (e != cudaSuccess) {
    set_last_error(std::string("rta_attention_decode_f16_noalloc: ") + cudaGetErrorName(e) + " (" +
                   cudaGetErrorString(e) + ")");
    return RTA_E_CUDA;
  }
  return RTA_OK;
}
