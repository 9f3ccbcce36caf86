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
#include <mutex>
#include <string>

#include "../../include/rta.h"
#include "rta_internal.h"
#include "attention.h"

namespace rta {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = 128;
constexpr int kTile = 16;      // positions per stage
constexpr int kStages = 8;     // two per warp
constexpr int kHD = 256;       // head dimension handled by this kernel
constexpr int kRowBytes = kHD * 2 + 16;
constexpr int kStageBytes = 2 * kTile * kRowBytes;  // K rows then V rows
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

__global__ void __launch_bounds__(kThreads) attention_split_kernel(const AttnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  __half* pbuf = reinterpret_cast<__half*>(smem + kStages * kStageBytes + 128);  // [warp][8 cols][16 pos]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = static_cast<uint32_t>(lane) >> 2, t4 = static_cast<uint32_t>(lane) & 3u;
  const uint32_t split = blockIdx.x, kv = blockIdx.y, z = blockIdx.z;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  if (p.running && p.running[blockIdx.z * p.ctrl_step] == 0u) return;

  uint32_t t, lo, n;
  window(p, z, t, lo, n);
  const uint32_t nsplit = gridDim.x;
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
    if (lane == 0) mbar_expect_tx(&bars[s], 2u * kTile * kHD * 2u);
    __syncwarp();
    const uint32_t row = static_cast<uint32_t>(lane) & 15u;
    uint32_t pos = first + tile * kTile + row;
    if (pos >= last) pos = last - 1u;  // finite filler for masked rows
    const size_t at = static_cast<size_t>(pos % p.capacity) * p.pos_stride;
    const __half* src = lane < 16 ? kbase + at : vbase + at;
    uint8_t* dst = st + (lane < 16 ? 0 : kTile * kRowBytes) + row * kRowBytes;
    bulk_g2s(dst, src, kHD * 2u, &bars[s]);
  };
  // warp w owns tiles w, w+4, w+8, ... and stages (tile % 8)
  for (uint32_t tile = warp; tile < ntiles && tile < static_cast<uint32_t>(warp + kStages); tile += kWarps) issue(tile);

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

  const float inv_scale = 1.0f / sqrtf(static_cast<float>(kHD));
  float o[16][4];
#pragma unroll
  for (int mt = 0; mt < 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, z_run[2] = {0.f, 0.f};
  bool failed = false;
  __half* pw = pbuf + warp * 8 * kTile;

  for (uint32_t tile = warp; tile < ntiles; tile += kWarps) {
    const uint32_t s = tile % kStages;
    if (!mbar_wait(&bars[s], (tile / kStages) & 1u, p.err)) {
      failed = true;
      break;
    }
    const uint32_t st = smem_u32(smem + s * kStageBytes);
    // S^T[pos][col] = K[pos] . Q[col]
    // four independent accumulators break the 16-deep MMA dependency chain
    float sp[4][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      const uint32_t addr = st + (lane & 15) * kRowBytes + (kk * 16 + (lane >> 4) * 8) * 2;
      ldsm_x4(addr, a0, a1, a2, a3);
      mma_f16(sp[kk & 3], a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
    }
    float sacc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sacc[i] = (sp[0][i] + sp[1][i]) + (sp[2][i] + sp[3][i]);
    // hi + lo columns -> full score; lanes t4 and t4^2 end up with the same values.
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sc[i] = (sacc[i] + __shfl_xor_sync(0xffffffffu, sacc[i], 2)) * inv_scale;
    const uint32_t pos0 = tile * kTile + g, pos1 = pos0 + 8u;
    if (pos0 >= count) sc[0] = sc[1] = -INFINITY;
    if (pos1 >= count) sc[2] = sc[3] = -INFINITY;
    float pr[4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {  // the two heads of this lane: 2*(t4&1)+hh
      float mx = fmaxf(sc[hh], sc[2 + hh]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m_run[hh], mx);
      const float scale = m_new == -INFINITY ? 1.f : expf(m_run[hh] - m_new);
      const float p0 = m_new == -INFINITY ? 0.f : expf(sc[hh] - m_new);
      const float p1 = m_new == -INFINITY ? 0.f : expf(sc[2 + hh] - m_new);
      float ps = p0 + p1;
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      z_run[hh] = z_run[hh] * scale + ps;
      m_run[hh] = m_new;
#pragma unroll
      for (int mt = 0; mt < 16; ++mt) {
        o[mt][hh] *= scale;
        o[mt][2 + hh] *= scale;
      }
      pr[hh] = p0;
      pr[2 + hh] = p1;
    }
    // P (split hi/lo) -> shared [col][pos] for the B operand of P*V.
    {
      const uint32_t hA = 2u * (t4 & 1u);
      const bool hi = t4 < 2u;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t col = (hi ? 0u : 4u) + hA + hh;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float pv = pr[2 * r + hh];
          const __half ph = __float2half_rn(pv);
          pw[col * kTile + g + 8u * r] = hi ? ph : __float2half_rn(pv - __half2float(ph));
        }
      }
    }
    __syncwarp();
    const uint32_t pb0 = *reinterpret_cast<const uint32_t*>(pw + g * kTile + 2u * t4);
    const uint32_t pb1 = *reinterpret_cast<const uint32_t*>(pw + g * kTile + 2u * t4 + 8u);
    const uint32_t vst = st + kTile * kRowBytes;
#pragma unroll
    for (int mt = 0; mt < 16; ++mt) {
      uint32_t a0, a1, a2, a3;
      const uint32_t mi = static_cast<uint32_t>(lane) >> 3, rr = static_cast<uint32_t>(lane) & 7u;
      const uint32_t prow = rr + ((mi >> 1) << 3), dcol = mt * 16 + (mi & 1u) * 8;
      ldsm_x4_t(vst + prow * kRowBytes + dcol * 2, a0, a1, a2, a3);
      mma_f16(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
    if (tile + kStages < ntiles) issue(tile + kStages);
  }

  // ---- combine the four warps of this CTA through shared memory ----------
  const size_t rec = (static_cast<size_t>(z) * p.kvh + kv) * gridDim.x + split;  // record index
  if (__syncthreads_or(failed ? 1 : 0)) {
    // A stage never arrived: publish an empty record (the host sees the
    // timeout bit) and leave shared memory alone, a copy may still land.
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
        const float e = cm[w * 4 + h] == -INFINITY ? 0.f : expf(cm[w * 4 + h] - m);
        zs += cz[w * 4 + h] * e;
        os += (co[(w * 8 + h) * kHD + d] + co[(w * 8 + 4 + h) * kHD + d]) * e;
      }
    p.part_o[(rec * kGroup + h) * kHD + d] = os;
    if (d == 0) {
      p.part_m[rec * kGroup + h] = m;
      p.part_z[rec * kGroup + h] = zs;
    }
  }
}

// Merge the split records of every (sequence, head): m = max m_s,
// Z = sum Z_s e^(m_s-m), U = sum U_s e^(m_s-m), out = U/max(Z,1e-30)*gate.
__global__ void __launch_bounds__(kHD) attention_merge_kernel(const AttnParams p, uint32_t nsplit) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t head = blockIdx.x, z = blockIdx.y, d = threadIdx.x;
  if (p.running && p.running[z * p.ctrl_step] == 0u) return;
  const uint32_t kv = head / kGroup, h = head % kGroup;
  const size_t rec0 = (static_cast<size_t>(z) * p.kvh + kv) * nsplit;
  float m = -INFINITY;
  for (uint32_t s = 0; s < nsplit; ++s) m = fmaxf(m, p.part_m[(rec0 + s) * kGroup + h]);
  float zs = 0.f, os = 0.f;
  if (m != -INFINITY)
    for (uint32_t s = 0; s < nsplit; ++s) {
      const float ms = p.part_m[(rec0 + s) * kGroup + h];
      if (ms == -INFINITY) continue;
      const float e = expf(ms - m);
      zs += p.part_z[(rec0 + s) * kGroup + h] * e;
      os += p.part_o[((rec0 + s) * kGroup + h) * kHD + d] * e;
    }
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

size_t attention_smem_bytes() { return kStages * kStageBytes + 128 + kWarps * 8 * kTile * 2; }

cudaError_t launch_attention(const AttnParams& p, uint32_t nsplit, uint32_t nseq, bool pdl, cudaStream_t s) {
  if (p.hd != kHD || p.heads != p.kvh * kGroup || !p.q || !p.k || !p.v || !p.out || !p.part_m || !p.part_z ||
      !p.part_o || nsplit == 0 || nseq == 0 || p.capacity == 0)
    return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(p.k) % 16 || reinterpret_cast<uintptr_t>(p.v) % 16 || p.pos_stride % 8 ||
      p.kv_stride % 8 || p.seq_stride % 8)
    return cudaErrorMisalignedAddress;
  const size_t smem = attention_smem_bytes();
  static bool attr_set[64] = {false};  // one-time per-device kernel setup, off the per-launch path
  cudaError_t e = cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(attention_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsplit, p.kvh, nseq);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, attention_split_kernel, p);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg2 = {};
  cfg2.gridDim = dim3(p.heads, nseq);
  cfg2.blockDim = dim3(kHD);
  cfg2.stream = s;
  cfg2.attrs = attr;
  cfg2.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg2, attention_merge_kernel, p, nsplit);
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
float* g_scratch_addr[64] = {nullptr};  // device address of the array, per device ordinal
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
  float* scratch = nullptr;
  {
    // One-time set-up per device, with that device current: the array's name is
    // only a host-side stand-in, the kernel needs its device address.
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
      void* addr = nullptr;
      e = cudaGetSymbolAddress(&addr, g_attention_scratch);
      if (e != cudaSuccess || !addr) {
        set_last_error(std::string("rta_attention_decode_f16_noalloc: cudaGetSymbolAddress: ") +
                       cudaGetErrorString(e));
        return RTA_E_CUDA;
      }
      g_scratch_addr[dev] = static_cast<float*>(addr);
    }
    scratch = g_scratch_addr[dev];
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
