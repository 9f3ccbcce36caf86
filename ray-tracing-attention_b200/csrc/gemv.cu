// gemv.cu -- dequant-fused Q4_K / Q6_K GEMV for decode (batch 1..32).
//
// Reference: op 2 of ray_tracing/native/shaders/resident_math.comp:39-75 with
// quantizedOctet (resident_quant.glsl:47-94): y[r] = sum_c W[r,c] x[c] over the
// packed GGUF blocks, epilogues store / residual add (kinds 2,4) / SwiGLU
// (kind 3, resident_math.comp:71), and the vocabulary readout op 16
// (resident_math.comp:117-125) with its argmax (ops 17/23).
//
// B200 design:
//  * Weights stream HBM -> shared memory through the bulk-copy (TMA) engine:
//    a stage is 16 consecutive rows x up to 8 blocks (2048 coefficients), one
//    cp.async.bulk per row, 3-4 stages in flight per CTA, 2 CTAs per SM,
//    mbarrier completion with bounded waits.  Under programmatic dependent
//    launch the first stages (and the norm weights) are requested before
//    griddepcontrol.wait, so weight streaming overlaps the tail of the kernel
//    that produces x.
//  * Each of the 8 warps owns one 256-coefficient block of the stage.
//    Products are exact integers: the packed 4/6-bit codes are the u8 A
//    operand of mma.sync m16n8k32 (one 32-wide Q4_K group, or two 16-wide
//    Q6_K groups side by side) and the activation is split per 32-group into
//    x ~= xs * (256*H + L) with H, L signed bytes (|X| <= 32639): the s8 B
//    operand (columns H, L).  Per (row, group) the block scale and xs fold
//    into one fp32 coefficient; the Q6_K -32 code offset enters the integer
//    accumulator as its initial value (-32 * sum X), the Q4_K dmin*m offset
//    is one per-row bias per block.  The activation split keeps |relative
//    error| <= 1.5e-5 per element.
//  * The activation prologue (RMSNorm, per-head gated norm, sigmoid gate) reads
//    x once with coalesced 16-byte loads into registers; no dependent global
//    load sits inside a loop.
#include "rta_internal.h"

#include <atomic>
#include <mutex>

namespace rta {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = 8;
constexpr int kTileRows = 16;
constexpr int kStageBlocks = 8;
constexpr int kMaxChunks = 16;        // float4 chunks of x per thread: cols <= 16384
constexpr int kPass = 4;              // chunks held in registers per pass (normed inputs: cols <= 4096)
constexpr float kXLevels = 32639.0f;  // 127*256 + 127: keeps H in [-127, 127]

struct Params {
  const uint8_t* w[2];
  uint32_t nmat, rows, cols, kb_total, row_bytes;
  uint32_t ks;           // stages per matrix per tile
  uint32_t nstage;       // pipeline depth
  uint32_t stage_bytes;  // bytes of one stage buffer
  uint32_t row_pad;      // shared-memory padding after each staged row (bank spreading)
  const float* x;
  uint32_t x_stride, batch;
  int prologue;
  const float* norm_w;
  float eps;
  const float* z;
  uint32_t z_stride;
  int epilogue;
  float* y;
  uint32_t y_stride;
  unsigned long long* argmax;
  uint32_t* err;
  const uint32_t* running;
  uint32_t run_step, arg_step;  // elements between batch rows' running flags / argmax keys
  // shared-memory carve (byte offsets from the dynamic base)
  uint32_t off_bar, off_xq, off_xsc, off_scr, off_red, off_misc;
};

template <int FMT>
struct Fmt;
template <>
struct Fmt<kQ4K> {
  static constexpr uint32_t kBytes = 144;
  static constexpr uint32_t kGroups = 8;
  static constexpr uint32_t kPad = 16;  // 1152-byte rows are a multiple of 128 B: pad to spread banks
};
template <>
struct Fmt<kQ6K> {
  static constexpr uint32_t kBytes = 210;
  static constexpr uint32_t kGroups = 16;
  static constexpr uint32_t kPad = 0;   // 1680-byte rows already fall on distinct banks
};

__device__ __forceinline__ float block_sum(float v, float* red8) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red8[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kWarps; ++i) s += red8[i];
  return s;
}

// Activation prologue: x (and z, norm weights) -> int16 split tables in shared memory.
//   xq  : [batch][xgroup][half][H,L][4 words]  (16 words per 32-coefficient group)
//   xsc : [batch][xgroup] float4(xs, -32 * sum X first 16, -32 * sum X last 16 (int bits), xs * sum X)
// Thread i owns float4 chunks i, i+256, ...; 8 consecutive chunks form one
// 32-coefficient group (8 consecutive lanes), 32 chunks one 128-wide head.
// Batch row 0's first pass of x (and z), loaded right after the PDL wait so
// that its round trip overlaps the running-flag check instead of following it.
struct XFirst {
  float4 xv[kPass], zv[kPass];
};
__device__ __forceinline__ void load_x_first(const Params& p, XFirst& f) {
  const float4* xr = reinterpret_cast<const float4*>(p.x);
  const float4* zr = reinterpret_cast<const float4*>(p.z);
  const uint32_t nchunk = p.cols / 4u;
#pragma unroll
  for (int i = 0; i < kPass; ++i) {
    const uint32_t c = threadIdx.x + i * kThreads;
    f.xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    f.zv[i] = f.xv[i];
    if (c < nchunk) {
      f.xv[i] = xr[c];
      if (zr) f.zv[i] = zr[c];
    }
  }
}

__device__ void prepare_x(const Params& p, uint8_t* smem, const float4 (&wv)[kPass], const XFirst& first) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_xq);
  float4* xsc = reinterpret_cast<float4*>(smem + p.off_xsc);
  float* red8 = reinterpret_cast<float*>(smem + p.off_misc);
  const uint32_t G = p.cols / 32u, nchunk = p.cols / 4u;
  const uint32_t tid = threadIdx.x;
  const uint32_t npass = (nchunk + kPass * kThreads - 1) / (kPass * kThreads);
  for (uint32_t b = 0; b < p.batch; ++b) {
    const float4* xr = reinterpret_cast<const float4*>(p.x + static_cast<size_t>(b) * p.x_stride);
    const float4* zr = p.z ? reinterpret_cast<const float4*>(p.z + static_cast<size_t>(b) * p.z_stride) : nullptr;
    for (uint32_t pass = 0; pass < npass; ++pass) {
      float4 xv[kPass], zv[kPass];
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        const uint32_t c = tid + (pass * kPass + i) * kThreads;
        xv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        zv[i] = xv[i];
        if (b == 0u && pass == 0u) {
          xv[i] = first.xv[i];
          zv[i] = first.zv[i];
        } else if (c < nchunk) {
          xv[i] = xr[c];
          if (zr) zv[i] = zr[c];
        }
      }
      float inv = 1.f;
      if (p.prologue == kRmsNorm) {  // single pass: cols <= kPass * 4 * kThreads
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < kPass; ++i)
          s += xv[i].x * xv[i].x + xv[i].y * xv[i].y + xv[i].z * xv[i].z + xv[i].w * xv[i].w;
        inv = rsqrtf(block_sum(s, red8) / static_cast<float>(p.cols) + p.eps);
      }
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        const uint32_t ci = (pass * kPass + i) * kThreads;
        if (ci >= nchunk) break;  // uniform across the CTA
        const uint32_t c = tid + ci;
        float v[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        if (p.prologue == kRmsNorm) {
          const float w4[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = v[e] * inv * w4[e];
        } else if (p.prologue == kHeadGate) {
          // one 128-wide head = the 32 chunks of this warp in this iteration
          float s = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
          s = warp_sum(s);
          const float hinv = rsqrtf(s / 128.0f + p.eps);
          const float w4[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
          const float z4[4] = {zv[i].x, zv[i].y, zv[i].z, zv[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = v[e] * (((hinv * w4[e]) * z4[e]) * detector_sigmoid(z4[e]));
        } else if (p.prologue == kSigmoidGate) {
          const float z4[4] = {zv[i].x, zv[i].y, zv[i].z, zv[i].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = v[e] * detector_sigmoid(z4[e]);
        }
        float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        const float scale = amax > 0.f ? kXLevels / amax : 0.f;
        uint32_t hw = 0u, lw = 0u;
        int sx = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          int X = __float2int_rn(v[e] * scale);
          X = max(-32639, min(32639, X));
          const int L = static_cast<int>(static_cast<int8_t>(X & 0xff));
          const int H = (X - L) >> 8;
          hw |= (static_cast<uint32_t>(H) & 0xffu) << (8 * e);
          lw |= (static_cast<uint32_t>(L) & 0xffu) << (8 * e);
          sx += X;
        }
        sx += __shfl_xor_sync(0xffffffffu, sx, 1);
        sx += __shfl_xor_sync(0xffffffffu, sx, 2);  // 16-element half sums
        const int sx_hi = __shfl_xor_sync(0xffffffffu, sx, 4);
        if (c < nchunk) {
          const uint32_t g = c / 8u, k8 = c % 8u, half = k8 / 4u, t = k8 % 4u;
          uint32_t* base = xq + (static_cast<size_t>(b) * G + g) * 16u + half * 8u;
          base[t] = hw;
          base[4u + t] = lw;
          if (k8 == 0u) {
            const float xs = amax / kXLevels;
            // .y/.z: the Q6_K code offset -32 * (sum of X over each 16-wide half),
            // as integer bits: it seeds the MMA accumulator of that half.
            xsc[b * G + g] = make_float4(xs, __int_as_float(-32 * sx), __int_as_float(-32 * sx_hi),
                                         __fmul_rn(xs, static_cast<float>(sx + sx_hi)));
          }
        }
      }
    }
  }
  __syncthreads();
}

template <int FMT>
__device__ __forceinline__ const uint8_t* stage_src(const Params& p, uint32_t tile, uint32_t mat, uint32_t kst,
                                                    uint32_t row) {
  return p.w[mat] + static_cast<size_t>(tile * kTileRows + row) * p.row_bytes +
         static_cast<size_t>(kst) * kStageBlocks * Fmt<FMT>::kBytes;
}

// Position of a stage in the (tile, matrix, k-stage) walk of one CTA, advanced
// by counting instead of dividing the stage index on every iteration.
struct StageCursor {
  uint32_t s = 0, parity = 0, tile_local = 0, r = 0, mat = 0, kst = 0;
  __device__ __forceinline__ void next(uint32_t nstage, uint32_t ks, uint32_t ipt) {
    if (++s == nstage) {
      s = 0;
      parity ^= 1u;
    }
    if (++kst == ks) {
      kst = 0;
      ++mat;
    }
    if (++r == ipt) {
      r = 0;
      mat = 0;
      ++tile_local;
    }
  }
};

// True while at least one batch row of the launch is still generating.
__device__ __forceinline__ bool any_running(const Params& p) {
  if (!p.running) return true;
  for (uint32_t b = 0; b < p.batch; ++b)
    if (p.running[b * p.run_step] != 0u) return true;
  return false;
}

// Per-warp scratch (floats): dsc[16 groups][17] | dmm[16][17] | bias[16 rows]
constexpr uint32_t kScrStride = 17;
constexpr uint32_t kScrFloats = 2 * 16 * kScrStride + kTileRows;

// NB: batch rows per launch (1, 2, 4, 8).  Every batch row runs the identical
// batch-1 arithmetic, so a row's result does not depend on the batch size.
template <int FMT, int NB>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = static_cast<uint32_t>(lane) >> 2, t = static_cast<uint32_t>(lane) & 3u;
  const uint32_t tiles = p.rows / kTileRows;
  const uint32_t ipt = p.nmat * p.ks;  // stages per tile
  const uint32_t my_tiles = blockIdx.x < tiles ? (tiles - 1u - blockIdx.x) / gridDim.x + 1u : 0u;
  const uint32_t total = my_tiles * ipt;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + p.off_misc + 64);
  constexpr uint32_t NG = Fmt<FMT>::kGroups;

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.nstage; ++s) mbar_init(&bars[s], 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t policy = evict_first_policy();

  StageCursor prod;  // producer position (warp 0 only); stages are issued in order
  auto issue = [&]() {
    const uint32_t s = prod.s, tile = blockIdx.x + prod.tile_local * gridDim.x;
    const uint32_t nb = min(static_cast<uint32_t>(kStageBlocks), p.kb_total - prod.kst * kStageBlocks);
    const uint32_t chunk = nb * Fmt<FMT>::kBytes;
    if (lane == 0) mbar_expect_tx(&bars[s], chunk * kTileRows);
    __syncwarp();
    if (lane < kTileRows)
      bulk_g2s_stream(smem + s * p.stage_bytes + lane * (chunk + p.row_pad),
                      stage_src<FMT>(p, tile, prod.mat, prod.kst, lane), chunk, &bars[s], policy);
    prod.next(p.nstage, p.ks, ipt);
  };

  uint32_t issued = min(total, p.nstage), drain_from = 0;  // tracked by every thread alike
  if (warp == 0)
    for (uint32_t it = 0; it < issued; ++it) issue();

  // norm weights are constant: read them before waiting on the producer
  float4 wv[kPass];
#pragma unroll
  for (int i = 0; i < kPass; ++i) wv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (p.prologue == kRmsNorm || p.prologue == kHeadGate) {
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
#pragma unroll
    for (int i = 0; i < kPass; ++i)
      if (threadIdx.x + i * kThreads < p.cols / 4u) wv[i] = w4[threadIdx.x + i * kThreads];
  }

  pdl_wait();                 // activations (and residual target) are now visible
  pdl_launch_dependents();    // let the next kernel start streaming its weights
  XFirst xfirst;
  load_x_first(p, xfirst);
  if (!any_running(p)) {
    if (threadIdx.x == 0)  // generation stopped: drain the stages in flight and leave
      for (uint32_t j = 0; j < issued; ++j) (void)mbar_wait(&bars[j % p.nstage], (j / p.nstage) & 1u, nullptr);
    return;
  }
  prepare_x(p, smem, wv, xfirst);

  const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem + p.off_xq);
  const float4* xsc = reinterpret_cast<const float4*>(smem + p.off_xsc);
  float* scr = reinterpret_cast<float*>(smem + p.off_scr) + warp * kScrFloats;
  float* dsc_s = scr;
  float* dmm_s = scr + 16 * kScrStride;
  float* bias_s = scr + 2 * 16 * kScrStride;
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  const uint32_t G = p.cols / 32u;
  const uint32_t redsz = kWarps * 2u * kTileRows * p.batch;  // one buffer (per parity)
  const uint32_t nbatch = p.batch;

  // acc: the matrix being streamed; held: matrix 0 of a two-matrix (SwiGLU)
  // tile once its k-range is done.  Only static indices, so both stay in registers.
  float acc[NB][2], held[NB][2];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b][0] = acc[b][1] = held[b][0] = held[b][1] = 0.f;

  unsigned long long best = 0ull;  // epilogue thread's running argmax key
  bool aborted = false;
  StageCursor cons;

  for (uint32_t it = 0; it < total; ++it, cons.next(p.nstage, p.ks, ipt)) {
    const uint32_t s = cons.s, parity = cons.parity, tile_local = cons.tile_local, r = cons.r, kst = cons.kst;
    const uint32_t tile = blockIdx.x + tile_local * gridDim.x;
    if (!mbar_wait(&bars[s], parity, p.err)) *abort_flag = 1u;
    const bool ok = *abort_flag == 0u;
    const uint32_t nb = min(static_cast<uint32_t>(kStageBlocks), p.kb_total - kst * kStageBlocks);
    const uint32_t chunk = nb * Fmt<FMT>::kBytes, rstride = chunk + p.row_pad;
    const uint8_t* stage = smem + s * p.stage_bytes;
    const uint32_t kb = static_cast<uint32_t>(warp);

    if (ok && kb < nb) {
      const uint32_t xg0 = (kst * kStageBlocks + kb) * 8u;  // first x-group of this block
      // ---- per (row, group) block scales: lane -> row lane/2, half of the groups
      {
        const uint32_t row = static_cast<uint32_t>(lane) >> 1, gh = (static_cast<uint32_t>(lane) & 1u) * (NG / 2u);
        const uint8_t* bk = stage + row * rstride + kb * Fmt<FMT>::kBytes;
        float bias = 0.f;  // batch-1 only: sum over this lane's groups
        if constexpr (FMT == kQ4K) {
          const float d = half_bits_to_float(bk[0] | (bk[1] << 8));
          const float dmin = half_bits_to_float(bk[2] | (bk[3] << 8));
#pragma unroll
          for (uint32_t q = 0; q < NG / 2u; ++q) {
            const uint32_t grp = gh + q;
            uint32_t sc, mn;
            if (grp < 4u) {
              sc = bk[4 + grp] & 63u;
              mn = bk[8 + grp] & 63u;
            } else {
              const uint32_t u = grp - 4u, mixed = bk[12 + u];
              sc = (mixed & 15u) | ((static_cast<uint32_t>(bk[4 + u]) >> 6) << 4);
              mn = (mixed >> 4) | ((static_cast<uint32_t>(bk[8 + u]) >> 6) << 4);
            }
            const float dsc = __fmul_rn(d, static_cast<float>(sc)), dmm = __fmul_rn(dmin, static_cast<float>(mn));
            if constexpr (NB == 1) {
              const float4 xv = xsc[xg0 + grp];
              dsc_s[grp * kScrStride + row] = __fmul_rn(dsc, xv.x);
              bias = fmaf(dmm, xv.w, bias);
            } else {
              dsc_s[grp * kScrStride + row] = dsc;
              dmm_s[grp * kScrStride + row] = dmm;
            }
          }
        } else {
          const float d = half_bits_to_float(bk[208] | (bk[209] << 8));
#pragma unroll
          for (uint32_t q = 0; q < NG / 2u; ++q) {
            const uint32_t grp = gh + q;
            const float dsc = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(bk[192 + grp])));
            if constexpr (NB == 1) {
              dsc_s[grp * kScrStride + row] = __fmul_rn(dsc, xsc[xg0 + grp / 2u].x);
            } else {
              dsc_s[grp * kScrStride + row] = dsc;
            }
          }
        }
        if constexpr (NB == 1 && FMT == kQ4K) {
          const float other = __shfl_xor_sync(0xffffffffu, bias, 1);
          if ((lane & 1) == 0) bias_s[row] = bias + other;  // (first half) + (second half)
        }
      }
      __syncwarp();

      // coefficient of (row, group) for batch row b (identical arithmetic for every NB)
      auto coef = [&](uint32_t grp, uint32_t row, uint32_t b, uint32_t xg) -> float {
        if constexpr (NB == 1) return dsc_s[grp * kScrStride + row];
        else return __fmul_rn(dsc_s[grp * kScrStride + row], xsc[b * G + xg].x);
      };

      if constexpr (FMT == kQ4K) {
        const uint8_t* rg = stage + g * rstride + kb * 144u + 16u;
        const uint8_t* rg8 = stage + (g + 8u) * rstride + kb * 144u + 16u;
#pragma unroll
        for (uint32_t pch = 0; pch < 4u; ++pch) {
          const uint32_t w0 = *reinterpret_cast<const uint32_t*>(rg + 32u * pch + 4u * t);
          const uint32_t w2 = *reinterpret_cast<const uint32_t*>(rg + 32u * pch + 16u + 4u * t);
          const uint32_t w1 = *reinterpret_cast<const uint32_t*>(rg8 + 32u * pch + 4u * t);
          const uint32_t w3 = *reinterpret_cast<const uint32_t*>(rg8 + 32u * pch + 16u + 4u * t);
#pragma unroll
          for (uint32_t nib = 0; nib < 2u; ++nib) {
            const uint32_t grp = 2u * pch + nib, sh = 4u * nib;
            const uint32_t a0 = (w0 >> sh) & 0x0f0f0f0fu, a1 = (w1 >> sh) & 0x0f0f0f0fu;
            const uint32_t a2 = (w2 >> sh) & 0x0f0f0f0fu, a3 = (w3 >> sh) & 0x0f0f0f0fu;
            const uint32_t xg = xg0 + grp;
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              if (static_cast<uint32_t>(b) >= nbatch) break;
              const uint32_t* xw = xq + (static_cast<size_t>(b) * G + xg) * 16u;
              const uint32_t b0 = g < 2u ? xw[g * 4u + t] : 0u, b1 = g < 2u ? xw[8u + g * 4u + t] : 0u;
              int c[4] = {0, 0, 0, 0};
              mma_u8s8_k32(c, a0, a1, a2, a3, b0, b1);
              if (t == 0u) {
                acc[b][0] = fmaf(coef(grp, g, b, xg), static_cast<float>(c[0] * 256 + c[1]), acc[b][0]);
                acc[b][1] = fmaf(coef(grp, g + 8u, b, xg), static_cast<float>(c[2] * 256 + c[3]), acc[b][1]);
              }
            }
          }
        }
      } else {
        // Two 16-wide groups per m16n8k32: the first group's (H, L) in B
        // columns 0-1 over k 0..15, the second group's in columns 2-3 over k
        // 16..31; lanes t = 0 / 1 accumulate the first / second group.
        const uint32_t rowg = g * rstride + kb * 210u, rowg8 = (g + 8u) * rstride + kb * 210u;
#pragma unroll
        for (uint32_t part = 0; part < 2u; ++part) {
          uint32_t ql[2][4], qh[2][2];
#pragma unroll
          for (uint32_t q = 0; q < 4u; ++q) {
            const uint32_t off = part * 64u + 16u * q + 4u * t;
            ql[0][q] = lds_u32_unaligned(stage, rowg + off);
            ql[1][q] = lds_u32_unaligned(stage, rowg8 + off);
          }
#pragma unroll
          for (uint32_t q = 0; q < 2u; ++q) {
            const uint32_t off = 128u + part * 32u + 16u * q + 4u * t;
            qh[0][q] = lds_u32_unaligned(stage, rowg + off);
            qh[1][q] = lds_u32_unaligned(stage, rowg8 + off);
          }
#pragma unroll
          for (uint32_t j = 0; j < 4u; ++j) {
            uint32_t a[4];
#pragma unroll
            for (uint32_t h = 0; h < 2u; ++h) {  // h: first / second group of the pair
              const uint32_t jj = 2u * j + h, ns = (jj / 4u) * 4u, hs = (jj / 2u) * 2u;
              a[2 * h] = ((ql[0][jj % 4u] >> ns) & 0x0f0f0f0fu) | (((qh[0][jj % 2u] >> hs) & 0x03030303u) << 4);
              a[2 * h + 1] = ((ql[1][jj % 4u] >> ns) & 0x0f0f0f0fu) | (((qh[1][jj % 2u] >> hs) & 0x03030303u) << 4);
            }
            const uint32_t xg = xg0 + part * 4u + j;
            const uint32_t grp = part * 8u + 2u * j + (t & 1u);
#pragma unroll
            for (int b = 0; b < NB; ++b) {
              if (static_cast<uint32_t>(b) >= nbatch) break;
              const uint32_t word = g < 4u ? xq[(static_cast<size_t>(b) * G + xg) * 16u + g * 4u + t] : 0u;
              const uint32_t b0 = g < 2u ? word : 0u, b1 = (g >= 2u && g < 4u) ? word : 0u;
              // seed the L column with -32 * sum(X) of this lane's 16-group: the
              // integer is then sum((q - 32) * X), |.| < 2^24, exact in fp32
              const int off = __float_as_int((t & 1u) ? xsc[b * G + xg].z : xsc[b * G + xg].y);
              int c[4] = {0, off, 0, off};
              mma_u8s8_k32(c, a[0], a[1], a[2], a[3], b0, b1);
              if (t < 2u) {
                acc[b][0] = fmaf(coef(grp, g, b, xg), static_cast<float>(c[0] * 256 + c[1]), acc[b][0]);
                acc[b][1] = fmaf(coef(grp, g + 8u, b, xg), static_cast<float>(c[2] * 256 + c[3]), acc[b][1]);
              }
            }
          }
        }
      }
      // Q4_K block offsets (dmin * m), in the same order for every NB; the
      // Q6_K offset is already inside the integer products
      if constexpr (FMT == kQ4K) {
        if (t == 0u) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            if (static_cast<uint32_t>(b) >= nbatch) break;
#pragma unroll
            for (uint32_t hr = 0; hr < 2u; ++hr) {
              const uint32_t row = g + 8u * hr;
              float bias;
              if constexpr (NB == 1) {
                bias = bias_s[row];
              } else {
                float part_b[2] = {0.f, 0.f};
#pragma unroll
                for (uint32_t grp = 0; grp < NG; ++grp)
                  part_b[grp / (NG / 2u)] =
                      fmaf(dmm_s[grp * kScrStride + row], xsc[b * G + xg0 + grp].w, part_b[grp / (NG / 2u)]);
                bias = part_b[0] + part_b[1];
              }
              acc[b][hr] = acc[b][hr] - bias;
            }
          }
        }
      }
      __syncwarp();
    }

    const bool tile_end = (r == ipt - 1u);
    float* redbuf = red + (tile_local & 1u) * redsz;
    if (p.nmat == 2u && kst == p.ks - 1u && cons.mat == 0u) {  // matrix 0 of the tile is complete
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        held[b][0] = acc[b][0];
        held[b][1] = acc[b][1];
        acc[b][0] = acc[b][1] = 0.f;
      }
    }
    if (tile_end) {
      // Q6_K: the second group of every pair was accumulated by lane t = 1
      auto publish = [&](int m, float (&v)[NB][2]) {
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float o0 = __shfl_down_sync(0xffffffffu, v[b][0], 1);
          const float o1 = __shfl_down_sync(0xffffffffu, v[b][1], 1);
          if (t == 0u && static_cast<uint32_t>(b) < nbatch) {
            redbuf[((warp * 2 + m) * kTileRows + g) * nbatch + b] = FMT == kQ6K ? v[b][0] + o0 : v[b][0];
            redbuf[((warp * 2 + m) * kTileRows + g + 8u) * nbatch + b] = FMT == kQ6K ? v[b][1] + o1 : v[b][1];
          }
          v[b][0] = v[b][1] = 0.f;
        }
      };
      if (p.nmat == 2u) {
        publish(0, held);
        publish(1, acc);
      } else {
        publish(0, acc);
      }
    }
    __syncthreads();  // stage s consumed; reduction buffer visible
    if (*abort_flag) {
      aborted = true;
      drain_from = it;
      break;
    }
    if (it + p.nstage < total) {
      if (warp == 0) issue();
      issued = it + p.nstage + 1u;
    }
    if (tile_end)
      for (uint32_t idx = threadIdx.x; idx < kTileRows * nbatch; idx += kThreads) {
        const uint32_t row = idx % kTileRows, b = idx / kTileRows;
        float v[2] = {0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (static_cast<uint32_t>(m) >= p.nmat) break;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) v[m] += redbuf[((w * 2 + m) * kTileRows + row) * nbatch + b];
        }
        const uint32_t R = tile * kTileRows + row;
        if (p.running && p.running[b * p.run_step] == 0u) continue;  // this batch row has stopped
        float* yp = p.y ? p.y + static_cast<size_t>(b) * p.y_stride + R : nullptr;
        if (p.epilogue == kSwiGLU) {
          const float gv = v[0], uv = v[1];
          const float amp = fabsf(gv) * fabsf(uv) * detector_sigmoid(gv);
          const float sgn = (gv > 0.f ? 1.f : gv < 0.f ? -1.f : 0.f) * (uv > 0.f ? 1.f : uv < 0.f ? -1.f : 0.f);
          *yp = sgn * amp;
        } else if (p.epilogue == kAccumulate) {
          *yp += v[0];
        } else if (yp) {
          *yp = v[0];
        }
        if (p.argmax) {
          const unsigned long long key = pack_argmax(v[0], R);
          best = key > best ? key : best;
        }
      }
  }

  if (aborted) {
    // Bounded drain of the copies this CTA still has in flight, so no bulk
    // copy lands in shared memory after the CTA has exited.
    if (threadIdx.x == 0)
      for (uint32_t j = drain_from; j < issued; ++j) (void)mbar_wait(&bars[j % p.nstage], (j / p.nstage) & 1u, nullptr);
    return;
  }
  if (p.argmax) {
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem + p.off_red);
    __syncthreads();
    cand[threadIdx.x] = threadIdx.x < kTileRows * nbatch ? best : 0ull;
    __syncthreads();
    if (threadIdx.x < nbatch) {
      unsigned long long m = 0ull;
      for (uint32_t row = 0; row < kTileRows; ++row) {
        const unsigned long long c = cand[threadIdx.x * kTileRows + row];
        m = c > m ? c : m;
      }
      if (m) atomicMax(p.argmax + static_cast<size_t>(threadIdx.x) * p.arg_step, m);
    }
  }
}

// ------------------------------------------------------------ tiled layout
// Engine-resident weights are re-laid out once at load ("tiled" formats): for
// every 16-row tile rt and block column kb the 16 blocks (rows 16rt..16rt+15,
// column kb) form one contiguous tile of 16 * block_bytes bytes, tiles ordered
// (rt, kb) row-major, so a stage of 16 rows x 8 blocks is one bulk copy.
// Inside a tile the codes are stored in mma.sync A-fragment order, in planes of
// 32 lanes x 16 bytes (one conflict-free 16-byte shared load per lane and
// plane), followed by the per-row scale bytes.  Same bytes, new order:
//  Q4_K tile (2304 B): planes p = 0..3: lane (g, t) holds the 4-byte words
//    row g [16+32p+4t], row g+8 [same], row g [16+32p+16+4t], row g+8 [same]
//    (GGUF code bytes, both nibbles); then 16 rows x 16 header bytes
//    (d, dmin, 12 packed 6-bit scales) exactly as in the block.
//  Q6_K tile (3360 B): lane (g, t) owns 96 bytes, 12 per 32-coefficient chunk j:
//    L0: byte e = code(row g, 32j+4t+e) & 15 | (code(row g+8, same) & 15) << 4
//    L1: the same for coefficient 32j+16+4t+e
//    Hh: byte e = top 2 bits of those four codes at bits 0-1, 2-3, 4-5, 6-7
//    lane byte b is stored in plane b/16 at lane*16 + b%16 (6 planes); then
//    16 rows x 16 int8 scales, then 16 rows x fp16 d.
template <int FMT>
struct TileFmt;
template <>
struct TileFmt<kQ4K> {
  static constexpr uint32_t kBytes = 2304, kPlanes = 4, kScaleAt = 2048;
};
template <>
struct TileFmt<kQ6K> {
  static constexpr uint32_t kBytes = 3360, kPlanes = 6, kScaleAt = 3072, kDAt = 3328;
};

__device__ __forceinline__ uint32_t q6_code(const uint8_t* blk, uint32_t n) {
  const uint32_t part = n / 128u, within = n % 128u;
  const uint32_t lo = (blk[part * 64u + within % 64u] >> (4u * (within / 64u))) & 15u;
  const uint32_t hi = (blk[128u + part * 32u + within % 32u] >> (2u * (within / 32u))) & 3u;
  return lo | (hi << 4);
}

template <int FMT>
__device__ __forceinline__ uint8_t tile_byte(const uint8_t* blocks, uint32_t o) {
  constexpr uint32_t BB = FMT == kQ4K ? kQ4KBytes : kQ6KBytes;
  if constexpr (FMT == kQ4K) {
    if (o < 2048u) {
      const uint32_t pl = o / 512u, lane = (o % 512u) / 16u, w = (o % 16u) / 4u, bi = o % 4u;
      const uint32_t g = lane >> 2, t = lane & 3u, row = g + 8u * (w & 1u);
      return blocks[row * BB + 16u + 32u * pl + 16u * (w >> 1) + 4u * t + bi];
    }
    const uint32_t r = (o - 2048u) / 16u, i = (o - 2048u) % 16u;
    return blocks[r * BB + i];
  } else {
    if (o < 3072u) {
      const uint32_t lane = (o % 512u) / 16u, lb = (o / 512u) * 16u + o % 16u;
      const uint32_t j = lb / 12u, word = (lb % 12u) / 4u, e = lb % 4u, g = lane >> 2, t = lane & 3u;
      const uint8_t* rg = blocks + g * BB;
      const uint8_t* rg8 = blocks + (g + 8u) * BB;
      const uint32_t k0 = 32u * j + 4u * t + e, k1 = k0 + 16u;
      if (word == 0u) return static_cast<uint8_t>((q6_code(rg, k0) & 15u) | ((q6_code(rg8, k0) & 15u) << 4));
      if (word == 1u) return static_cast<uint8_t>((q6_code(rg, k1) & 15u) | ((q6_code(rg8, k1) & 15u) << 4));
      return static_cast<uint8_t>((q6_code(rg, k0) >> 4) | ((q6_code(rg8, k0) >> 4) << 2) |
                                  ((q6_code(rg, k1) >> 4) << 4) | ((q6_code(rg8, k1) >> 4) << 6));
    }
    if (o < 3328u) {
      const uint32_t r = (o - 3072u) / 16u, i = (o - 3072u) % 16u;
      return blocks[r * BB + 192u + i];
    }
    const uint32_t r = (o - 3328u) / 2u, i = (o - 3328u) % 2u;
    return blocks[r * BB + 208u + i];
  }
}

// grid (column blocks, row tiles); one tile per CTA
template <int FMT>
__global__ void __launch_bounds__(256) tile_weights_kernel(const uint8_t* __restrict__ src, uint32_t KB,
                                                           uint8_t* __restrict__ dst) {
  constexpr uint32_t BB = FMT == kQ4K ? kQ4KBytes : kQ6KBytes, TB = TileFmt<FMT>::kBytes;
  __shared__ uint8_t blocks[16 * BB];
  const uint32_t kb = blockIdx.x, rt = blockIdx.y;
  for (uint32_t i = threadIdx.x; i < 16u * BB; i += blockDim.x) {
    const uint32_t r = i / BB, o = i % BB;
    blocks[i] = src[(static_cast<size_t>(rt * 16u + r) * KB + kb) * BB + o];
  }
  __syncthreads();
  uint8_t* out = dst + (static_cast<size_t>(rt) * KB + kb) * TB;
  for (uint32_t o = threadIdx.x; o < TB; o += blockDim.x) out[o] = tile_byte<FMT>(blocks, o);
}

// Activation terms one lane needs for one 256-coefficient block of one batch
// row: the s8 B fragments of the 8 mma steps (zero except in the lanes whose
// columns carry that step's (H, L) pair), and per accumulator chain the
// activation scale xs and the offset term (Q4_K: xs * sum X; Q6_K: -32 * sum X
// as integer bits).
template <int FMT>
struct XTerms {
  uint32_t b[8][2];
  float xs[FMT == kQ4K ? 2 : 4];
  float aux[FMT == kQ4K ? 2 : 4];
};

template <int FMT>
__device__ __forceinline__ void load_xterms(XTerms<FMT>& x, const uint32_t* xq, const float4* xsc, uint32_t xg0,
                                            uint32_t g, uint32_t t) {
  const uint32_t hl = g & 1u;
  if constexpr (FMT == kQ4K) {
    // step grp (group grp): columns 2*(grp%4) (H) and +1 (L), i.e. lanes g = 2*(grp%4) + hl
#pragma unroll
    for (uint32_t grp = 0; grp < 8u; ++grp) {
      const uint32_t* xw = xq + (xg0 + grp) * 16u;
      const bool mine = (g >> 1) == (grp & 3u);
      x.b[grp][0] = mine ? xw[hl * 4u + t] : 0u;
      x.b[grp][1] = mine ? xw[8u + hl * 4u + t] : 0u;
    }
#pragma unroll
    for (uint32_t u = 0; u < 2u; ++u) {
      const float4 v = xsc[xg0 + 4u * u + t];  // this lane accumulates group 4u + t
      x.xs[u] = v.x;
      x.aux[u] = v.w;
    }
  } else {
    // step j (32-coefficient chunk j = two 16-groups): first group in columns
    // 4*(j%2) + (0, 1) over k 0..15, second in columns 4*(j%2) + (2, 3) over k 16..31
#pragma unroll
    for (uint32_t j = 0; j < 8u; ++j) {
      const uint32_t* xw = xq + (xg0 + j) * 16u;
      const bool mine = (g >> 2) == (j & 1u);
      const bool second = ((g >> 1) & 1u) != 0u;
      x.b[j][0] = (mine && !second) ? xw[hl * 4u + t] : 0u;
      x.b[j][1] = (mine && second) ? xw[8u + hl * 4u + t] : 0u;
    }
#pragma unroll
    for (uint32_t u = 0; u < 4u; ++u) {
      const float4 v = xsc[xg0 + 2u * u + (t >> 1)];  // this lane accumulates group 4u + t
      x.xs[u] = v.x;
      x.aux[u] = (t & 1u) ? v.z : v.y;
    }
  }
}

// NB: batch rows per launch (1, 2, 4, 8); every batch row runs the identical
// batch-1 arithmetic, so a row's result does not depend on the batch size.
// One 16-row x 256-column block for up to 4*NJ batch rows in the batch-column
// layout.  B column g of column set j is batch row 4j + g/2 (H for even g, L for
// odd); lane t receives rows g and g+8 of batch row 4j + t.  Per batch row the
// float operations and their order equal the batch-1 layout's: a (row, group)
// product enters slot group % 4 with coefficient fmul(fmul(d, sc), xs), groups in
// increasing order, then (Q4_K) the slot's dmin * m offset.
template <int FMT, int NJ>
__device__ __forceinline__ void column_block(const uint8_t* tb, const uint4 (&pl)[TileFmt<FMT>::kPlanes],
                                             const uint32_t* xq, const float4* xsc, uint32_t G, uint32_t xg0,
                                             uint32_t nbatch, uint32_t g, uint32_t t, float (&cacc)[NJ][2][4]) {
  const uint32_t hl = g & 1u, bsel = g >> 1;
  if constexpr (FMT == kQ4K) {
    uint4 hdr[2];
    float d[2], dmin[2];
#pragma unroll
    for (uint32_t hr = 0; hr < 2u; ++hr) {
      hdr[hr] = *reinterpret_cast<const uint4*>(tb + TileFmt<FMT>::kScaleAt + (g + 8u * hr) * 16u);
      d[hr] = half_bits_to_float(hdr[hr].x & 0xffffu);
      dmin[hr] = half_bits_to_float(hdr[hr].x >> 16);
    }
    float dmm[8][2];
#pragma unroll
    for (uint32_t grp = 0; grp < 8u; ++grp) {
      float dsc[2];
#pragma unroll
      for (uint32_t hr = 0; hr < 2u; ++hr) {
        const uint4 h = hdr[hr];
        uint32_t sc, mn;
        if (grp < 4u) {
          sc = (h.y >> (8u * grp)) & 63u;
          mn = (h.z >> (8u * grp)) & 63u;
        } else {
          const uint32_t u = grp - 4u, e = (h.w >> (8u * u)) & 0xffu;
          sc = (e & 15u) | (((h.y >> (8u * u + 6u)) & 3u) << 4);
          mn = (e >> 4) | (((h.z >> (8u * u + 6u)) & 3u) << 4);
        }
        dsc[hr] = __fmul_rn(d[hr], static_cast<float>(sc));
        dmm[grp][hr] = __fmul_rn(dmin[hr], static_cast<float>(mn));
      }
      const uint4 w = pl[grp / 2u];
      const uint32_t sh = 4u * (grp % 2u);
      const uint32_t a0 = (w.x >> sh) & 0x0f0f0f0fu, a1 = (w.y >> sh) & 0x0f0f0f0fu;
      const uint32_t a2 = (w.z >> sh) & 0x0f0f0f0fu, a3 = (w.w >> sh) & 0x0f0f0f0fu;
      const uint32_t xg = xg0 + grp;
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        if (4u * j >= nbatch) break;
        const uint32_t bb = 4u * j + bsel, bm = 4u * j + t;
        uint32_t b0 = 0u, b1 = 0u;
        if (bb < nbatch) {
          const uint32_t* xw = xq + (static_cast<size_t>(bb) * G + xg) * 16u;
          b0 = xw[hl * 4u + t];
          b1 = xw[8u + hl * 4u + t];
        }
        int c[4] = {0, 0, 0, 0};
        mma_u8s8_k32(c, a0, a1, a2, a3, b0, b1);
        const float xs = bm < nbatch ? xsc[static_cast<size_t>(bm) * G + xg].x : 0.f;
        cacc[j][0][grp & 3u] =
            fmaf(__fmul_rn(dsc[0], xs), static_cast<float>(c[0] * 256 + c[1]), cacc[j][0][grp & 3u]);
        cacc[j][1][grp & 3u] =
            fmaf(__fmul_rn(dsc[1], xs), static_cast<float>(c[2] * 256 + c[3]), cacc[j][1][grp & 3u]);
      }
    }
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const uint32_t bm = 4u * j + t;
      if (4u * j >= nbatch) break;
#pragma unroll
      for (uint32_t q = 0; q < 4u; ++q) {
        const float aux0 = bm < nbatch ? xsc[static_cast<size_t>(bm) * G + xg0 + q].w : 0.f;
        const float aux1 = bm < nbatch ? xsc[static_cast<size_t>(bm) * G + xg0 + 4u + q].w : 0.f;
#pragma unroll
        for (uint32_t hr = 0; hr < 2u; ++hr)
          cacc[j][hr][q] -= fmaf(dmm[4u + q][hr], aux1, __fmul_rn(dmm[q][hr], aux0));
      }
    }
  } else {
    const uint4 sc4[2] = {*reinterpret_cast<const uint4*>(tb + TileFmt<FMT>::kScaleAt + g * 16u),
                          *reinterpret_cast<const uint4*>(tb + TileFmt<FMT>::kScaleAt + (g + 8u) * 16u)};
    const uint16_t* dp = reinterpret_cast<const uint16_t*>(tb + TileFmt<FMT>::kDAt);
    const float dr[2] = {half_bits_to_float(dp[g]), half_bits_to_float(dp[g + 8u])};
    const uint32_t w[24] = {pl[0].x, pl[0].y, pl[0].z, pl[0].w, pl[1].x, pl[1].y, pl[1].z, pl[1].w,
                            pl[2].x, pl[2].y, pl[2].z, pl[2].w, pl[3].x, pl[3].y, pl[3].z, pl[3].w,
                            pl[4].x, pl[4].y, pl[4].z, pl[4].w, pl[5].x, pl[5].y, pl[5].z, pl[5].w};
#pragma unroll
    for (uint32_t jc = 0; jc < 8u; ++jc) {  // 32-coefficient chunk = groups 2jc, 2jc + 1
      const uint32_t L0 = w[3u * jc], L1 = w[3u * jc + 1u], Hh = w[3u * jc + 2u];
      const uint32_t a[4] = {(L0 & 0x0f0f0f0fu) | ((Hh << 4) & 0x30303030u),
                             ((L0 >> 4) & 0x0f0f0f0fu) | ((Hh << 2) & 0x30303030u),
                             (L1 & 0x0f0f0f0fu) | (Hh & 0x30303030u),
                             ((L1 >> 4) & 0x0f0f0f0fu) | ((Hh >> 2) & 0x30303030u)};
      const uint32_t xg = xg0 + jc;
#pragma unroll
      for (uint32_t h2 = 0; h2 < 2u; ++h2) {
        const uint32_t grp = 2u * jc + h2;
        float dsc[2];
#pragma unroll
        for (uint32_t hr = 0; hr < 2u; ++hr) {
          const uint32_t word = grp / 4u == 0u ? sc4[hr].x : grp / 4u == 1u ? sc4[hr].y
                                : grp / 4u == 2u ? sc4[hr].z : sc4[hr].w;
          const int sc = static_cast<int8_t>((word >> (8u * (grp % 4u))) & 0xffu);
          dsc[hr] = __fmul_rn(dr[hr], static_cast<float>(sc));
        }
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          if (4u * j >= nbatch) break;
          const uint32_t bb = 4u * j + bsel, bm = 4u * j + t;
          const uint32_t b0 =
              bb < nbatch ? xq[(static_cast<size_t>(bb) * G + xg) * 16u + h2 * 8u + hl * 4u + t] : 0u;
          const float4 xv = bm < nbatch ? xsc[static_cast<size_t>(bm) * G + xg] : make_float4(0.f, 0.f, 0.f, 0.f);
          // the L column starts at -32 * sum X of the 16-group (the batch-1 seed)
          const int off = __float_as_int(h2 ? xv.z : xv.y);
          int c[4] = {0, off, 0, off};
          mma_u8s8_k16(c, a[2u * h2], a[2u * h2 + 1u], b0);
          cacc[j][0][grp & 3u] =
              fmaf(__fmul_rn(dsc[0], xv.x), static_cast<float>(c[0] * 256 + c[1]), cacc[j][0][grp & 3u]);
          cacc[j][1][grp & 3u] =
              fmaf(__fmul_rn(dsc[1], xv.x), static_cast<float>(c[2] * 256 + c[3]), cacc[j][1][grp & 3u]);
        }
      }
    }
  }
}

// NB <= 2: the lanes' MMA columns carry groups (four groups chained per
// accumulator, the batch-1 layout).  NB >= 4: the columns carry four batch
// rows each (H, L per row), NJ = NB / 4 column sets per MMA step, so one MMA
// serves four rows; each lane keeps, per row, the four per-slot partial sums
// (slot = group % 4) that the batch-1 layout keeps in its four lanes, and
// combines them in the same order, so every row's bits equal the batch-1 result.
template <int FMT, int NB>
__global__ void __launch_bounds__(kThreads, NB >= 8 ? 1 : 2) gemv_tiled_kernel(const Params p) {
  constexpr bool kCols = NB >= 4;
  constexpr int NJ = kCols ? NB / 4 : 1;
  constexpr int NR = kCols ? 1 : NB;
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr uint32_t kTile = TileFmt<FMT>::kBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = static_cast<uint32_t>(lane) >> 2, t = static_cast<uint32_t>(lane) & 3u;
  const uint32_t tiles = p.rows / kTileRows;
  const uint32_t ipt = p.nmat * p.ks;  // stages per tile
  const uint32_t my_tiles = blockIdx.x < tiles ? (tiles - 1u - blockIdx.x) / gridDim.x + 1u : 0u;
  const uint32_t total = my_tiles * ipt;
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + p.off_misc + 64);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < p.nstage; ++s) mbar_init(&bars[s], 1);
    *abort_flag = 0u;
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t policy = evict_first_policy();

  StageCursor prod;  // producer position (thread 0 only); stages are issued in order
  auto issue = [&]() {
    const uint32_t s = prod.s, tile = blockIdx.x + prod.tile_local * gridDim.x;
    const uint32_t nb = min(static_cast<uint32_t>(kStageBlocks), p.kb_total - prod.kst * kStageBlocks);
    const uint32_t bytes = nb * kTile;
    const uint8_t* src = p.w[prod.mat] + (static_cast<size_t>(tile) * p.kb_total + prod.kst * kStageBlocks) * kTile;
    mbar_expect_tx(&bars[s], bytes);
    bulk_g2s_stream(smem + s * p.stage_bytes, src, bytes, &bars[s], policy);
    prod.next(p.nstage, p.ks, ipt);
  };

  uint32_t issued = min(total, p.nstage), drain_from = 0;  // tracked by every thread alike
  if (threadIdx.x == 0)
    for (uint32_t it = 0; it < issued; ++it) issue();

  // norm weights are constant: read them before waiting on the producer
  float4 wv[kPass];
#pragma unroll
  for (int i = 0; i < kPass; ++i) wv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (p.prologue == kRmsNorm || p.prologue == kHeadGate) {
    const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
#pragma unroll
    for (int i = 0; i < kPass; ++i)
      if (threadIdx.x + i * kThreads < p.cols / 4u) wv[i] = w4[threadIdx.x + i * kThreads];
  }

  pdl_wait();                 // activations (and residual target) are now visible
  pdl_launch_dependents();    // let the next kernel start streaming its weights
  XFirst xfirst;
  load_x_first(p, xfirst);
  // the residual rows of the first tile, read now so the epilogue does not wait on them
  float ypre = 0.f;
  if (p.epilogue == kAccumulate && my_tiles > 0u && threadIdx.x < kTileRows * p.batch)
    ypre = p.y[static_cast<size_t>(threadIdx.x / kTileRows) * p.y_stride + blockIdx.x * kTileRows +
               threadIdx.x % kTileRows];
  if (!any_running(p)) {
    if (threadIdx.x == 0)  // generation stopped: drain the stages in flight and leave
      for (uint32_t j = 0; j < issued; ++j) (void)mbar_wait(&bars[j % p.nstage], (j / p.nstage) & 1u, nullptr);
    return;
  }
  prepare_x(p, smem, wv, xfirst);

  const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem + p.off_xq);
  const float4* xsc = reinterpret_cast<const float4*>(smem + p.off_xsc);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  const uint32_t G = p.cols / 32u;
  const uint32_t redsz = kWarps * 2u * kTileRows * p.batch;  // one buffer (per parity)
  const uint32_t nbatch = p.batch;

  // Batch-1 launches over one k-stage (cols <= 2048) see the same block in
  // every stage of a warp: its activation terms are loaded once.
  const bool hoist = NB == 1 && p.ks == 1u;
  XTerms<FMT> xh;
  if (hoist && static_cast<uint32_t>(warp) < p.kb_total)  // warps past the last block never read x
    load_xterms<FMT>(xh, xq, xsc, static_cast<uint32_t>(warp) * 8u, g, t);

  float acc[NR][2], held[NR][2];
#pragma unroll
  for (int b = 0; b < NR; ++b) acc[b][0] = acc[b][1] = held[b][0] = held[b][1] = 0.f;
  float cacc[NJ][2][4], cheld[NJ][2][4];  // batch columns: [column set][row g / g+8][slot]
#pragma unroll
  for (int j = 0; j < NJ; ++j)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr)
#pragma unroll
      for (int q = 0; q < 4; ++q) cacc[j][hr][q] = cheld[j][hr][q] = 0.f;

  unsigned long long best = 0ull;  // epilogue thread's running argmax key
  bool aborted = false;
  StageCursor cons;

  for (uint32_t it = 0; it < total; ++it, cons.next(p.nstage, p.ks, ipt)) {
    const uint32_t s = cons.s, tile_local = cons.tile_local, r = cons.r, kst = cons.kst;
    const uint32_t tile = blockIdx.x + tile_local * gridDim.x;
    if (!mbar_wait(&bars[s], cons.parity, p.err)) *abort_flag = 1u;
    const bool ok = *abort_flag == 0u;
    const uint32_t nb = min(static_cast<uint32_t>(kStageBlocks), p.kb_total - kst * kStageBlocks);
    const uint32_t kb = static_cast<uint32_t>(warp);

    if (ok && kb < nb) {
      const uint8_t* tb = smem + s * p.stage_bytes + kb * kTile;
      const uint32_t xg0 = (kst * kStageBlocks + kb) * 8u;  // first x-group of this block
      uint4 pl[TileFmt<FMT>::kPlanes];
#pragma unroll
      for (uint32_t i = 0; i < TileFmt<FMT>::kPlanes; ++i)
        pl[i] = *reinterpret_cast<const uint4*>(tb + i * 512u + static_cast<uint32_t>(lane) * 16u);
      if constexpr (kCols) {
        column_block<FMT, NJ>(tb, pl, xq, xsc, G, xg0, nbatch, g, t, cacc);
      } else {
      uint32_t a[8][4];  // A fragments of the 8 mma steps
      // per-chain scale factors of rows g and g+8 (before the activation scale)
      float dsc[FMT == kQ4K ? 2 : 4][2];
      float dmm[2][2];  // Q4_K: dmin * m for the lane's two groups
      if constexpr (FMT == kQ4K) {
#pragma unroll
        for (uint32_t q = 0; q < 4u; ++q) {
          const uint32_t w[4] = {pl[q].x, pl[q].y, pl[q].z, pl[q].w};
#pragma unroll
          for (uint32_t i = 0; i < 4u; ++i) {
            a[2u * q][i] = w[i] & 0x0f0f0f0fu;
            a[2u * q + 1u][i] = (w[i] >> 4) & 0x0f0f0f0fu;
          }
        }
#pragma unroll
        for (uint32_t hr = 0; hr < 2u; ++hr) {
          const uint4 h = *reinterpret_cast<const uint4*>(tb + TileFmt<FMT>::kScaleAt + (g + 8u * hr) * 16u);
          const float d = half_bits_to_float(h.x & 0xffffu), dmin = half_bits_to_float(h.x >> 16);
          const uint32_t sh = 8u * t, ys = h.y >> sh, zs = h.z >> sh, e = (h.w >> sh) & 0xffu;
          const uint32_t sc0 = ys & 63u, mn0 = zs & 63u;                              // group t
          const uint32_t sc1 = (e & 15u) | (((ys >> 6) & 3u) << 4);                   // group 4 + t
          const uint32_t mn1 = (e >> 4) | (((zs >> 6) & 3u) << 4);
          dsc[0][hr] = __fmul_rn(d, static_cast<float>(sc0));
          dsc[1][hr] = __fmul_rn(d, static_cast<float>(sc1));
          dmm[0][hr] = __fmul_rn(dmin, static_cast<float>(mn0));
          dmm[1][hr] = __fmul_rn(dmin, static_cast<float>(mn1));
        }
      } else {
        const uint32_t w[24] = {pl[0].x, pl[0].y, pl[0].z, pl[0].w, pl[1].x, pl[1].y, pl[1].z, pl[1].w,
                                pl[2].x, pl[2].y, pl[2].z, pl[2].w, pl[3].x, pl[3].y, pl[3].z, pl[3].w,
                                pl[4].x, pl[4].y, pl[4].z, pl[4].w, pl[5].x, pl[5].y, pl[5].z, pl[5].w};
#pragma unroll
        for (uint32_t j = 0; j < 8u; ++j) {
          const uint32_t L0 = w[3u * j], L1 = w[3u * j + 1u], Hh = w[3u * j + 2u];
          a[j][0] = (L0 & 0x0f0f0f0fu) | ((Hh << 4) & 0x30303030u);
          a[j][1] = ((L0 >> 4) & 0x0f0f0f0fu) | ((Hh << 2) & 0x30303030u);
          a[j][2] = (L1 & 0x0f0f0f0fu) | (Hh & 0x30303030u);
          a[j][3] = ((L1 >> 4) & 0x0f0f0f0fu) | ((Hh >> 2) & 0x30303030u);
        }
        const uint16_t* dp = reinterpret_cast<const uint16_t*>(tb + TileFmt<FMT>::kDAt);
        const float d0 = half_bits_to_float(dp[g]), d1 = half_bits_to_float(dp[g + 8u]);
#pragma unroll
        for (uint32_t hr = 0; hr < 2u; ++hr) {
          const uint4 h = *reinterpret_cast<const uint4*>(tb + TileFmt<FMT>::kScaleAt + (g + 8u * hr) * 16u);
          const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
#pragma unroll
          for (uint32_t u = 0; u < 4u; ++u) {  // group 4u + t
            const int sc = static_cast<int8_t>((hw[u] >> (8u * t)) & 0xffu);
            dsc[u][hr] = __fmul_rn(hr ? d1 : d0, static_cast<float>(sc));
          }
        }
      }

#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (static_cast<uint32_t>(b) >= nbatch) break;
        XTerms<FMT> x;
        if (hoist) x = xh;
        else load_xterms<FMT>(x, xq + static_cast<size_t>(b) * G * 16u, xsc + static_cast<size_t>(b) * G, xg0, g, t);
        if constexpr (FMT == kQ4K) {
#pragma unroll
          for (uint32_t u = 0; u < 2u; ++u) {  // chain u: groups 4u..4u+3, lane t ends with group 4u+t
            int c[4] = {0, 0, 0, 0};
#pragma unroll
            for (uint32_t q = 0; q < 4u; ++q) {
              const uint32_t grp = 4u * u + q;
              mma_u8s8_k32(c, a[grp][0], a[grp][1], a[grp][2], a[grp][3], x.b[grp][0], x.b[grp][1]);
            }
            acc[b][0] = fmaf(__fmul_rn(dsc[u][0], x.xs[u]), static_cast<float>(c[0] * 256 + c[1]), acc[b][0]);
            acc[b][1] = fmaf(__fmul_rn(dsc[u][1], x.xs[u]), static_cast<float>(c[2] * 256 + c[3]), acc[b][1]);
          }
#pragma unroll
          for (uint32_t hr = 0; hr < 2u; ++hr)
            acc[b][hr] -= fmaf(dmm[1][hr], x.aux[1], __fmul_rn(dmm[0][hr], x.aux[0]));
        } else {
#pragma unroll
          for (uint32_t u = 0; u < 4u; ++u) {  // chain u: chunks 2u, 2u+1, lane t ends with group 4u+t
            // the L column starts at -32 * sum X of the lane's 16-group: the
            // integer is sum((q - 32) * X), |.| < 2^24, exact in fp32
            const int off = __float_as_int(x.aux[u]);
            int c[4] = {0, off, 0, off};
            mma_u8s8_k32(c, a[2u * u][0], a[2u * u][1], a[2u * u][2], a[2u * u][3], x.b[2u * u][0], x.b[2u * u][1]);
            mma_u8s8_k32(c, a[2u * u + 1u][0], a[2u * u + 1u][1], a[2u * u + 1u][2], a[2u * u + 1u][3],
                         x.b[2u * u + 1u][0], x.b[2u * u + 1u][1]);
            acc[b][0] = fmaf(__fmul_rn(dsc[u][0], x.xs[u]), static_cast<float>(c[0] * 256 + c[1]), acc[b][0]);
            acc[b][1] = fmaf(__fmul_rn(dsc[u][1], x.xs[u]), static_cast<float>(c[2] * 256 + c[3]), acc[b][1]);
          }
        }
      }
      }  // lane-group layout
    }

    const bool tile_end = (r == ipt - 1u);
    float* redbuf = red + (tile_local & 1u) * redsz;
    if (p.nmat == 2u && kst == p.ks - 1u && cons.mat == 0u) {  // matrix 0 of the tile is complete
#pragma unroll
      for (int b = 0; b < NR; ++b) {
        held[b][0] = acc[b][0];
        held[b][1] = acc[b][1];
        acc[b][0] = acc[b][1] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr)
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            cheld[j][hr][q] = cacc[j][hr][q];
            cacc[j][hr][q] = 0.f;
          }
    }
    if (tile_end && kCols) {
      // lane t holds rows g, g+8 of batch rows 4j + t, four slots each: (s0 + s1) + (s2 + s3)
      auto publish_cols = [&](int m, float (&v)[NJ][2][4]) {
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
          const uint32_t bm = 4u * j + t;
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const float s2 = (v[j][hr][0] + v[j][hr][1]) + (v[j][hr][2] + v[j][hr][3]);
            if (bm < nbatch) redbuf[((warp * 2 + m) * kTileRows + g + 8u * hr) * nbatch + bm] = s2;
#pragma unroll
            for (int q = 0; q < 4; ++q) v[j][hr][q] = 0.f;
          }
        }
      };
      if (p.nmat == 2u) {
        publish_cols(0, cheld);
        publish_cols(1, cacc);
      } else {
        publish_cols(0, cacc);
      }
    } else if (tile_end) {
      // the four lanes of a row hold disjoint groups: (t0 + t1) + (t2 + t3)
      auto publish = [&](int m, float (&v)[NR][2]) {
#pragma unroll
        for (int b = 0; b < NR; ++b) {
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            float s2 = v[b][hr] + __shfl_xor_sync(0xffffffffu, v[b][hr], 1);
            s2 = s2 + __shfl_xor_sync(0xffffffffu, s2, 2);
            if (t == 0u && static_cast<uint32_t>(b) < nbatch)
              redbuf[((warp * 2 + m) * kTileRows + g + 8u * hr) * nbatch + b] = s2;
            v[b][hr] = 0.f;
          }
        }
      };
      if (p.nmat == 2u) {
        publish(0, held);
        publish(1, acc);
      } else {
        publish(0, acc);
      }
    }
    __syncthreads();  // stage s consumed; reduction buffer visible
    if (*abort_flag) {
      aborted = true;
      drain_from = it;
      break;
    }
    if (it + p.nstage < total) {
      if (threadIdx.x == 0) issue();
      issued = it + p.nstage + 1u;
    }
    if (tile_end)
      for (uint32_t idx = threadIdx.x; idx < kTileRows * nbatch; idx += kThreads) {
        const uint32_t row = idx % kTileRows, b = idx / kTileRows;
        float v[2] = {0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (static_cast<uint32_t>(m) >= p.nmat) break;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) v[m] += redbuf[((w * 2 + m) * kTileRows + row) * nbatch + b];
        }
        const uint32_t R = tile * kTileRows + row;
        if (p.running && p.running[b * p.run_step] == 0u) continue;  // this batch row has stopped
        float* yp = p.y ? p.y + static_cast<size_t>(b) * p.y_stride + R : nullptr;
        if (p.epilogue == kSwiGLU) {
          const float gv = v[0], uv = v[1];
          const float amp = fabsf(gv) * fabsf(uv) * detector_sigmoid(gv);
          const float sgn = (gv > 0.f ? 1.f : gv < 0.f ? -1.f : 0.f) * (uv > 0.f ? 1.f : uv < 0.f ? -1.f : 0.f);
          *yp = sgn * amp;
        } else if (p.epilogue == kAccumulate) {
          *yp = (tile_local == 0u ? ypre : *yp) + v[0];
        } else if (yp) {
          *yp = v[0];
        }
        if (p.argmax) {
          const unsigned long long key = pack_argmax(v[0], R);
          best = key > best ? key : best;
        }
      }
  }

  if (aborted) {
    // Bounded drain of the copies this CTA still has in flight, so no bulk
    // copy lands in shared memory after the CTA has exited.
    if (threadIdx.x == 0)
      for (uint32_t j = drain_from; j < issued; ++j) (void)mbar_wait(&bars[j % p.nstage], (j / p.nstage) & 1u, nullptr);
    return;
  }
  if (p.argmax) {
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(smem + p.off_red);
    __syncthreads();
    cand[threadIdx.x] = threadIdx.x < kTileRows * nbatch ? best : 0ull;
    __syncthreads();
    if (threadIdx.x < nbatch) {
      unsigned long long m = 0ull;
      for (uint32_t row = 0; row < kTileRows; ++row) {
        const unsigned long long c = cand[threadIdx.x * kTileRows + row];
        m = c > m ? c : m;
      }
      if (m) atomicMax(p.argmax + static_cast<size_t>(threadIdx.x) * p.arg_step, m);
    }
  }
}

// -------------------------------------------------------------- F32 GEMV
__global__ void gemv_f32_kernel(const float* __restrict__ W, uint32_t rows, uint32_t cols,
                                const float* __restrict__ x, uint32_t x_stride, uint32_t batch, float* __restrict__ y,
                                uint32_t y_stride) {
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
  if (warp >= rows * batch) return;
  const uint32_t r = warp % rows, b = warp / rows;
  float s = 0.f;
  for (uint32_t c = lane; c < cols; c += 32u) s += W[static_cast<size_t>(r) * cols + c] * x[b * x_stride + c];
  s = warp_sum(s);
  if (lane == 0) y[b * y_stride + r] = s;
}

template <int FMT, bool TILED = false>
uint32_t smem_bytes(uint32_t cols, uint32_t batch, Params* p) {
  const uint32_t G = cols / 32u;
  uint32_t off = 0;
  auto carve = [&](uint32_t sz, uint32_t align) {
    off = (off + align - 1) / align * align;
    const uint32_t at = off;
    off += sz;
    return at;
  };
  // batch launches spend shared memory on the activation tables instead of stages
  const uint32_t nstage = TILED && batch >= 4u ? 2u : FMT == kQ4K ? 4u : 3u;
  const uint32_t stage_bytes =
      TILED ? kStageBlocks * TileFmt<FMT>::kBytes : kTileRows * (kStageBlocks * Fmt<FMT>::kBytes + Fmt<FMT>::kPad);
  carve(nstage * stage_bytes, 128);
  const uint32_t off_bar = carve(8 * nstage, 8);
  const uint32_t off_xq = carve(batch * G * 64, 16);
  const uint32_t off_xsc = carve(batch * G * 16, 16);
  const uint32_t off_scr = TILED ? off_xsc : carve(kWarps * kScrFloats * 4, 16);
  const uint32_t red_floats = 2 * kWarps * 2 * kTileRows * batch;
  const uint32_t off_red = carve(max(red_floats * 4u, static_cast<uint32_t>(kThreads * 8)), 16);
  const uint32_t off_misc = carve(128, 16);
  if (p) {
    p->nstage = nstage;
    p->stage_bytes = stage_bytes;
    p->row_pad = TILED ? 0u : Fmt<FMT>::kPad;
    p->off_bar = off_bar;
    p->off_xq = off_xq;
    p->off_xsc = off_xsc;
    p->off_scr = off_scr;
    p->off_red = off_red;
    p->off_misc = off_misc;
  }
  return off;
}

template <int FMT, int NB, bool TILED>
cudaError_t launch_t(const GemvArgs& a, Params p, cudaStream_t s) {
  void (*kernel)(const Params);
  if constexpr (TILED) kernel = gemv_tiled_kernel<FMT, NB>;
  else kernel = gemv_kernel<FMT, NB>;
  const uint32_t smem = smem_bytes<FMT, TILED>(a.cols, p.batch, &p);
  // One-time kernel setup and occupancy per (kernel instance, smem size): these
  // queries cost microseconds and must stay off the per-launch path
  // (function attributes are per device: index the flags by device ordinal).
  // Host threads may make their first calls at the same time: the setup and
  // the cache fills run under a lock, and each entry is published with release
  // order (an SM count, or an occupancy after its shared-memory size), so the
  // lock-free reads never see half an entry.
  static std::mutex setup_mutex;
  static std::atomic<int> sms_of[64];
  static std::atomic<uint32_t> cached_smem[8];
  static std::atomic<int> cached_grid[8];
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
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      if (sms <= 0) return cudaErrorInvalidDevice;
      sms_of[dev].store(sms, std::memory_order_release);
    }
  }
  if (smem > 227u * 1024u) return cudaErrorInvalidConfiguration;
  int per_sm = 0;
  for (int i = 0; i < 8; ++i)
    if (cached_smem[i].load(std::memory_order_acquire) == smem) per_sm = cached_grid[i].load(std::memory_order_relaxed);
  if (per_sm == 0) {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    std::lock_guard<std::mutex> lock(setup_mutex);
    bool held = false;
    for (int i = 0; i < 8 && !held; ++i) held = cached_smem[i].load(std::memory_order_relaxed) == smem;
    for (int i = 0; i < 8 && !held; ++i)
      if (cached_smem[i].load(std::memory_order_relaxed) == 0) {
        cached_grid[i].store(per_sm, std::memory_order_relaxed);
        cached_smem[i].store(smem, std::memory_order_release);
        held = true;
      }
  }
  const uint32_t tiles = a.rows / kTileRows;
  const uint32_t grid = min(tiles, static_cast<uint32_t>(per_sm * sms));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int FMT, bool TILED>
cudaError_t launch_fmt(const GemvArgs& a, Params p, cudaStream_t s) {
  if (p.batch == 1) return launch_t<FMT, 1, TILED>(a, p, s);
  if (p.batch == 2) return launch_t<FMT, 2, TILED>(a, p, s);
  if (p.batch <= 4) return launch_t<FMT, 4, TILED>(a, p, s);
  if constexpr (TILED)
    if (p.batch > 8) return launch_t<FMT, 16, TILED>(a, p, s);
  return launch_t<FMT, 8, TILED>(a, p, s);
}

template <int FMT, bool TILED>
uint32_t smem_for(uint32_t cols, uint32_t nb) {
  return smem_bytes<FMT, TILED>(cols, nb, nullptr);
}

}  // namespace

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (dense_format(a.fmt)) return launch_gemv_dense(a, s);
  const bool tiled = a.fmt == kQ4KTiled || a.fmt == kQ6KTiled;
  const int fmt = tiled ? a.fmt - kTiledOffset : a.fmt;
  if ((fmt != kQ4K && fmt != kQ6K) || !a.w0 || !a.x || a.rows == 0 || a.rows % kTileRows ||
      a.cols == 0 || a.cols % 256 || a.cols > 4u * kThreads * kMaxChunks || a.batch == 0 || a.batch > kMaxBatch)
    return cudaErrorInvalidValue;
  if (a.epilogue == kSwiGLU && !a.w1) return cudaErrorInvalidValue;
  if (a.epilogue != kSwiGLU && a.w1) return cudaErrorInvalidValue;
  if (!a.y && !a.argmax) return cudaErrorInvalidValue;
  if ((a.prologue == kHeadGate || a.prologue == kSigmoidGate) && !a.z) return cudaErrorInvalidValue;
  if ((a.prologue == kRmsNorm || a.prologue == kHeadGate) && !a.norm_w) return cudaErrorInvalidValue;
  if (a.prologue == kHeadGate && a.cols % 128) return cudaErrorInvalidValue;
  if ((a.prologue == kRmsNorm || a.prologue == kHeadGate) && a.cols > 4u * kThreads * kPass)
    return cudaErrorInvalidValue;  // normed inputs are held in registers in one pass
  const uint32_t row_bytes = a.cols / 256 * block_bytes(fmt);
  const uint32_t x_stride = a.x_stride ? a.x_stride : a.cols;
  if ((!tiled && row_bytes % 16) || reinterpret_cast<uintptr_t>(a.w0) % 16 || reinterpret_cast<uintptr_t>(a.w1) % 16 ||
      reinterpret_cast<uintptr_t>(a.x) % 16 || reinterpret_cast<uintptr_t>(a.z) % 16 ||
      reinterpret_cast<uintptr_t>(a.norm_w) % 16 || x_stride % 4 || a.z_stride % 4)
    return cudaErrorMisalignedAddress;  // rows, activations and norm weights are read as 16-byte vectors
  Params p = {};
  p.w[0] = a.w0;
  p.w[1] = a.w1;
  p.nmat = a.w1 ? 2u : 1u;
  p.rows = a.rows;
  p.cols = a.cols;
  p.kb_total = a.cols / 256;
  p.row_bytes = row_bytes;
  p.ks = (p.kb_total + kStageBlocks - 1) / kStageBlocks;
  p.x = a.x;
  p.x_stride = x_stride;
  p.batch = a.batch;
  p.prologue = a.prologue;
  p.norm_w = a.norm_w;
  p.eps = a.eps;
  p.z = a.z;
  p.z_stride = a.z_stride ? a.z_stride : x_stride;
  p.epilogue = a.epilogue;
  p.y = a.y;
  p.y_stride = a.y_stride ? a.y_stride : a.rows;
  p.argmax = a.argmax;
  p.err = a.err;
  p.running = a.running;
  p.run_step = a.running_step ? a.running_step : 1u;
  p.arg_step = a.argmax_step ? a.argmax_step : 1u;
  // Batch rows run in launches of at most 8 rows (each launch streams the
  // weights once); a launch's activation tables must fit in shared memory.
  for (uint32_t b0 = 0; b0 < a.batch;) {
    uint32_t nb = min(tiled ? 16u : 8u, a.batch - b0);
    auto smem = [&](uint32_t n) {
      return tiled ? (fmt == kQ4K ? smem_for<kQ4K, true>(a.cols, n) : smem_for<kQ6K, true>(a.cols, n))
                   : (fmt == kQ4K ? smem_for<kQ4K, false>(a.cols, n) : smem_for<kQ6K, false>(a.cols, n));
    };
    while (nb > 1 && smem(nb) > 227u * 1024u) nb /= 2;
    Params q = p;
    q.batch = nb;
    q.x = a.x + static_cast<size_t>(b0) * x_stride;
    q.z = a.z ? a.z + static_cast<size_t>(b0) * p.z_stride : nullptr;
    q.y = a.y ? a.y + static_cast<size_t>(b0) * p.y_stride : nullptr;
    q.argmax = a.argmax ? a.argmax + static_cast<size_t>(b0) * p.arg_step : nullptr;
    q.running = a.running ? a.running + static_cast<size_t>(b0) * p.run_step : nullptr;
    const cudaError_t e = tiled ? (fmt == kQ4K ? launch_fmt<kQ4K, true>(a, q, s) : launch_fmt<kQ6K, true>(a, q, s))
                                : (fmt == kQ4K ? launch_fmt<kQ4K, false>(a, q, s) : launch_fmt<kQ6K, false>(a, q, s));
    if (e != cudaSuccess) return e;
    b0 += nb;
  }
  return cudaSuccess;
}

cudaError_t launch_gemv_f32(const float* W, uint32_t rows, uint32_t cols, const float* x, uint32_t x_stride,
                            uint32_t batch, float* y, uint32_t y_stride, cudaStream_t s) {
  const uint32_t warps = rows * batch;
  gemv_f32_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>(W, rows, cols, x, x_stride ? x_stride : cols, batch, y,
                                                             y_stride ? y_stride : rows);
  return cudaGetLastError();
}

cudaError_t launch_tile_weights(int fmt, const uint8_t* src, uint32_t rows, uint32_t cols, uint8_t* dst,
                                cudaStream_t s) {
  if ((fmt != kQ4K && fmt != kQ6K) || !src || !dst || rows == 0 || rows % kTileRows || cols == 0 || cols % 256)
    return cudaErrorInvalidValue;
  if (src == dst) return cudaErrorInvalidValue;  // not in place
  const dim3 grid(cols / 256, rows / kTileRows);
  if (fmt == kQ4K) tile_weights_kernel<kQ4K><<<grid, 256, 0, s>>>(src, cols / 256, dst);
  else tile_weights_kernel<kQ6K><<<grid, 256, 0, s>>>(src, cols / 256, dst);
  return cudaGetLastError();
}

}  // namespace rta
