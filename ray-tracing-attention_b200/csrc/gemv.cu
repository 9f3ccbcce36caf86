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
//    cp.async.bulk per row, NSTAGE stages in flight per CTA, mbarrier
//    completion with bounded waits.  Under programmatic dependent launch the
//    first stages are issued before griddepcontrol.wait, so weight streaming
//    overlaps the tail of the kernel that produces x.
//  * Products are exact integers: the packed 4/6-bit codes are the u8 A
//    operand of mma.sync (m16n8k32 for a 32-wide Q4_K group, m16n8k16 for a
//    16-wide Q6_K group) and the activation is split per 32-group into
//    x ~= xs * (256*H + L) with H, L signed bytes (|X| <= 32639), the s8 B
//    operand (columns = (H, L) x 4 batch rows).  Group scales d*sc, the
//    dmin*m offset and the Q6_K -32 offset are applied in fp32 per group.
//    The activation split keeps |relative error| <= 1.5e-5 per element.
#include "rta_internal.h"

namespace rta {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = 4;
constexpr int kTileRows = 16;
constexpr int kStageBlocks = 8;
constexpr float kXLevels = 32639.0f;  // 127*256 + 127: keeps H in [-127, 127]

struct Params {
  const uint8_t* w[2];
  uint32_t nmat, rows, cols, kb_total, row_bytes;
  uint32_t ks;           // stages per matrix per tile
  uint32_t nstage;       // pipeline depth
  uint32_t stage_bytes;  // bytes of one stage buffer
  const float* x;
  uint32_t x_stride, batch, ncol;
  int prologue;
  const float* norm_w;
  float eps;
  const float* z;
  int epilogue;
  float* y;
  uint32_t y_stride;
  unsigned long long* argmax;
  uint32_t* err;
  const uint32_t* running;
  // shared-memory carve (byte offsets from the dynamic base)
  uint32_t off_bar, off_xq, off_xsc, off_scr, off_red, off_misc;
};

template <int FMT>
struct Fmt;
template <>
struct Fmt<kQ4K> {
  static constexpr uint32_t kBytes = 144;
};
template <>
struct Fmt<kQ6K> {
  static constexpr uint32_t kBytes = 210;
};

__device__ __forceinline__ float block_sum(float v, float* red4) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red4[w] = v;
  __syncthreads();
  return red4[0] + ((red4[1] + red4[2]) + red4[3]);
}

// Build the int16-split activation tables in shared memory.
//   xq  : [xgroup][slice][half][ncol][4 words]   (B fragments, zero padded)
//   xsc : [batch][xgroup] float4(xs, sum X first 16, sum X last 16, 0)
template <int NSL>
__device__ void prepare_x(const Params& p, uint8_t* smem) {
  uint32_t* xq = reinterpret_cast<uint32_t*>(smem + p.off_xq);
  float4* xsc = reinterpret_cast<float4*>(smem + p.off_xsc);
  float* misc = reinterpret_cast<float*>(smem + p.off_misc);
  const uint32_t G = p.cols / 32u;
  const uint32_t words = G * NSL * 2u * p.ncol * 4u;
  for (uint32_t i = threadIdx.x; i < words; i += kThreads) xq[i] = 0u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t b = 0; b < p.batch; ++b) {
    const float* xr = p.x + static_cast<size_t>(b) * p.x_stride;
    const float* zr = p.z ? p.z + static_cast<size_t>(b) * p.x_stride : nullptr;
    float inv = 1.f;
    if (p.prologue == kRmsNorm) {
      float s = 0.f;
      for (uint32_t c = threadIdx.x; c < p.cols; c += kThreads) s += xr[c] * xr[c];
      const float total = block_sum(s, misc);
      inv = rsqrtf(total / static_cast<float>(p.cols) + p.eps);
    }
    __syncthreads();  // xq zero-fill and misc reuse complete
    for (uint32_t g = warp; g < G; g += kWarps) {
      const uint32_t c = g * 32u + lane;
      float v = xr[c];
      if (p.prologue == kRmsNorm) {
        v = v * inv * p.norm_w[c];
      } else if (p.prologue == kHeadGate) {
        // per 128-wide head RMS: the 4 groups of a head are 4 consecutive g.
        const uint32_t head0 = (c / 128u) * 128u;
        float s = 0.f;
        for (uint32_t k = lane; k < 128u; k += 32u) s += xr[head0 + k] * xr[head0 + k];
        s = warp_sum(s);
        const float hinv = rsqrtf(s / 128.0f + p.eps);
        const float gz = zr[c];
        v = v * (((hinv * p.norm_w[c]) * gz) * detector_sigmoid(gz));
      } else if (p.prologue == kSigmoidGate) {
        v = v * detector_sigmoid(zr[c]);
      }
      const float amax = warp_max(fabsf(v));
      int X = 0;
      float xs = 0.f;
      if (amax > 0.f) {
        X = __float2int_rn(v * (kXLevels / amax));
        X = max(-32639, min(32639, X));
        xs = amax / kXLevels;
      }
      const int L = static_cast<int>(static_cast<int8_t>(X & 0xff));
      const int H = (X - L) >> 8;
      float sx = static_cast<float>(X);
#pragma unroll
      for (int m = 8; m >= 1; m >>= 1) sx += __shfl_xor_sync(0xffffffffu, sx, m);
      const float sx_other = __shfl_xor_sync(0xffffffffu, sx, 16);
      const uint32_t sl = b / 4u, colH = 2u * (b % 4u), half = static_cast<uint32_t>(lane) / 16u;
      const uint32_t t = (static_cast<uint32_t>(lane) % 16u) / 4u, byte = static_cast<uint32_t>(lane) % 4u;
      uint8_t* base = reinterpret_cast<uint8_t*>(xq + (((g * NSL + sl) * 2u + half) * p.ncol) * 4u);
      base[(colH * 4u + t) * 4u + byte] = static_cast<uint8_t>(H & 0xff);
      base[((colH + 1u) * 4u + t) * 4u + byte] = static_cast<uint8_t>(L & 0xff);
      if (lane == 0) xsc[b * G + g] = make_float4(xs, sx, sx_other, 0.f);
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

template <int FMT, int NSL>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t g = static_cast<uint32_t>(lane) >> 2, t = static_cast<uint32_t>(lane) & 3u;
  const uint32_t tiles = p.rows / kTileRows;
  const uint32_t ipt = p.nmat * p.ks;  // iterations (stages) per tile
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

  auto issue = [&](uint32_t it) {
    // warp 0 only
    const uint32_t s = it % p.nstage;
    const uint32_t tile = blockIdx.x + (it / ipt) * gridDim.x;
    const uint32_t r = it % ipt, mat = r / p.ks, kst = r % p.ks;
    const uint32_t nb = min(static_cast<uint32_t>(kStageBlocks), p.kb_total - kst * kStageBlocks);
    const uint32_t chunk = nb * Fmt<FMT>::kBytes;
    if (lane == 0) mbar_expect_tx(&bars[s], chunk * kTileRows);
    __syncwarp();
    if (lane < kTileRows)
      bulk_g2s_stream(smem + s * p.stage_bytes + lane * chunk, stage_src<FMT>(p, tile, mat, kst, lane), chunk,
                      &bars[s], policy);
  };

  uint32_t issued = min(total, p.nstage), drain_from = 0;  // tracked by every thread alike
  if (warp == 0)
    for (uint32_t it = 0; it < issued; ++it) issue(it);

  pdl_wait();                 // activations (and residual target) are now visible
  pdl_launch_dependents();    // let the next kernel start streaming its weights
  if (p.running && *p.running == 0u) {
    // generation stopped: drain the stages already in flight and leave
    if (threadIdx.x == 0)
      for (uint32_t j = 0; j < issued; ++j) (void)mbar_wait(&bars[j % p.nstage], (j / p.nstage) & 1u, nullptr);
    return;
  }
  prepare_x<NSL>(p, smem);

  const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem + p.off_xq);
  const float4* xsc = reinterpret_cast<const float4*>(smem + p.off_xsc);
  float* scr = reinterpret_cast<float*>(smem + p.off_scr) + warp * 512;
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  const uint32_t G = p.cols / 32u;
  const uint32_t redsz = kWarps * 2u * kTileRows * p.batch;  // one buffer (per parity)

  float acc[2][NSL][2];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int s = 0; s < NSL; ++s) acc[m][s][0] = acc[m][s][1] = 0.f;

  unsigned long long best = 0ull;  // epilogue thread's running argmax key
  bool aborted = false;

  for (uint32_t it = 0; it < total; ++it) {
    const uint32_t s = it % p.nstage, parity = (it / p.nstage) & 1u;
    const uint32_t tile_local = it / ipt, r = it % ipt, mat = r / p.ks, kst = r % p.ks;
    const uint32_t tile = blockIdx.x + tile_local * gridDim.x;
    if (!mbar_wait(&bars[s], parity, p.err)) *abort_flag = 1u;
    const bool ok = *abort_flag == 0u;
    const uint32_t nb = min(static_cast<uint32_t>(kStageBlocks), p.kb_total - kst * kStageBlocks);
    const uint32_t chunk = nb * Fmt<FMT>::kBytes;
    const uint8_t* stage = smem + s * p.stage_bytes;

    if (ok) {
      for (uint32_t kb = warp; kb < nb; kb += kWarps) {
        const uint32_t xg0 = (kst * kStageBlocks + kb) * 8u;  // first x-group of this block
        if constexpr (FMT == kQ4K) {
          // scales of the 16 rows x 8 groups of this block -> (d*sc, dmin*m)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t pair = lane + 32u * i, row = pair >> 3, grp = pair & 7u;
            const uint8_t* h = stage + row * chunk + kb * 144u;
            const float d = half_bits_to_float(h[0] | (h[1] << 8));
            const float dmin = half_bits_to_float(h[2] | (h[3] << 8));
            uint32_t sc, mn;
            if (grp < 4u) {
              sc = h[4 + grp] & 63u;
              mn = h[8 + grp] & 63u;
            } else {
              const uint32_t q = grp - 4u, mixed = h[12 + q];
              sc = (mixed & 15u) | ((static_cast<uint32_t>(h[4 + q]) >> 6) << 4);
              mn = (mixed >> 4) | ((static_cast<uint32_t>(h[8 + q]) >> 6) << 4);
            }
            scr[2 * pair] = d * static_cast<float>(sc);
            scr[2 * pair + 1] = dmin * static_cast<float>(mn);
          }
          __syncwarp();
          const uint8_t* rg = stage + g * chunk + kb * 144u + 16u;
          const uint8_t* rg8 = stage + (g + 8u) * chunk + kb * 144u + 16u;
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
              const float2 sA = *reinterpret_cast<const float2*>(scr + 2 * (g * 8u + grp));
              const float2 sB = *reinterpret_cast<const float2*>(scr + 2 * ((g + 8u) * 8u + grp));
#pragma unroll
              for (int sl = 0; sl < NSL; ++sl) {
                const uint32_t* xw = xq + ((xg * NSL + sl) * 2u) * p.ncol * 4u;
                uint32_t b0 = 0u, b1 = 0u;
                if (g < p.ncol) {
                  b0 = xw[g * 4u + t];
                  b1 = xw[p.ncol * 4u + g * 4u + t];
                }
                int c[4] = {0, 0, 0, 0};
                mma_u8s8_k32(c, a0, a1, a2, a3, b0, b1);
                const uint32_t b = 4u * sl + t;
                if (b < p.batch) {
                  const float4 xv = xsc[b * G + xg];
                  const float sx = xv.y + xv.z;
                  const float dot0 = static_cast<float>(c[0] * 256 + c[1]);
                  const float dot1 = static_cast<float>(c[2] * 256 + c[3]);
                  acc[mat][sl][0] += xv.x * (sA.x * dot0 - sA.y * sx);
                  acc[mat][sl][1] += xv.x * (sB.x * dot1 - sB.y * sx);
                }
              }
            }
          }
          __syncwarp();
        } else {
          // Q6_K: d * int8 scale per (row, 16-group)
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t pair = lane + 32u * i, row = pair >> 4, grp = pair & 15u;
            const uint8_t* bk = stage + row * chunk + kb * 210u;
            const float d = half_bits_to_float(bk[208] | (bk[209] << 8));
            scr[pair] = d * static_cast<float>(static_cast<int8_t>(bk[192 + grp]));
          }
          __syncwarp();
          const uint32_t rowg = g * chunk + kb * 210u, rowg8 = (g + 8u) * chunk + kb * 210u;
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
            for (uint32_t jj = 0; jj < 8u; ++jj) {
              const uint32_t grp = part * 8u + jj, ns = (jj / 4u) * 4u, hs = (jj / 2u) * 2u;
              const uint32_t a0 = ((ql[0][jj % 4u] >> ns) & 0x0f0f0f0fu) | (((qh[0][jj % 2u] >> hs) & 0x03030303u) << 4);
              const uint32_t a1 = ((ql[1][jj % 4u] >> ns) & 0x0f0f0f0fu) | (((qh[1][jj % 2u] >> hs) & 0x03030303u) << 4);
              const uint32_t xg = xg0 + grp / 2u, half = grp & 1u;
              const float dA = scr[g * 16u + grp], dB = scr[(g + 8u) * 16u + grp];
#pragma unroll
              for (int sl = 0; sl < NSL; ++sl) {
                const uint32_t* xw = xq + ((xg * NSL + sl) * 2u + half) * p.ncol * 4u;
                const uint32_t b0 = g < p.ncol ? xw[g * 4u + t] : 0u;
                int c[4] = {0, 0, 0, 0};
                mma_u8s8_k16(c, a0, a1, b0);
                const uint32_t b = 4u * sl + t;
                if (b < p.batch) {
                  const float4 xv = xsc[b * G + xg];
                  const float sx32 = 32.0f * (half ? xv.z : xv.y);
                  const float dot0 = static_cast<float>(c[0] * 256 + c[1]) - sx32;
                  const float dot1 = static_cast<float>(c[2] * 256 + c[3]) - sx32;
                  acc[mat][sl][0] += xv.x * (dA * dot0);
                  acc[mat][sl][1] += xv.x * (dB * dot1);
                }
              }
            }
          }
          __syncwarp();
        }
      }
    }

    const bool tile_end = (r == ipt - 1u);
    float* redbuf = red + (tile_local & 1u) * redsz;
    if (tile_end) {
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (static_cast<uint32_t>(m) >= p.nmat) break;
#pragma unroll
        for (int sl = 0; sl < NSL; ++sl) {
          const uint32_t b = 4u * sl + t;
          if (b < p.batch) {
            redbuf[((warp * 2 + m) * kTileRows + g) * p.batch + b] = acc[m][sl][0];
            redbuf[((warp * 2 + m) * kTileRows + g + 8u) * p.batch + b] = acc[m][sl][1];
          }
          acc[m][sl][0] = acc[m][sl][1] = 0.f;
        }
      }
    }
    __syncthreads();  // stage s consumed; reduction buffer visible
    if (*abort_flag) {
      aborted = true;
      drain_from = it;
      break;
    }
    if (it + p.nstage < total) {
      if (warp == 0) issue(it + p.nstage);
      issued = it + p.nstage + 1u;
    }
    if (tile_end)
    for (uint32_t idx = threadIdx.x; idx < kTileRows * p.batch; idx += kThreads) {
      const uint32_t row = idx % kTileRows, b = idx / kTileRows;
      float v[2] = {0.f, 0.f};
      for (uint32_t m = 0; m < p.nmat; ++m)
        for (int w = 0; w < kWarps; ++w) v[m] += redbuf[((w * 2 + m) * kTileRows + row) * p.batch + b];
      const uint32_t R = tile * kTileRows + row;
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
    cand[threadIdx.x] = threadIdx.x < kTileRows * p.batch ? best : 0ull;
    __syncthreads();
    if (threadIdx.x < p.batch) {
      unsigned long long m = 0ull;
      for (uint32_t row = 0; row < kTileRows; ++row) {
        const unsigned long long c = cand[threadIdx.x * kTileRows + row];
        m = c > m ? c : m;
      }
      if (m) atomicMax(p.argmax + threadIdx.x, m);
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

template <int FMT, int NSL>
cudaError_t launch_t(const GemvArgs& a, Params p, cudaStream_t s) {
  auto kernel = gemv_kernel<FMT, NSL>;
  const uint32_t bytes = Fmt<FMT>::kBytes;
  p.stage_bytes = kTileRows * kStageBlocks * bytes;
  p.nstage = 4;
  p.ncol = (a.batch == 1u && NSL == 1) ? 2u : 8u;
  const uint32_t G = a.cols / 32u;
  uint32_t off = 0;
  auto carve = [&](uint32_t sz, uint32_t align) {
    off = (off + align - 1) / align * align;
    const uint32_t at = off;
    off += sz;
    return at;
  };
  const uint32_t off_stage = carve(p.nstage * p.stage_bytes, 128);
  (void)off_stage;
  p.off_bar = carve(8 * p.nstage, 8);
  p.off_xq = carve(G * NSL * 2 * p.ncol * 16, 16);
  p.off_xsc = carve(a.batch * G * 16, 16);
  p.off_scr = carve(kWarps * 512 * 4, 16);
  const uint32_t red_floats = 2 * kWarps * 2 * kTileRows * a.batch;
  p.off_red = carve(max(red_floats * 4u, static_cast<uint32_t>(kThreads * 8)), 16);
  p.off_misc = carve(128, 16);
  const uint32_t smem = off;
  // One-time kernel setup and occupancy per (kernel instance, smem size): these
  // queries cost microseconds and must stay off the per-launch path.
  // (function attributes are per device: index the cache by device ordinal)
  static int max_smem_set[64] = {0};
  static uint32_t cached_smem[8] = {0};
  static int cached_grid[8] = {0};
  static int sms = 0;
  cudaError_t e = cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!max_smem_set[dev]) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    max_smem_set[dev] = 1;
  }
  if (smem > 227u * 1024u) return cudaErrorInvalidConfiguration;
  int per_sm = 0;
  for (int i = 0; i < 8; ++i)
    if (cached_smem[i] == smem) per_sm = cached_grid[i];
  if (per_sm == 0) {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    for (int i = 0; i < 8; ++i)
      if (cached_smem[i] == 0) {
        cached_smem[i] = smem;
        cached_grid[i] = per_sm;
        break;
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

}  // namespace

cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t s) {
  if ((a.fmt != kQ4K && a.fmt != kQ6K) || !a.w0 || !a.x || a.rows == 0 || a.rows % kTileRows ||
      a.cols == 0 || a.cols % 256 || a.batch == 0 || a.batch > kMaxBatch)
    return cudaErrorInvalidValue;
  if (a.fmt == kQ6K && (a.cols / 256) % kStageBlocks && a.cols / 256 > static_cast<uint32_t>(kStageBlocks))
    return cudaErrorInvalidValue;  // Q6_K row chunks must stay 16-byte aligned
  if (a.epilogue == kSwiGLU && !a.w1) return cudaErrorInvalidValue;
  if (a.epilogue != kSwiGLU && a.w1) return cudaErrorInvalidValue;
  if (!a.y && !a.argmax) return cudaErrorInvalidValue;
  if (a.argmax && a.batch * kTileRows > static_cast<uint32_t>(kThreads)) return cudaErrorInvalidValue;
  if ((a.prologue == kHeadGate || a.prologue == kSigmoidGate) && !a.z) return cudaErrorInvalidValue;
  if ((a.prologue == kRmsNorm || a.prologue == kHeadGate) && !a.norm_w) return cudaErrorInvalidValue;
  if (a.prologue == kHeadGate && a.cols % 128) return cudaErrorInvalidValue;
  const uint32_t row_bytes = a.cols / 256 * block_bytes(a.fmt);
  if (row_bytes % 16 || reinterpret_cast<uintptr_t>(a.w0) % 16 || reinterpret_cast<uintptr_t>(a.w1) % 16)
    return cudaErrorMisalignedAddress;
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
  p.x_stride = a.x_stride ? a.x_stride : a.cols;
  p.batch = a.batch;
  p.prologue = a.prologue;
  p.norm_w = a.norm_w;
  p.eps = a.eps;
  p.z = a.z;
  p.epilogue = a.epilogue;
  p.y = a.y;
  p.y_stride = a.y_stride ? a.y_stride : a.rows;
  p.argmax = a.argmax;
  p.err = a.err;
  p.running = a.running;
  const uint32_t nsl = (a.batch + 3) / 4;
  if (a.fmt == kQ4K) {
    if (nsl == 1) return launch_t<kQ4K, 1>(a, p, s);
    if (nsl == 2) return launch_t<kQ4K, 2>(a, p, s);
    return launch_t<kQ4K, 8>(a, p, s);
  }
  if (nsl == 1) return launch_t<kQ6K, 1>(a, p, s);
  if (nsl == 2) return launch_t<kQ6K, 2>(a, p, s);
  return launch_t<kQ6K, 8>(a, p, s);
}

cudaError_t launch_gemv_f32(const float* W, uint32_t rows, uint32_t cols, const float* x, uint32_t x_stride,
                            uint32_t batch, float* y, uint32_t y_stride, cudaStream_t s) {
  const uint32_t warps = rows * batch;
  gemv_f32_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>(W, rows, cols, x, x_stride ? x_stride : cols, batch, y,
                                                             y_stride ? y_stride : rows);
  return cudaGetLastError();
}

}  // namespace rta
