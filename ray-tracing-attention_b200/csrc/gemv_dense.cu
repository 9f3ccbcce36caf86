// gemv_dense.cu -- decode GEMV for matrices the exporter keeps in a dense
// float format: F32 (code 0), F16 (1) and BF16 (30), export.py:12.
//
// Reference: op 2 of ray_tracing/native/shaders/resident_math.comp:39-75 over
// ggufValue's dense branches (resident_quant.glsl:6-9: the word's bits, an
// unpacked half, the bf16 bits shifted into the high half of a float).  A
// real rt-compile of safetensors weights emits BF16 projections, so the engine
// serves them here with the same prologues (RMSNorm, per-head gated norm,
// sigmoid gate, SwiGLU of gate / up rows) and epilogues (store, residual add,
// SwiGLU of two matrices, vocabulary argmax) as the quantized GEMVs.
//
// B200 design: HBM-bound streaming.  A CTA of 8 warps owns 16 rows (two per
// warp); the prologue-applied activation rows of the launch (up to 8) sit in
// shared memory as fp32; every lane streams 16-byte weight vectors with
// no-allocate loads (each weight is read once) and keeps one fp32 accumulator
// per (row, batch row); a warp butterfly then sums the lanes.
#include <mutex>

#include "rta_internal.h"

namespace rta {
namespace {

constexpr uint32_t kDThreads = 256, kDWarps = 8, kDRowsPerWarp = 2, kDRows = kDWarps * kDRowsPerWarp;
constexpr uint32_t kDenseSmemBudget = 200u * 1024u;  // activation rows of one launch

struct DenseParams {
  const uint8_t* w[2];
  uint32_t nmat, rows, cols, row_bytes;
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
  uint32_t arg_step;
  const uint32_t* running;
  uint32_t run_step;
};

__device__ __forceinline__ float swiglu_value(float gv, float uv) {
  const float amp = fabsf(gv) * fabsf(uv) * detector_sigmoid(gv);
  const float sgn = (gv > 0.f ? 1.f : gv < 0.f ? -1.f : 0.f) * (uv > 0.f ? 1.f : uv < 0.f ? -1.f : 0.f);
  return sgn * amp;
}

// Eight weights of a row from one 16-byte (F16 / BF16) or two 16-byte (F32) vectors.
template <int FMT>
__device__ __forceinline__ void load8(const uint8_t* row, uint32_t k, float (&w)[8]) {
  if constexpr (FMT == kF32) {
    const float4* p = reinterpret_cast<const float4*>(row + static_cast<size_t>(k) * 4u);
    const float4 a = __ldcs(p), b = __ldcs(p + 1);
    w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
  } else {
    const uint4 u = __ldcs(reinterpret_cast<const uint4*>(row + static_cast<size_t>(k) * 2u));
    const uint32_t words[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (FMT == kF16) {
        w[2 * i] = half_bits_to_float(words[i]);
        w[2 * i + 1] = half_bits_to_float(words[i] >> 16);
      } else {  // BF16: the 16 bits are the high half of the float
        w[2 * i] = __uint_as_float(words[i] << 16);
        w[2 * i + 1] = __uint_as_float(words[i] & 0xffff0000u);
      }
    }
  }
}

template <int FMT, int NB>
__global__ void __launch_bounds__(kDThreads) gemv_dense_kernel(const DenseParams p) {
  extern __shared__ __align__(16) float xs[];  // [NB][cols] prologue-applied activation rows
  __shared__ float red[kDWarps];
  __shared__ unsigned long long best_s[NB];
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  const uint32_t r0 = blockIdx.x * kDRows + warp * kDRowsPerWarp;
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x < NB) best_s[threadIdx.x] = 0ull;
  // ---- prologue: x rows -> shared memory
  for (uint32_t b = 0; b < static_cast<uint32_t>(NB); ++b) {
    const float* xr = p.x + static_cast<size_t>(b) * p.x_stride;
    const float* zr = p.z ? p.z + static_cast<size_t>(b) * p.z_stride : nullptr;
    float* dst = xs + static_cast<size_t>(b) * p.cols;
    float inv = 1.f;
    if (p.prologue == kRmsNorm) {
      float ss = 0.f;
      for (uint32_t c = threadIdx.x; c < p.cols; c += kDThreads) ss += xr[c] * xr[c];
      ss = warp_sum(ss);
      __syncthreads();
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float t = 0.f;
#pragma unroll
      for (uint32_t i = 0; i < kDWarps; ++i) t += red[i];
      inv = rsqrtf(t / static_cast<float>(p.cols) + p.eps);
    }
    if (p.prologue == kHeadGate) {  // one warp per 128-wide head at a time
      for (uint32_t h = warp; h < p.cols / 128u; h += kDWarps) {
        float v[4], s = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[e] = xr[h * 128u + lane * 4u + e];
          s += v[e] * v[e];
        }
        const float hinv = rsqrtf(warp_sum(s) / 128.0f + p.eps);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t c = h * 128u + lane * 4u + e;
          const float zv = zr[c];
          dst[c] = v[e] * (((hinv * p.norm_w[c]) * zv) * detector_sigmoid(zv));
        }
      }
    } else {
      for (uint32_t c = threadIdx.x; c < p.cols; c += kDThreads) {
        float v = xr[c];
        if (p.prologue == kRmsNorm) v = v * inv * p.norm_w[c];
        else if (p.prologue == kSigmoidGate) v = v * detector_sigmoid(zr[c]);
        else if (p.prologue == kSwiGLUIn) v = swiglu_value(v, zr[c]);
        dst[c] = v;
      }
    }
  }
  __syncthreads();
  // ---- rows: lane-strided 8-weight vectors, fp32 accumulators per batch row
#pragma unroll
  for (uint32_t i = 0; i < kDRowsPerWarp; ++i) {
    const uint32_t r = r0 + i;
    if (r >= p.rows) break;  // warp-uniform
    float acc[2][NB];
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[m][b] = 0.f;
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (static_cast<uint32_t>(m) >= p.nmat) break;
      const uint8_t* row = p.w[m] + static_cast<size_t>(r) * p.row_bytes;
      for (uint32_t k = lane * 8u; k < p.cols; k += 256u) {
        float w[8];
        load8<FMT>(row, k, w);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const float4* xv = reinterpret_cast<const float4*>(xs + static_cast<size_t>(b) * p.cols + k);
          const float4 x0 = xv[0], x1 = xv[1];
          acc[m][b] += w[0] * x0.x + w[1] * x0.y + w[2] * x0.z + w[3] * x0.w + w[4] * x1.x + w[5] * x1.y +
                       w[6] * x1.z + w[7] * x1.w;
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const float g = warp_sum(acc[0][b]);
      const float u = p.nmat > 1u ? warp_sum(acc[1][b]) : 0.f;
      if (lane != 0u) continue;
      if (p.running && p.running[static_cast<size_t>(b) * p.run_step] == 0u) continue;  // stopped batch row
      float* yp = p.y ? p.y + static_cast<size_t>(b) * p.y_stride + r : nullptr;
      if (p.epilogue == kSwiGLU) *yp = swiglu_value(g, u);
      else if (p.epilogue == kAccumulate) *yp += g;
      else if (yp) *yp = g;
      if (p.argmax) {
        const unsigned long long key = pack_argmax(g, r);
        atomicMax(&best_s[b], key);
      }
    }
  }
  if (p.argmax) {
    __syncthreads();
    if (threadIdx.x < static_cast<uint32_t>(NB) && best_s[threadIdx.x])
      atomicMax(p.argmax + static_cast<size_t>(threadIdx.x) * p.arg_step, best_s[threadIdx.x]);
  }
}

template <int FMT, int NB>
cudaError_t launch_nb(const DenseParams& p, bool pdl, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(NB) * p.cols * 4u;
  {  // opt-in to large dynamic shared memory (with the static arrays above 48 KB in all), once per device
    static std::mutex m;
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(m);
    if (!done[dev]) {
      // the launcher keeps a launch's activation rows within 200 KB (kDenseSmemBudget),
      // leaving the static shared memory its room under the 227 KB limit
      e = cudaFuncSetAttribute(gemv_dense_kernel<FMT, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kDenseSmemBudget));
      if (e != cudaSuccess) return e;
      done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((p.rows + kDRows - 1) / kDRows);
  cfg.blockDim = dim3(kDThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_dense_kernel<FMT, NB>, p);
  if (e != cudaSuccess) (void)cudaGetLastError();  // a refused launch is reported here, not to the next call
  return e;
}

template <int FMT>
cudaError_t launch_fmt_dense(const DenseParams& p, uint32_t nb, bool pdl, cudaStream_t s) {
  switch (nb) {
    case 1: return launch_nb<FMT, 1>(p, pdl, s);
    case 2: return launch_nb<FMT, 2>(p, pdl, s);
    case 4: return launch_nb<FMT, 4>(p, pdl, s);
    default: return launch_nb<FMT, 8>(p, pdl, s);
  }
}

}  // namespace

bool dense_format(int fmt) { return fmt == kF32 || fmt == kF16 || fmt == kBF16; }
uint32_t dense_bytes(int fmt) { return fmt == kF32 ? 4u : 2u; }

cudaError_t launch_gemv_dense(const GemvArgs& a, cudaStream_t s) {
  if (!dense_format(a.fmt) || !a.w0 || !a.x || a.rows == 0 || a.cols == 0 || a.cols % 8u || a.batch == 0 ||
      a.batch > kMaxBatch || (!a.y && !a.argmax))
    return cudaErrorInvalidValue;
  if ((a.epilogue == kSwiGLU) != (a.w1 != nullptr)) return cudaErrorInvalidValue;
  if ((a.prologue == kHeadGate || a.prologue == kSigmoidGate || a.prologue == kSwiGLUIn) && !a.z)
    return cudaErrorInvalidValue;
  if ((a.prologue == kRmsNorm || a.prologue == kHeadGate) && !a.norm_w) return cudaErrorInvalidValue;
  if (a.prologue == kHeadGate && a.cols % 128u) return cudaErrorInvalidValue;
  const uint32_t row_bytes = a.cols * dense_bytes(a.fmt);
  if ((reinterpret_cast<uintptr_t>(a.w0) | reinterpret_cast<uintptr_t>(a.w1)) % 16u || row_bytes % 16u)
    return cudaErrorMisalignedAddress;
  DenseParams p = {};
  p.w[0] = a.w0;
  p.w[1] = a.w1;
  p.nmat = a.w1 ? 2u : 1u;
  p.rows = a.rows;
  p.cols = a.cols;
  p.row_bytes = row_bytes;
  p.x_stride = a.x_stride ? a.x_stride : a.cols;
  p.prologue = a.prologue;
  p.norm_w = a.norm_w;
  p.eps = a.eps;
  p.z_stride = a.z_stride ? a.z_stride : p.x_stride;
  p.epilogue = a.epilogue;
  p.y_stride = a.y_stride ? a.y_stride : a.rows;
  p.arg_step = a.argmax_step ? a.argmax_step : 1u;
  p.run_step = a.running_step ? a.running_step : 1u;
  // batch rows in launches of up to 8 whose activation rows fit in shared memory
  const uint32_t fit = static_cast<uint32_t>(kDenseSmemBudget / (static_cast<size_t>(a.cols) * 4u));
  for (uint32_t b0 = 0; b0 < a.batch;) {
    uint32_t nb = 8u;
    while (nb > 1u && (nb > a.batch - b0 || nb > fit)) nb /= 2u;
    if (fit == 0u) return cudaErrorInvalidValue;  // a single row's activation does not fit
    DenseParams q = p;
    q.batch = nb;
    q.x = a.x + static_cast<size_t>(b0) * p.x_stride;
    q.z = a.z ? a.z + static_cast<size_t>(b0) * p.z_stride : nullptr;
    q.y = a.y ? a.y + static_cast<size_t>(b0) * p.y_stride : nullptr;
    q.argmax = a.argmax ? a.argmax + static_cast<size_t>(b0) * p.arg_step : nullptr;
    q.running = a.running ? a.running + static_cast<size_t>(b0) * p.run_step : nullptr;
    cudaError_t e = a.fmt == kF32 ? launch_fmt_dense<kF32>(q, nb, a.pdl, s)
                    : a.fmt == kF16 ? launch_fmt_dense<kF16>(q, nb, a.pdl, s)
                                    : launch_fmt_dense<kBF16>(q, nb, a.pdl, s);
    if (e != cudaSuccess) return e;
    b0 += nb;
  }
  return cudaSuccess;
}

}  // namespace rta
