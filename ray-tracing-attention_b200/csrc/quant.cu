// quant.cu -- Q4_K / Q6_K block quantization and dequantization on the GPU.
//
// The quantizer is the reference's own history-packet quantizer
// (ray_tracing/native/shaders/resident_history_quant.glsl:11-38): per-group
// min/max -> fp16 super-scales -> 6-bit (Q4_K) / 8-bit (Q6_K) group codes ->
// 4/6-bit values.  Every rounding step is written with explicit _rn intrinsics
// so no multiply-add is contracted and results match the CPU restatement bit
// for bit.  The dequantizer is ggufValue (resident_quant.glsl:10-19):
// (d*sc)*q - dmin*m and (d*scale)*(q6-32).
#include <algorithm>

#include "packets.cuh"
#include "rta_internal.h"

namespace rta {

__device__ __forceinline__ float round_half(float v) { return __half2float(__float2half_rn(v)); }
// GLSL max(x,y) = x < y ? y : x, min(x,y) = y < x ? y : x: the operand order
// fixes the sign of zero results (fmaxf/fminf leave it unspecified).
__device__ __forceinline__ float gmax(float a, float b) { return a < b ? b : a; }
__device__ __forceinline__ float gmin(float a, float b) { return b < a ? b : a; }
__device__ __forceinline__ float clampf_(float v, float lo, float hi) { return gmin(gmax(v, lo), hi); }
__device__ __forceinline__ void put_half(uint8_t* p, float v) {
  const unsigned short h = __half_as_ushort(__float2half_rn(v));
  p[0] = static_cast<uint8_t>(h);
  p[1] = static_cast<uint8_t>(h >> 8);
}

__device__ void quant_q4k_block(const float* v, uint8_t* out) {
  float gscale[8], gminv[8];
  uint32_t sc[8], mn[8];
  for (int g = 0; g < 8; ++g) {
    float lo = 0.f, hi = 0.f;
    for (int i = 0; i < 32; ++i) {
      const float x = v[g * 32 + i];
      lo = gmin(lo, x);
      hi = gmax(hi, x);
    }
    gscale[g] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    gminv[g] = -lo;
  }
  float maxD = 0.f, maxMin = 0.f;
  for (int g = 0; g < 8; ++g) {
    maxD = gmax(maxD, gscale[g]);
    maxMin = gmax(maxMin, gminv[g]);
  }
  const float d = round_half(__fdiv_rn(maxD, 63.0f));
  const float dm = round_half(__fdiv_rn(maxMin, 63.0f));
  uint8_t blk[144];
  for (int i = 0; i < 144; ++i) blk[i] = 0;
  put_half(blk, d);
  put_half(blk + 2, dm);
  for (int g = 0; g < 8; ++g) {
    sc[g] = static_cast<uint32_t>(clampf_(roundf(__fdiv_rn(gscale[g], gmax(d, 1e-30f))), 0.f, 63.f));
    mn[g] = static_cast<uint32_t>(clampf_(roundf(__fdiv_rn(gminv[g], gmax(dm, 1e-30f))), 0.f, 63.f));
  }
  for (int g = 0; g < 4; ++g) {
    blk[4 + g] = static_cast<uint8_t>(sc[g] | ((sc[g + 4] >> 4) << 6));
    blk[8 + g] = static_cast<uint8_t>(mn[g] | ((mn[g + 4] >> 4) << 6));
    blk[12 + g] = static_cast<uint8_t>((sc[g + 4] & 15u) | ((mn[g + 4] & 15u) << 4));
  }
  for (uint32_t i = 0; i < 256u; ++i) {
    const uint32_t g = i / 32u;
    const float offset = __fmul_rn(dm, static_cast<float>(mn[g]));
    const float step = __fmul_rn(d, static_cast<float>(sc[g]));
    const uint32_t q = static_cast<uint32_t>(
        clampf_(roundf(__fdiv_rn(__fadd_rn(v[i], offset), gmax(step, 1e-30f))), 0.f, 15.f));
    blk[16 + (i / 64u) * 32u + i % 32u] |= static_cast<uint8_t>(q << ((i % 64u) / 32u * 4u));
  }
  for (int i = 0; i < 144; ++i) out[i] = blk[i];
}

__device__ void quant_q6k_block(const float* v, uint8_t* out) {
  float gscale[16];
  for (int g = 0; g < 16; ++g) {
    float hi = 0.f;
    for (int i = 0; i < 16; ++i) hi = gmax(hi, fabsf(v[g * 16 + i]));
    gscale[g] = __fdiv_rn(hi, 31.0f);
  }
  float maxD = 0.f;
  for (int g = 0; g < 16; ++g) maxD = gmax(maxD, gscale[g]);
  const float d = round_half(__fdiv_rn(maxD, 127.0f));
  uint8_t blk[210];
  for (int i = 0; i < 210; ++i) blk[i] = 0;
  put_half(blk + 208, d);
  uint32_t sc[16];
  for (int g = 0; g < 16; ++g) {
    sc[g] = static_cast<uint32_t>(clampf_(roundf(__fdiv_rn(gscale[g], gmax(d, 1e-30f))), 0.f, 127.f));
    blk[192 + g] = static_cast<uint8_t>(sc[g]);
  }
  for (uint32_t i = 0; i < 256u; ++i) {
    const float step = __fmul_rn(d, static_cast<float>(sc[i / 16u]));
    const uint32_t q = static_cast<uint32_t>(
        static_cast<int>(clampf_(roundf(__fdiv_rn(v[i], gmax(step, 1e-30f))), -32.f, 31.f)) + 32);
    const uint32_t part = i / 128u, within = i % 128u;
    blk[part * 64u + within % 64u] |= static_cast<uint8_t>((q & 15u) << ((within / 64u) * 4u));
    blk[128u + part * 32u + within % 32u] |= static_cast<uint8_t>((q >> 4) << ((within / 32u) * 2u));
  }
  for (int i = 0; i < 210; ++i) out[i] = blk[i];
}


// Counter-based N(0, 1) source for synthetic weights and histories: an
// Irwin-Hall sum of eight 16-bit uniforms taken from two splitmix64 outputs
// keyed by (seed, element index), centred and scaled to unit variance.  Only
// integer operations, one exact int -> float conversion and one rounded
// multiply are involved, so a CPU restatement reproduces every value bit for
// bit (the synthetic model of a test can be rebuilt on the host).  The tails
// end at about 4.9 sigma, which synthetic weights do not miss.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
constexpr float kIrwinHall8Scale = 1.8688124e-05f;  // 1 / sqrt(8 (2^32 - 1) / 12)
__device__ __forceinline__ float synthetic_normal(uint64_t seed, uint64_t index) {
  const uint64_t r1 = splitmix64(seed * 0x632be59bd9b4e019ull ^ index);
  const uint64_t r2 = splitmix64(r1);
  int32_t sum = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    sum += static_cast<int32_t>((r1 >> (16 * i)) & 0xffffu) + static_cast<int32_t>((r2 >> (16 * i)) & 0xffffu);
  return __fmul_rn(static_cast<float>(sum - 262140), kIrwinHall8Scale);
}

__global__ void random_quantize_kernel(int fmt, uint64_t seed, float sigma, uint64_t first_block, size_t nblocks,
                                       uint8_t* __restrict__ dst) {
  const size_t b = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  float v[256];
  const uint64_t base = (first_block + b) * 256ull;
  for (int i = 0; i < 256; ++i) v[i] = __fmul_rn(sigma, synthetic_normal(seed, base + i));
  if (fmt == kQ4K) quant_q4k_block(v, dst + b * kQ4KBytes);
  else quant_q6k_block(v, dst + b * kQ6KBytes);
}

__global__ void random_normal_kernel(uint64_t seed, float sigma, float mean, size_t n, float* __restrict__ dst) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __fadd_rn(mean, __fmul_rn(sigma, synthetic_normal(seed, i)));
}

// fp16 variant (synthetic K/V histories); grid-stride for multi-GB rings
__global__ void random_normal_half_kernel(uint64_t seed, float sigma, size_t n, __half* __restrict__ dst) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2half_rn(__fmul_rn(sigma, synthetic_normal(seed, i)));
}

__device__ __forceinline__ float q4k_value(const uint8_t* b, uint32_t index) {
  const uint32_t group = index / 32u;
  uint32_t sc, mn;
  if (group < 4u) {
    sc = b[4 + group] & 63u;
    mn = b[8 + group] & 63u;
  } else {
    const uint32_t p = group - 4u, mixed = b[12 + p];
    sc = (mixed & 15u) | ((static_cast<uint32_t>(b[4 + p]) >> 6) << 4);
    mn = (mixed >> 4) | ((static_cast<uint32_t>(b[8 + p]) >> 6) << 4);
  }
  const uint32_t packed = b[16 + (index / 64u) * 32u + index % 32u];
  const uint32_t q = (packed >> ((index % 64u) / 32u * 4u)) & 15u;
  const float d = half_bits_to_float(b[0] | (b[1] << 8)), dmin = half_bits_to_float(b[2] | (b[3] << 8));
  return __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                   __fmul_rn(dmin, static_cast<float>(mn)));
}
__device__ __forceinline__ float q6k_value(const uint8_t* b, uint32_t index) {
  const uint32_t half = index / 128u, local = index % 128u;
  const uint32_t ql = (b[half * 64u + local % 64u] >> ((local / 64u) * 4u)) & 15u;
  const uint32_t qh = (b[128u + half * 32u + local % 32u] >> ((local / 32u) * 2u)) & 3u;
  const int scale = static_cast<int>(static_cast<int8_t>(b[192u + index / 16u]));
  const float d = half_bits_to_float(b[208] | (b[209] << 8));
  return __fmul_rn(__fmul_rn(d, static_cast<float>(scale)), static_cast<float>(static_cast<int>(ql | (qh << 4)) - 32));
}

__global__ void dequantize_kernel(int fmt, const uint8_t* __restrict__ src, size_t nvalues, float* __restrict__ dst) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nvalues) return;
  const size_t blk = i / 256;
  const uint32_t j = static_cast<uint32_t>(i % 256);
  dst[i] = fmt == kQ4K ? q4k_value(src + blk * kQ4KBytes, j) : q6k_value(src + blk * kQ6KBytes, j);
}

// One 256-thread CTA per block (the packet quantizer of packets.cuh, also used
// by the decode step to pack history); grid-stride over blocks.
__global__ void __launch_bounds__(256) quantize_cta_kernel(int fmt, const float* __restrict__ src, size_t nblocks,
                                                           uint8_t* __restrict__ dst) {
  __shared__ PackScratch sh;
  for (size_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
    const float x = src[b * 256 + threadIdx.x];
    if (fmt == kQ4K) pack_q4k_block(x, dst + b * kQ4KBytes, sh);
    else pack_q6k_block(x, dst + b * kQ6KBytes, sh);
  }
}

// History packets of `rows` positions from fp32 K and V rows [row][kvh][256]:
// CTA (row, j) packs key head j (j < kvh) or value head j - kvh.
__global__ void __launch_bounds__(256) pack_history_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                                           uint32_t kvh, uint8_t* __restrict__ dst) {
  __shared__ PackScratch sh;
  const uint32_t row = blockIdx.x, j = blockIdx.y;
  uint8_t* pkt = dst + static_cast<size_t>(row) * packet_bytes(kvh);
  if (j < kvh) pack_q4k_block(k[(static_cast<size_t>(row) * kvh + j) * 256 + threadIdx.x], pkt + j * kPacketKeyBytes, sh);
  else
    pack_q6k_block(v[(static_cast<size_t>(row) * kvh + (j - kvh)) * 256 + threadIdx.x],
                   pkt + kvh * kPacketKeyBytes + (j - kvh) * kPacketValueBytes, sh);
}

// Seeded history packets (throughput runs): values N(0, 1) per block, packed.
__global__ void __launch_bounds__(256) random_packets_kernel(uint64_t seed, size_t rows, uint32_t kvh,
                                                             uint8_t* __restrict__ dst) {
  __shared__ PackScratch sh;
  const size_t blocks = rows * 2u * kvh;
  for (size_t b = blockIdx.x; b < blocks; b += gridDim.x) {
    const size_t row = b / (2u * kvh);
    const uint32_t j = static_cast<uint32_t>(b % (2u * kvh));
    const float x = synthetic_normal(seed, b * 256 + threadIdx.x);
    uint8_t* pkt = dst + row * packet_bytes(kvh);
    if (j < kvh) pack_q4k_block(x, pkt + j * kPacketKeyBytes, sh);
    else pack_q6k_block(x, pkt + kvh * kPacketKeyBytes + (j - kvh) * kPacketValueBytes, sh);
  }
}

cudaError_t launch_pack_history(const float* k, const float* v, uint32_t rows, uint32_t kvh, uint8_t* dst,
                                cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (!k || !v || !dst || kvh == 0) return cudaErrorInvalidValue;
  pack_history_kernel<<<dim3(rows, 2 * kvh), 256, 0, s>>>(k, v, kvh, dst);
  return cudaGetLastError();
}
cudaError_t launch_random_packets(uint64_t seed, size_t rows, uint32_t kvh, uint8_t* dst, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const size_t grid = std::min<size_t>(rows * 2u * kvh, 148u * 16u);
  random_packets_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(seed, rows, kvh, dst);
  return cudaGetLastError();
}

cudaError_t launch_quantize(int fmt, const float* src, size_t nblocks, uint8_t* dst, cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  const size_t grid = std::min<size_t>(nblocks, 148u * 16u);
  quantize_cta_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(fmt, src, nblocks, dst);
  return cudaGetLastError();
}
cudaError_t launch_random_quantize(int fmt, uint64_t seed, float sigma, uint64_t first_block, size_t nblocks,
                                   uint8_t* dst, cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  random_quantize_kernel<<<static_cast<unsigned>((nblocks + 127) / 128), 128, 0, s>>>(fmt, seed, sigma, first_block,
                                                                                        nblocks, dst);
  return cudaGetLastError();
}
cudaError_t launch_random_normal(uint64_t seed, float sigma, float mean, size_t n, float* dst, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  random_normal_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(seed, sigma, mean, n, dst);
  return cudaGetLastError();
}
cudaError_t launch_random_normal_half(uint64_t seed, float sigma, size_t n, __half* dst, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const size_t blocks = std::min<size_t>((n + 255) / 256, 148u * 64u);
  random_normal_half_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(seed, sigma, n, dst);
  return cudaGetLastError();
}
cudaError_t launch_dequantize(int fmt, const uint8_t* src, size_t nblocks, float* dst, cudaStream_t s) {
  const size_t n = nblocks * 256;
  if (n == 0) return cudaSuccess;
  dequantize_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(fmt, src, n, dst);
  return cudaGetLastError();
}

}  // namespace rta
