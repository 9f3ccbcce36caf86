// packets.cuh -- the reference's history-packet quantizer, one 256-thread CTA
// per 256-value block, and the packet layout of one history position.
//
// Quantizer: resident_history_quant.glsl:11-38 (the same steps as the serial
// restatement in quant.cu and the oracle): per-group min/max -> fp16 block
// scales d (and dmin) -> 6-bit (Q4_K) / 8-bit (Q6_K) group codes -> 4/6-bit
// values, every rounding written with explicit _rn intrinsics.  GLSL min/max
// start from +0 and only a strictly smaller / larger value replaces the running
// one, so a reduction over a group equals "m if m < 0 else +0" (min) and
// "M if M > 0 else +0" (max) of the group's true extrema, whatever the order.
//
// Packet of one position (1416 bytes for 4 KV heads x 256): the 4 keys as Q4_K
// blocks (144 B each) then the 4 values as Q6_K blocks (210 B each)
// (HISTORY_RECORD_BYTES, resident_history_quant.glsl:2-9).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#include "rta_device.cuh"

namespace rta {

constexpr uint32_t kPacketKeyBytes = 144, kPacketValueBytes = 210;
__host__ __device__ constexpr uint32_t packet_bytes(uint32_t kvh) { return kvh * (kPacketKeyBytes + kPacketValueBytes); }

namespace pq {
__device__ __forceinline__ float round_half(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ float gmax(float a, float b) { return a < b ? b : a; }
__device__ __forceinline__ float gmin(float a, float b) { return b < a ? b : a; }
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return gmin(gmax(v, lo), hi); }
// fp16 field of a block: every one sits at an even offset of a block that
// starts at an even address, so one 16-bit store writes it
__device__ __forceinline__ void put_half(uint8_t* p, float v) {
  *reinterpret_cast<unsigned short*>(p) = __half_as_ushort(__float2half_rn(v));
}
}  // namespace pq

// Scratch a CTA needs for one block: 32 floats + 256 code bytes (shared).
struct PackScratch {
  float f[32];
  uint8_t codes[256];
};

// Q4_K block of v[0..255] (thread i holds v[i]; 256 threads) into out[0..143].
__device__ __forceinline__ void pack_q4k_block(float x, uint8_t* out, PackScratch& sh) {
  const uint32_t i = threadIdx.x, w = i >> 5;  // warp w = group w of 32
  float mn = x, mx = x;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float lo = mn < 0.f ? mn : 0.f, hi = mx > 0.f ? mx : 0.f;
  if ((i & 31u) == 0u) {
    sh.f[w] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);  // group scale
    sh.f[8 + w] = -lo;                              // group minimum
  }
  __syncthreads();
  float maxD = 0.f, maxMin = 0.f;
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    maxD = pq::gmax(maxD, sh.f[g]);
    maxMin = pq::gmax(maxMin, sh.f[8 + g]);
  }
  const float d = pq::round_half(__fdiv_rn(maxD, 63.0f)), dm = pq::round_half(__fdiv_rn(maxMin, 63.0f));
  const uint32_t sc = static_cast<uint32_t>(pq::clampf(roundf(__fdiv_rn(sh.f[w], pq::gmax(d, 1e-30f))), 0.f, 63.f));
  const uint32_t mc = static_cast<uint32_t>(pq::clampf(roundf(__fdiv_rn(sh.f[8 + w], pq::gmax(dm, 1e-30f))), 0.f, 63.f));
  const float offset = __fmul_rn(dm, static_cast<float>(mc)), step = __fmul_rn(d, static_cast<float>(sc));
  sh.codes[i] = static_cast<uint8_t>(
      pq::clampf(roundf(__fdiv_rn(__fadd_rn(x, offset), pq::gmax(step, 1e-30f))), 0.f, 15.f));
  __syncthreads();  // codes and the group scales (read below) are complete
  if (i < 128u) {   // byte 16 + 32p + j: element 64p + j (low nibble) and 64p + 32 + j (high)
    const uint32_t e = 64u * (i / 32u) + i % 32u;
    out[16u + i] = static_cast<uint8_t>(sh.codes[e] | (sh.codes[e + 32u] << 4));
  } else if (i == 128u) {
    pq::put_half(out, d);
    pq::put_half(out + 2, dm);
  } else if (i >= 132u && i < 136u) {
    const uint32_t g = i - 132u;
    auto code = [&](uint32_t grp, bool minimum) {
      const float val = sh.f[(minimum ? 8u : 0u) + grp];
      const float div = pq::gmax(minimum ? dm : d, 1e-30f);
      return static_cast<uint32_t>(pq::clampf(roundf(__fdiv_rn(val, div)), 0.f, 63.f));
    };
    const uint32_t s0 = code(g, false), s4 = code(g + 4u, false), m0 = code(g, true), m4 = code(g + 4u, true);
    out[4u + g] = static_cast<uint8_t>(s0 | ((s4 >> 4) << 6));
    out[8u + g] = static_cast<uint8_t>(m0 | ((m4 >> 4) << 6));
    out[12u + g] = static_cast<uint8_t>((s4 & 15u) | ((m4 & 15u) << 4));
  }
  __syncthreads();  // scratch reusable
}

// Q6_K block of v[0..255] (thread i holds v[i]; 256 threads) into out[0..209].
__device__ __forceinline__ void pack_q6k_block(float x, uint8_t* out, PackScratch& sh) {
  const uint32_t i = threadIdx.x;  // group i/16; lanes 0-15 / 16-31 of a warp hold two groups
  float hi = fabsf(x);
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  if ((i & 15u) == 0u) sh.f[i / 16u] = __fdiv_rn(hi, 31.0f);
  __syncthreads();
  float maxD = 0.f;
#pragma unroll
  for (int g = 0; g < 16; ++g) maxD = pq::gmax(maxD, sh.f[g]);
  const float d = pq::round_half(__fdiv_rn(maxD, 127.0f));
  const uint32_t sc =
      static_cast<uint32_t>(pq::clampf(roundf(__fdiv_rn(sh.f[i / 16u], pq::gmax(d, 1e-30f))), 0.f, 127.f));
  const float step = __fmul_rn(d, static_cast<float>(sc));
  sh.codes[i] = static_cast<uint8_t>(
      static_cast<int>(pq::clampf(roundf(__fdiv_rn(x, pq::gmax(step, 1e-30f))), -32.f, 31.f)) + 32);
  __syncthreads();
  if (i < 128u) {  // ql byte part*64 + w: element part*128 + w (low nibble), part*128 + 64 + w (high)
    const uint32_t e = 128u * (i / 64u) + i % 64u;
    out[i] = static_cast<uint8_t>((sh.codes[e] & 15u) | ((sh.codes[e + 64u] & 15u) << 4));
  } else if (i < 192u) {  // qh byte 128 + part*32 + w: elements part*128 + w + 32k at bits 2k
    const uint32_t b = i - 128u, e = 128u * (b / 32u) + b % 32u;
    out[i] = static_cast<uint8_t>((sh.codes[e] >> 4) | ((sh.codes[e + 32u] >> 4) << 2) |
                                  ((sh.codes[e + 64u] >> 4) << 4) | ((sh.codes[e + 96u] >> 4) << 6));
  } else if (i < 208u) {
    const uint32_t g = i - 192u;
    out[i] = static_cast<uint8_t>(
        pq::clampf(roundf(__fdiv_rn(sh.f[g], pq::gmax(d, 1e-30f))), 0.f, 127.f));
  } else if (i == 208u) {
    pq::put_half(out + 208, d);
  }
  __syncthreads();
}

}  // namespace rta
