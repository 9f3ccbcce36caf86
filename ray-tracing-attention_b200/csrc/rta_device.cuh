// rta_device.cuh -- sm_100a device primitives shared by the decode kernels.
//
// * mbarrier + cp.async.bulk (TMA bulk copy engine) staging with bounded waits:
//   every spin ends after RTA_WAIT_NS of %globaltimer time, records
//   RTA_DEVERR_TIMEOUT in the launch's error word and lets the CTA return.
// * Programmatic dependent launch (griddepcontrol) so a kernel can stream its
//   weights before the producer of its activations has finished.
// * Integer mma.sync tiles (u8 x s8 -> s32): the GEMV products are exact
//   integers; block scales are applied in fp32 afterwards.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

#ifndef RTA_WAIT_NS
#define RTA_WAIT_NS 1000000000ull  // 1 s bound on any device-side wait
#endif

// Device error bits (the host maps any non-zero word to RTA_E_DEVICE_CHECK).
enum : uint32_t {
  RTA_DEVERR_TIMEOUT = 1u,        // an mbarrier / counter wait exceeded RTA_WAIT_NS
  RTA_DEVERR_NONFINITE = 256u,    // mirrors the reference's control[3] bit 256
  RTA_DEVERR_TOKEN = 2048u,       // argmax produced no valid vocabulary row
  RTA_DEVERR_DETECTOR = 65536u,   // mirrors the reference detector error bit
};

namespace rta {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------ mbarrier / TMA
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0,1,0,p; }"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded wait on one mbarrier phase.  Returns false (and flags the error
// word) when the bound is exceeded.
// The spin is out of line: call sites keep only the first test, which keeps
// warp-specialized kernels' hot loops small in the instruction cache.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, uint32_t* err) {
  const uint64_t start = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 0u && globaltimer() - start > RTA_WAIT_NS) {
      if (err) atomicOr(err, RTA_DEVERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err);
}
// 1-D bulk copy global -> shared, completing on `bar` (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same, with an L2 eviction hint for streamed-once weights.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ------------------------------------------------------------------- PDL
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ------------------------------------------------------------ integer MMA
// D(16x8,s32) += A(16x32,u8,row) * B(32x8,s8,col)
__device__ __forceinline__ void mma_u8s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D(16x8,s32) += A(16x16,u8,row) * B(16x8,s8,col)
__device__ __forceinline__ void mma_u8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// ------------------------------------------------------------------ misc
__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}
// detectorSigmoid (reference resident_common.glsl:138)
__device__ __forceinline__ float detector_sigmoid(float v) {
  if (v >= 0.f) return 1.0f / (1.0f + expf(-v));
  const float light = expf(v);
  return light / (1.0f + light);
}
__device__ __forceinline__ float softplus(float v) { return fmaxf(v, 0.f) + logf(1.0f + expf(-fabsf(v))); }
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
// Load 4 bytes at byte offset `byte_off` from a 4-byte aligned shared base
// (Q6_K blocks are 210 bytes, so odd blocks of a row start 2 bytes off a word
// boundary).  `base` itself must be word aligned.
__device__ __forceinline__ uint32_t lds_u32_unaligned(const uint8_t* base, uint32_t byte_off) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(base + (byte_off & ~3u));
  const uint32_t lo = w[0];
  if ((byte_off & 3u) == 0u) return lo;
  return __funnelshift_r(lo, w[1], (byte_off & 3u) * 8u);
}
// Ordered key for a float so that unsigned max == float max.
__device__ __forceinline__ uint32_t float_order_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float float_from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// Packed (value, id) with max == larger value, then lower id.
__device__ __forceinline__ unsigned long long pack_argmax(float v, uint32_t id) {
  return (static_cast<unsigned long long>(float_order_key(v)) << 32) | static_cast<uint32_t>(~id);
}

}  // namespace rta
