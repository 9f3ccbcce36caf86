// qgemm.cu -- batched products with Q4_K / Q6_K weights on the 5th-generation
// tensor cores (tcgen05), for batches of 16 rows or more (the ragged
// multi-sequence decode and the batch-64 vocabulary readout).
//
// Y[n][r] (op)= sum_k W[r][k] X[n][k] is op 2 of the reference
// (ray_tracing/native/shaders/resident_math.comp:39-75) at batch > 1; the
// batch-1 decode keeps the integer mma.sync GEMV (gemv.cu).
//
// Arithmetic.  Per 256-wide block b of a weight row the quantized value is
//   Q4_K: w = (d*sc_G)*q - dmin*m_G  (resident_quant.glsl:10-15)
//   Q6_K: w = (d*sc_g)*(q - 32)      (resident_quant.glsl:16-19)
// so  sum_k w_k x_k = sum_G (d sc_G) sum_{k in G} (q_k - 8) x_k
//                    + sum_G (8 d sc_G - dmin m_G) X_G       (Q4_K)
// with the exact integers sc (q - 8) (Q4_K, |.| <= 504) or sc (q - 32) (Q6_K,
// |.| <= 4096; fp16 holds them exactly up to 2048 and rounds to even above)
// and the group sums X_G.  The A operand in tensor memory is fp16(2^6 d *
// integer) (one rounding), the mins term is one more K=16 MMA per block of
// fp16(2^6 (8 d sc - dmin m)) against the group sums of the same fp16 x (fp32
// sums split into two fp16 halves, so the mins cancel against exactly what
// the codes see), the tensor cores accumulate every block of a work unit in
// fp32, and the epilogue scales by 2^-6.  Beyond fp32 accumulation the
// roundings are x -> fp16 and the two operand roundings.
//
// Weights use the "panel" layout of this library (formats 212 / 214, made by
// launch_tile_tc): per 128-row tile and 256-wide block column one contiguous
// panel of the same bytes, ordered so that the dequantizing thread of row m
// reads its bytes with conflict-free 16-byte shared loads:
//   Q4_K panel (18432 B): codes [pl 4][part 2][row 128][16 B] = GGUF bytes
//     16 + 32*pl + 16*part .. +15 of the row, each 4-byte word as bytes
//     (0, 2, 1, 3); then headers [row 128][16 B] (d, dmin, 12 packed 6-bit
//     scales and mins).
//   Q6_K panel (26880 B): per half h (2): ql [j 2][part 2][row 128][16 B] =
//     GGUF ql bytes 64h + 32j + 16part .. +15, then qh [part 2][row 128][16 B]
//     = qh bytes 128 + 32h + 16part .. +15; then scales [row 128][16 int8],
//     then d [row 128][fp16].
//
// Work order: tile by tile, within a tile every block column (K slices of
// `width` block columns are supported; every launch now takes the whole K).
// One persistent CTA per SM (608 threads) takes an equal contiguous range of
// that order (whole tiles when an argmax needs whole sums), and the
// activation block columns stream through the slots (slot = block column %
// slots, prefetched ahead of the MMAs); a unit (one tile's run of block
// columns inside the range) ends in a partial sum that lands atomically, so a
// CTA emits about 1 + tiles/CTAs partial sums.  (Slices as narrow as the slots,
// with the activations resident while a CTA walks a slice's tiles, emitted 2-4x
// more partial sums, 128 x N fp32 atomics each, and measured slower: 9007 vs
// 9247 tokens/s in the 9B ragged decode.)
//   warp 0      bulk-copies the range's weight panels, one per block column,
//               from kernel start (weights do not depend on earlier kernels)
//   warp 18     bulk-copies an activation block column into its slot (block
//               column % slots) when the slot holds another one, after
//               griddepcontrol.wait (written by the preceding prep kernel)
//   warps 10-17 dequantize the panel into tensor memory (A operand; thread =
//               row, tcgen05.st), two warps per 32-lane quarter (warp % 4)
//   warp 1      issues tcgen05.mma kind::f16 M=128 N=batch K=16 (A from tensor
//               memory, B from the slot), the K steps taking 128/N unit
//               accumulators in turn (double-buffered by unit), and commits
//               stage and slot releases to mbarriers
//   warps 2-9   add a finished unit's accumulators (tcgen05.ld; thread = row,
//               each warp half of the batch columns) and run the atomic /
//               store / residual / argmax epilogue
// Every wait is bounded (RTA_WAIT_NS): a stuck pipeline flags
// RTA_DEVERR_TIMEOUT, drains its copies and MMAs and frees tensor memory.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "rta_device.cuh"
#include "rta_internal.h"

namespace rta {
namespace tc {

constexpr uint32_t kThreads = 608;  // 19 warps
constexpr uint32_t kTileRows = 128;
constexpr uint32_t kQ4KPanel = 128u * kQ4KBytes, kQ6KPanel = 128u * kQ6KBytes;  // 18432, 26880
constexpr uint32_t kAStages = 3;  // tensor-memory A stages
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAColBase = 256, kA2ColBase = 448;  // tensor-memory columns of the A / A2 stages
constexpr uint32_t kMinSmem = 120u * 1024u;             // keeps one CTA per SM (tensor memory is taken whole)

template <int FMT>
struct Cfg {
  static constexpr bool kQ4 = FMT == kQ4K;
  static constexpr uint32_t kPanel = kQ4 ? kQ4KPanel : kQ6KPanel;
  static constexpr uint32_t kRawStages = kQ4 ? 4u : 3u;
};

// prep-buffer bytes per 256-wide block for a launch of N batch rows
__host__ __device__ constexpr uint32_t blk_bytes(bool q4, uint32_t N) { return N * 512u + (q4 ? N * 32u : 0u); }

struct Params {
  const uint8_t* w[2];  // panels of matrix 0 / 1 (rows appended after matrix 0's in the output)
  uint32_t nmat, rows, KB, ntiles;
  // Work order: K slices of `width` block columns, within a slice every tile,
  // within a tile the slice's block columns -- one panel per step.  A CTA takes
  // a contiguous range of that order (whole tiles when `whole_tiles`), and a
  // unit is a run of one tile's block columns inside the range.
  uint32_t width;        // block columns per K slice (== slots: activations resident per slice; == KB: streamed)
  uint32_t slots;        // activation block columns held in shared memory (slot = block column % slots)
  uint32_t total;        // panels of the product (ntiles * KB)
  uint32_t whole_tiles;  // 1: every unit is a whole tile (argmax, plain stores); 0: partial sums land atomically
  uint32_t split;        // 1: B columns n and n + N/2 carry fp16(x) and fp16(x - fp16(x)) of batch row n
  const uint8_t* xb;  // prep output
  uint32_t blk;       // prep bytes per block
  uint32_t batch;     // live batch rows of this launch (<= N)
  float* y;
  uint32_t y_stride;
  int epilogue;
  unsigned long long* argmax;
  uint32_t arg_step;
  const uint32_t* running;
  uint32_t run_step;
  uint32_t* err;
  uint32_t off_b, off_bar, off_misc, b_slot;  // b_slot: bytes between activation slots
};

// Position of one panel in the work order.
struct Walk {
  uint32_t t, kb, k0, k1;  // tile, block column, the slice's block columns [k0, k1)
  __device__ __forceinline__ void start(const Params& p, uint32_t q) {
    const uint32_t full = p.ntiles * p.width;  // panels of a full-width slice (only the last may be narrower)
    const uint32_t sl = q / full, r = q - sl * full;
    k0 = sl * p.width;
    k1 = min(p.KB, k0 + p.width);
    t = r / (k1 - k0);
    kb = k0 + r % (k1 - k0);
  }
  __device__ __forceinline__ void next(const Params& p) {
    if (++kb < k1) return;
    kb = k0;
    if (++t < p.ntiles) return;
    t = 0;
    k0 = k1;
    k1 = min(p.KB, k0 + p.width);
    kb = k0;
  }
};
__device__ __forceinline__ void cta_range(const Params& p, uint32_t& q0, uint32_t& q1) {
  if (p.whole_tiles) {
    q0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * p.ntiles / gridDim.x) * p.KB;
    q1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1u) * p.ntiles / gridDim.x) * p.KB;
  } else {
    q0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * p.total / gridDim.x);
    q1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1u) * p.total / gridDim.x);
  }
}
// After panel q at `w`, does the activation slot of w.kb get another block
// column before its next use (so its MMAs must release it)?  The next use of
// the slot is the same tile's block column kb + slots, else the next tile's
// first block column in the slot (k0 + (kb - k0) % slots), else a later slice.
__device__ __forceinline__ bool slot_changes(const Params& p, const Walk& w, uint32_t q, uint32_t q1) {
  const bool keep = w.kb + p.slots >= w.k1 && w.kb - w.k0 < p.slots && w.t + 1u < p.ntiles &&
                    q + (w.k1 - w.k0) < q1;
  return !keep;
}

struct Prep {
  const float* x;
  uint32_t x_stride;
  const float* z;
  uint32_t z_stride;
  const float* norm_w;
  float eps;
  int prologue;
  uint32_t cols, batch, N;
  const uint32_t* running;
  uint32_t run_step;
  uint8_t* xb;
  uint32_t blk;
  bool q4;
  bool split;  // rows N/2 .. N-1 of the stage carry the fp16 remainders of rows 0 .. N/2-1
  float* zero_y;  // split stores: y rows of live sequences are zeroed here before the partial sums land
  uint32_t zero_cols, zero_stride;
};
constexpr uint32_t kPrepCols = 2048;  // activation columns per prep CTA (grid: batch rows x column chunks)

// ------------------------------------------------------------- tcgen05 glue
__device__ __forceinline__ uint32_t h2_bits(__half2 h) {
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}
__device__ __forceinline__ __half2 bits_h2(uint32_t u) {
  __half2 h;
  memcpy(&h, &u, 4);
  return h;
}
__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, __half2 b, __half2 c) {
  return h2_bits(__hfma2(bits_h2(a), b, c));
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, __half2 b) { return h2_bits(__hmul2(bits_h2(a), b)); }

// The block scales are folded into the fp16 operand, pre-multiplied by 2^6 so
// that small weights stay clear of fp16 subnormals (|w| < 1023 stays finite);
// the epilogue multiplies the accumulator by 2^-6.
constexpr float kOperandScale = 64.0f;

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core
// matrices, `lbo` bytes between the two core matrices of one K=16 step, `sbo`
// bytes between 8-row groups (version 1, base offset 0).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// Instruction descriptor of kind::f16: fp16 A and B (K-major), fp32 D, M=128.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t N) {
  return (1u << 4) | ((N >> 3) << 17) | ((kTileRows >> 4) << 24);
}

// MMA and commit, issued by a whole warp in warp-uniform control flow: one
// elected lane issues.  (Operands computed uniformly stay in uniform
// registers; a loop run by a single lane pays register moves per MMA and
// issues at about half the rate.)
__device__ __forceinline__ void mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Four MMAs under one election: D_i += A_i B_i (D_i, A_i tensor-memory
// addresses, B_i shared-memory descriptors); the first `fresh` of them
// overwrite their accumulators instead.
__device__ __forceinline__ void mma4_ts_elect(const uint32_t (&d)[4], const uint32_t (&a)[4], const uint64_t (&b)[4],
                                              uint32_t idesc, uint32_t fresh) {
  asm volatile(
      "{\n\t.reg .pred e, p0, p1, p2, p3;\n\t.reg .b32 r;\n\t"
      "setp.le.u32 p0, %13, 0;\n\tsetp.le.u32 p1, %13, 1;\n\tsetp.le.u32 p2, %13, 2;\n\tsetp.le.u32 p3, %13, 3;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %12, p0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%1], [%5], %9, %12, p1;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%2], [%6], %10, %12, p2;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%3], [%7], %11, %12, p3;\n\t}\n" ::"r"(d[0]),
      "r"(d[1]), "r"(d[2]), "r"(d[3]), "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]),
      "l"(b[3]), "r"(idesc), "r"(fresh));
}
// Bounded wait by a whole warp, with the first test inline.
__device__ __forceinline__ bool warp_wait_fast(uint64_t* bar, uint32_t parity, uint32_t* err,
                                               volatile uint32_t* abort_flag);
__device__ __forceinline__ void mma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\telect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(smem_u32(bar))
      : "memory");
}

// Which block column each activation slot holds (8 bits per slot, 0xFF: none)
// and the parity of each slot's copy count, in registers (slot indices are
// not compile-time constants, so an array would live in local memory).
struct SlotTable {
  uint32_t w[4], par;
  __device__ __forceinline__ void clear() { w[0] = w[1] = w[2] = w[3] = 0xFFFFFFFFu, par = 0u; }
  __device__ __forceinline__ uint32_t get(uint32_t s) const {
    const uint32_t x = s < 8u ? (s < 4u ? w[0] : w[1]) : (s < 12u ? w[2] : w[3]);
    return (x >> (8u * (s & 3u))) & 0xFFu;
  }
  __device__ __forceinline__ void set(uint32_t s, uint32_t v) {
    const uint32_t sh = 8u * (s & 3u), keep = ~(0xFFu << sh), put = (v & 0xFFu) << sh, i = s >> 2;
#pragma unroll
    for (uint32_t k = 0; k < 4u; ++k) w[k] = i == k ? (w[k] & keep) | put : w[k];
  }
};
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded wait by every lane of a warp whose later tcgen05.ld / st must run
// converged: the outcome and the CTA's abort flag are made warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t* err,
                                          volatile uint32_t* abort_flag) {
  const bool ok = *abort_flag == 0u && mbar_wait(bar, parity, err);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ bool warp_wait_fast(uint64_t* bar, uint32_t parity, uint32_t* err,
                                               volatile uint32_t* abort_flag) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  return warp_wait(bar, parity, err, abort_flag);
}

// ------------------------------------------------------------- dequantizers
// Scale operands of one thread's four Q4_K groups: the thread (j) of row m
// expands groups 2j, 2j+1 (half 0) and 4+2j, 5+2j (half 1), i.e. the
// header's 6-bit scale / min fields at bytes 4+2j.., 8+2j.., 12+2j..
// (get_scale_min_k4 order, resident_quant.glsl:10-15).
struct Q4Scales {
  __half2 s[4], k[4];  // per group g of (2j, 2j+1, 4+2j, 5+2j): sc/16 and -72 sc (both exact in fp16)
  uint32_t mins[2];    // fp16 pairs 2^6 (8 d sc - dmin m) of groups (2j, 2j+1) and (4+2j, 5+2j)
};
__device__ __forceinline__ Q4Scales q4_scales(const uint4& hdr, uint32_t j, float d64, float dmin64) {
  const uint32_t sh = 16u * j;
  const uint32_t Y = hdr.y >> sh, Z = hdr.z >> sh, W = hdr.w >> sh;  // bytes 4+2j.., 8+2j.., 12+2j.. in bits 0-15
  const uint32_t sc[4] = {Y & 63u, (Y >> 8) & 63u, (W & 15u) | ((Y >> 2) & 48u), ((W >> 8) & 15u) | ((Y >> 10) & 48u)};
  const uint32_t mn[4] = {Z & 63u, (Z >> 8) & 63u, ((W >> 4) & 15u) | ((Z >> 2) & 48u),
                          ((W >> 12) & 15u) | ((Z >> 10) & 48u)};
  Q4Scales r;
  float c[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float f = static_cast<float>(sc[g]);
    r.s[g] = __float2half2_rn(f * 0.0625f);
    r.k[g] = __float2half2_rn(-72.f * f);
    c[g] = 8.f * d64 * f - dmin64 * static_cast<float>(mn[g]);
  }
  r.mins[0] = h2_bits(__floats2half2_rn(c[0], c[1]));
  r.mins[1] = h2_bits(__floats2half2_rn(c[2], c[3]));
  return r;
}

// Sixteen coefficients of each group of one Q4_K group pair of row m (one
// 16-byte part of the pair's 32 code bytes: coefficients 16 wh .. +15 of the
// low group in the low nibbles, of the high group in the high nibbles) ->
// fp16 pairs 2^6 d sc (q - 8), eight per group, for tensor memory.  The panel
// stores each 4-byte word of codes as bytes (0, 2, 1, 3), so one mask-and-or
// of the word, or of the word shifted by 4 or 8 bits, puts two consecutive
// coefficients' nibbles at bits 4-7 of the two halves under the exponent byte
// 0x64: 1024 + 16q.  One fp16 FMA (1024 + 16q) * (sc/16) - 72 sc = sc (q - 8)
// is exact (every operand and the result are small integers or sc/16), and
// the product with 2^6 d is the one rounding.  The centring on 8 keeps the
// operand and the mins term small next to the weight they sum to.
__device__ __forceinline__ void expand_q4(const uint4& c, __half2 slo, __half2 klo, __half2 shi, __half2 khi,
                                          __half2 dd, uint32_t (&lo)[8], uint32_t (&hi)[8]) {
  constexpr uint32_t kMask = 0x00F000F0u, kMagic = 0x64006400u;
  const uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t x = words[w];
    lo[2 * w] = hmul2_bits(hfma2_bits(((x << 4) & kMask) | kMagic, slo, klo), dd);      // coefficients 4w, 4w+1
    lo[2 * w + 1] = hmul2_bits(hfma2_bits(((x >> 4) & kMask) | kMagic, slo, klo), dd);  // 4w+2, 4w+3
    hi[2 * w] = hmul2_bits(hfma2_bits((x & kMask) | kMagic, shi, khi), dd);             // the same of the high group
    hi[2 * w + 1] = hmul2_bits(hfma2_bits(((x >> 8) & kMask) | kMagic, shi, khi), dd);
  }
}

// Sixteen coefficients of each run of one Q6_K run pair of row m, half h:
// coefficients 128h + 32j + 16wh .. +15 (low run) and 128h + 64 + 32j + 16wh
// .. +15 (high run) -> fp16 sc (q - 32) times 2^6 d, eight pairs per run.  ql
// holds the runs' 16 ql bytes (low nibbles: low run, high nibbles: high run),
// qh the 16 qh bytes (bit pairs 2j and 4+2j).  Each fp16 pair is assembled by
// one bit-select of two byte permutes: the nibble (at bits 4-7) and the 0x64
// exponent byte from the ql permute, the two high bits (at bits 8-9) from the
// permute of the pre-shifted qh word: 0x6400 | 16q = 1024 + 16q, then
// (1024 + 16q)*(sc/16) - 96*sc = sc*(q-32).
__device__ __forceinline__ void expand_q6(const uint4& ql, const uint4& qh, const uint4& s4, uint32_t h, uint32_t j,
                                          uint32_t wh, __half2 dd, uint32_t (&lo)[8], uint32_t (&hi)[8]) {
  const uint32_t qlw[4] = {ql.x, ql.y, ql.z, ql.w};
  const uint32_t qhw[4] = {qh.x, qh.y, qh.z, qh.w};
  // int8 scales 8h + 2j + wh (low run) and 8h + 4 + 2j + wh (high run): byte 2j + wh of words 2h and 2h + 1
  const uint32_t sl_w = h ? s4.z : s4.x, sh_w = h ? s4.w : s4.y;
  const float a = static_cast<float>(static_cast<int8_t>((sl_w >> (8u * (2u * j + wh))) & 0xFFu));
  const float b = static_cast<float>(static_cast<int8_t>((sh_w >> (8u * (2u * j + wh))) & 0xFFu));
  const __half2 sl = __float2half2_rn(a * 0.0625f), kl = __float2half2_rn(-96.f * a);
  const __half2 sh = __float2half2_rn(b * 0.0625f), kh = __float2half2_rn(-96.f * b);
  constexpr uint32_t kSel = 0xFCF0FCF0u;  // bits taken from the ql permute
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t qs = qlw[w] << 4;               // low-run nibbles to bits 4-7 of each byte
    const uint32_t hl = qhw[w] >> (2u * j);        // low-run high bits to bits 0-1 of each byte
    const uint32_t hh = qhw[w] >> (4u + 2u * j);   // high-run high bits to bits 0-1 of each byte
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const uint32_t sel_l = pr == 0 ? 0x5140u : 0x5342u;  // bytes (2pr, 2pr+1) -> low byte of each half
      const uint32_t sel_h = pr == 0 ? 0x1404u : 0x3424u;  // the same bytes -> high byte of each half
      const uint32_t al = __byte_perm(qs, 0x64646464u, sel_l), ah = __byte_perm(qlw[w], 0x64646464u, sel_l);
      const uint32_t bl = __byte_perm(hl, 0u, sel_h), bh = __byte_perm(hh, 0u, sel_h);
      lo[2 * w + pr] = hmul2_bits(hfma2_bits((al & kSel) | (bl & ~kSel), sl, kl), dd);
      hi[2 * w + pr] = hmul2_bits(hfma2_bits((ah & kSel) | (bh & ~kSel), sh, kh), dd);
    }
  }
}

// ---------------------------------------------------------------- the kernel
template <int FMT, int N>
__global__ void __maxnreg__(96) tc_gemm_kernel(const Params p) {  // 19 warps: <= 5 per sub-partition x 96 x 32 <= 16384
  using C = Cfg<FMT>;
  constexpr bool kQ4 = C::kQ4;
  constexpr uint32_t kPanel = C::kPanel, kRawS = C::kRawStages;
  // A unit's sum is spread over kParts accumulators that the K=16 steps of a
  // block column take in turn, so consecutive MMAs do not wait on one another's
  // accumulation (at N <= 64 one MMA's work is shorter than that latency); the
  // epilogue adds the parts.  Two units' accumulators (double buffering):
  // 2 * kParts * N = 256 columns below the A stages.
  constexpr uint32_t kParts = 128u / static_cast<uint32_t>(N);
  constexpr uint32_t kDStride = kParts * static_cast<uint32_t>(N);  // tensor-memory columns of one unit's parts
  constexpr uint32_t kMaxSlots = 4u * 64u / static_cast<uint32_t>(N);
  static_assert(2u * kDStride <= kAColBase, "accumulators overlap the A stages");
  static_assert(kParts <= 8u, "every part takes its first K step in the first half block");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + kRawS;
  // A stage s of a half block: full once the 8 dequantizing warps have written
  // it, empty once the MMAs that read it have completed (one commit)
  uint64_t* ab_full = raw_empty + kRawS;
  uint64_t* ab_empty = ab_full + kAStages;
  uint64_t* d_full = ab_empty + kAStages;
  uint64_t* d_empty = d_full + 2;
  uint64_t* drain = d_empty + 2;
  // activation slot s: full when its block column has landed (expect-tx),
  // empty when the MMAs of the last use of that block column have completed
  uint64_t* b_full = drain + 1;
  uint64_t* b_empty = b_full + kMaxSlots;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + p.off_misc);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(misc + 4);  // [N] argmax candidates

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  uint32_t q0, q1;  // this CTA's panels of the work order
  cta_range(p, q0, q1);
  const uint32_t tiles_per_mat = p.rows / kTileRows;
  auto panel_src = [&](const Walk& w) {
    const uint32_t mat = w.t / tiles_per_mat, mt = w.t % tiles_per_mat;
    return (mat ? p.w[1] : p.w[0]) + (static_cast<size_t>(mt) * p.KB + w.kb) * kPanel;
  };
  uint8_t* raw = smem;
  // Thread 0 initialises the barriers and is also the panel producer: its first
  // kRawS copies (free stages, no wait) leave before the block-wide set-up.
  uint32_t early = 0;  // panel copies issued before the set-up (thread 0)
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kRawS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 8);
    }
    fence_mbar_init();
    const uint64_t policy = evict_first_policy();
    Walk w;
    if (q0 < q1) w.start(p, q0);
    for (uint32_t q = q0; q < q1 && early < kRawS; ++q, ++early, w.next(p)) {
      mbar_expect_tx(&raw_full[early], kPanel);
      bulk_g2s_stream(raw + early * kPanel, panel_src(w), kPanel, &raw_full[early], policy);
    }
    for (uint32_t s = 0; s < kAStages; ++s) {
      mbar_init(&ab_full[s], 8);
      mbar_init(&ab_empty[s], 1);
    }
    for (uint32_t s = 0; s < 2; ++s) {
      mbar_init(&d_full[s], 1);
      mbar_init(&d_empty[s], 8);
    }
    mbar_init(drain, 1);
    for (uint32_t s = 0; s < p.slots; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    fence_mbar_init();
    *abort_flag = 0u;
  }
  for (uint32_t i = threadIdx.x; i < static_cast<uint32_t>(N); i += kThreads) cand[i] = 0ull;
  if (warp == 1) {  // the whole warp allocates all 512 columns (one CTA per SM)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(const_cast<uint32_t*>(tmem_slot))),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();
  uint8_t* bst = smem + p.off_b;
  const uint32_t b_bytes0 = static_cast<uint32_t>(N) * 256u + (kQ4 ? static_cast<uint32_t>(N) * 32u : 0u);

  if (warp == 0) {
    // ----------------------------------------------- weight panel producer
    // Weights never depend on earlier kernels: their copies start at once, so
    // the dequantizers fill tensor memory while the prep kernel still runs.
    if (lane == 0) {
      const uint64_t policy = evict_first_policy();
      uint32_t rit = 0;  // copies issued into the raw ring
      bool stop = false;
      Walk w;
      if (q0 < q1) w.start(p, q0);
      for (uint32_t q = q0; q < q1; ++q, w.next(p)) {
        const uint32_t rs = rit % kRawS;
        if (rit < early) {  // issued before the set-up
          ++rit;
          continue;
        }
        if (*abort_flag || !mbar_wait(&raw_empty[rs], ((rit / kRawS) & 1u) ^ 1u, p.err)) {
          stop = true;
          break;
        }
        mbar_expect_tx(&raw_full[rs], kPanel);
        bulk_g2s_stream(raw + rs * kPanel, panel_src(w), kPanel, &raw_full[rs], policy);
        ++rit;
      }
      if (stop) {
        *abort_flag = 1u;
        // bounded drain: the last copy into each stage has landed before the CTA exits
        for (uint32_t s = 0; s < kRawS; ++s) {
          const uint32_t n = rit / kRawS + (s < rit % kRawS ? 1u : 0u);
          if (n) (void)mbar_wait(&raw_full[s], (n - 1u) & 1u, nullptr);
        }
      }
    }
  } else if (warp == 18) {
    // ------------------------------------------------- activation slot stager
    // A block column is copied into slot kb % slots when the slot holds another
    // one, after the MMAs of that one's last use have released the slot.
    if (lane == 0) {
      SlotTable tab;  // par bit s: copies into slot s so far, mod 2
      tab.clear();
      uint32_t used = 0;  // slots that received a copy
      bool stop = false;
      pdl_wait();  // the activation blocks are written by the preceding prep kernel
      Walk w;
      if (q0 < q1) w.start(p, q0);
      for (uint32_t q = q0; q < q1; ++q, w.next(p)) {
        const uint32_t s = w.kb % p.slots;
        if (tab.get(s) == w.kb) continue;
        // wait for as many releases as copies so far
        if (*abort_flag || !mbar_wait(&b_empty[s], ((tab.par >> s) & 1u) ^ 1u, p.err)) {
          stop = true;
          break;
        }
        mbar_expect_tx(&b_full[s], p.blk);
        bulk_g2s(bst + s * p.b_slot, p.xb + static_cast<size_t>(w.kb) * p.blk, p.blk, &b_full[s]);
        tab.set(s, w.kb);
        tab.par ^= 1u << s;
        used |= 1u << s;
      }
      if (stop) {
        *abort_flag = 1u;
        for (uint32_t s = 0; s < p.slots; ++s)  // the last copy into each used slot (bounded)
          if ((used >> s) & 1u) (void)mbar_wait(&b_full[s], ((tab.par >> s) & 1u) ^ 1u, nullptr);
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    // The whole warp walks the work (warp-uniform), one elected lane issues.
    constexpr uint32_t idesc = instr_desc(N);
    SlotTable tab;
    tab.clear();
    uint32_t ait = 0, u = 0;  // A stages consumed, units begun
    bool stop = false;
    const uint32_t b0 = smem_u32(bst);
    Walk w;
    if (q0 < q1) w.start(p, q0);
    for (uint32_t q = q0; q < q1 && !stop; ++q, w.next(p)) {
      const bool first = q == q0 || w.kb == w.k0, last = q + 1u == q1 || w.kb + 1u == w.k1;
      // one set of accumulators per unit (block scales are in the operand), double-buffered by unit
      const uint32_t buf = u & 1u;
      if (first) {
        if (!warp_wait(&d_empty[buf], ((u >> 1) & 1u) ^ 1u, p.err, abort_flag)) {
          stop = true;
          break;
        }
        tc_fence_after();
      }
      const uint32_t s = w.kb % p.slots;
      if (tab.get(s) != w.kb) {  // the stager copies this block column in: wait for it
        if (!warp_wait(&b_full[s], (tab.par >> s) & 1u, p.err, abort_flag)) {
          stop = true;
          break;
        }
        tab.set(s, w.kb);
        tab.par ^= 1u << s;
      }
      const uint32_t d1 = tmem + buf * kDStride;
      const uint32_t sb = b0 + s * p.b_slot;
#pragma unroll
      for (uint32_t h = 0; h < 2u; ++h) {
        const uint32_t as = ait % kAStages;
        if (!warp_wait_fast(&ab_full[as], (ait / kAStages) & 1u, p.err, abort_flag)) {
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t acol = tmem + kAColBase + 64u * as;
        const uint64_t bd = smem_desc(sb + (h ? b_bytes0 : 0u), 128u, 2048u);  // + 16 per K step (256 bytes)
        const uint32_t fresh = (first && h == 0u) ? kParts : 0u;  // each part's first step overwrites it
#pragma unroll
        for (uint32_t k4 = 0; k4 < 8u; k4 += 4u) {
          uint32_t dd[4], aa[4];
          uint64_t bb[4];
#pragma unroll
          for (uint32_t i = 0; i < 4u; ++i) {
            dd[i] = d1 + ((k4 + i) % kParts) * static_cast<uint32_t>(N);
            aa[i] = acol + 8u * (k4 + i);
            bb[i] = bd + 16u * (k4 + i);
          }
          mma4_ts_elect(dd, aa, bb, idesc, fresh > k4 ? fresh - k4 : 0u);
        }
        if (kQ4 && h == 0u)  // mins term: c_G against the group sums (hi, lo), into part 0
          mma_ts_elect(d1, tmem + kA2ColBase + 8u * as, smem_desc(sb + static_cast<uint32_t>(N) * 256u, 128u, 256u),
                       idesc, 1u);
        mma_commit_elect(&ab_empty[as]);
        ++ait;
      }
      if (stop) break;
      if (slot_changes(p, w, q, q1)) mma_commit_elect(&b_empty[s]);  // the slot's next use is another block column
      if (last) {
        mma_commit_elect(&d_full[buf]);
        ++u;
      }
    }
    if (stop) *abort_flag = 1u;
    mma_commit_elect(drain);  // every MMA issued above has completed once this arrives
    (void)mbar_wait(drain, 0u, nullptr);
    __syncwarp();
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------- epilogue
    const uint32_t NB = p.split ? static_cast<uint32_t>(N) / 2u : static_cast<uint32_t>(N);  // batch columns
    const uint32_t NH = NB / 2u;  // batch columns of this warp (<= 32)
    const uint32_t qd = warp & 3u, m = 32u * qd + lane, c0 = (warp - 2u) >> 2;  // columns c0*NH ..
    const uint32_t lane_addr = (32u * qd) << 16;
    pdl_wait();  // residual targets and running flags are written by earlier kernels
    uint32_t live = 0;  // bit i: batch column c0*NH + i is in the launch and still generating
    for (uint32_t i = 0; i < NH; ++i) {
      const uint32_t n = c0 * NH + i;
      if (n < p.batch && (!p.running || p.running[static_cast<size_t>(n) * p.run_step] != 0u)) live |= 1u << i;
    }
    bool stop = false;
    Walk w;
    if (q0 < q1) w.start(p, q0);
    for (uint32_t q = q0, u = 0; q < q1 && !stop; ++u) {
      const uint32_t t = w.t;
      const uint32_t len = min(q1 - q, w.k1 - w.kb);  // panels of this unit
      for (uint32_t i = 0; i < len; ++i) w.next(p);
      q += len;
      const uint32_t mat = t / tiles_per_mat, mt = t % tiles_per_mat;
      const uint32_t R = mat * p.rows + mt * kTileRows + m;  // this thread's output row
      // the unit's whole sum (block scales were folded into the operand)
      const uint32_t buf = u & 1u;
      if (!warp_wait(&d_full[buf], (u >> 1) & 1u, p.err, abort_flag)) {
        stop = true;
        break;
      }
      tc_fence_after();
      const uint32_t dcol = tmem + lane_addr + buf * kDStride + c0 * NH;  // part 0; part i at + i * N
      // eight columns at a time: a warp's 32 rows of one column are one 128-byte
      // line, so scalar atomics of partial sums cost one L2 line operation per instruction
#pragma unroll 1
      for (uint32_t c = 0; c < NH; c += 8u) {
        float v[8];
        tmem_ld8(dcol + c, v);
#pragma unroll
        for (uint32_t i = 1; i < kParts; ++i) {
          float v2[8];
          tmem_ld8(dcol + c + i * static_cast<uint32_t>(N), v2);
          tmem_wait_ld();
#pragma unroll
          for (uint32_t e = 0; e < 8u; ++e) v[e] += v2[e];
        }
        if (p.split) {  // + the products of the remainders (D columns N/2 on)
#pragma unroll
          for (uint32_t i = 0; i < kParts; ++i) {
            float v2[8];
            tmem_ld8(dcol + c + static_cast<uint32_t>(N) / 2u + i * static_cast<uint32_t>(N), v2);
            tmem_wait_ld();
#pragma unroll
            for (uint32_t e = 0; e < 8u; ++e) v[e] += v2[e];
          }
        }
        tmem_wait_ld();
        if (p.y) {
          float* yp = p.y + static_cast<size_t>(c0 * NH + c) * p.y_stride + R;
          if (!p.whole_tiles) {  // partial sum of one K range (into the residual, or into rows the prep zeroed)
#pragma unroll
            for (uint32_t e = 0; e < 8u; ++e)
              if ((live >> (c + e)) & 1u) atomicAdd(yp + static_cast<size_t>(e) * p.y_stride, v[e] * (1.0f / kOperandScale));
          } else {
#pragma unroll
            for (uint32_t e = 0; e < 8u; ++e) {
              if (!((live >> (c + e)) & 1u)) continue;
              float* ye = yp + static_cast<size_t>(e) * p.y_stride;
              *ye = (p.epilogue == kAccumulate ? *ye : 0.f) + v[e] * (1.0f / kOperandScale);
            }
          }
        }
        if (p.argmax) {
#pragma unroll
          for (uint32_t e = 0; e < 8u; ++e) {
            unsigned long long key = pack_argmax(v[e] * (1.0f / kOperandScale), R);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
              const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
              key = other > key ? other : key;
            }
            if (lane == 0 && ((live >> (c + e)) & 1u)) atomicMax(&cand[c0 * NH + c + e], key);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&d_empty[buf])) : "memory");
    }
    if (stop) *abort_flag = 1u;
  } else if (warp >= 10 && warp < 18) {
    // ---------------------------------------------------------- dequantizers
    // Warp (quarter qd, j): rows 32 qd .. +31; of each half block, the pair of
    // groups j (Q4_K) or run pair j (Q6_K).  Each half is expanded into
    // registers before its stage is waited for.
    const uint32_t qd = warp & 3u, j = (warp - 10u) >> 2, m = 32u * qd + lane;
    const uint32_t lane_addr = (32u * qd) << 16;
    uint32_t rit = 0, ait = 0;
    bool stop = false;
    for (uint32_t q = q0; q < q1 && !stop; ++q) {
      const uint32_t rs = rit % kRawS;
      if (!warp_wait_fast(&raw_full[rs], (rit / kRawS) & 1u, p.err, abort_flag)) {
        stop = true;
        break;
      }
      const uint8_t* panel = raw + rs * kPanel;
      // everything this thread needs from the panel, then the panel is released
      uint4 hdr, c[2][2], g[2][2];  // header / int8 scales of row m; codes (Q4_K) or ql and qh (Q6_K) [half][part]
      uint32_t scale_word;
      if constexpr (kQ4) {
        hdr = *reinterpret_cast<const uint4*>(panel + 16384u + 16u * m);
        scale_word = hdr.x;  // d, dmin
#pragma unroll
        for (uint32_t h = 0; h < 2u; ++h)
#pragma unroll
          for (uint32_t wh = 0; wh < 2u; ++wh)  // codes [pl 4][part 2][row 128][16 B], pl = 2h + j
            c[h][wh] = *reinterpret_cast<const uint4*>(panel + (((2u * h + j) * 2u + wh) * 128u + m) * 16u);
      } else {
        hdr = *reinterpret_cast<const uint4*>(panel + 24576u + 16u * m);
        scale_word = *reinterpret_cast<const unsigned short*>(panel + 26624u + 2u * m);  // d
#pragma unroll
        for (uint32_t h = 0; h < 2u; ++h)
#pragma unroll
          for (uint32_t wh = 0; wh < 2u; ++wh) {  // per half: ql [j 2][part 2][row][16 B], then qh [part 2][row][16 B]
            const uint8_t* base = panel + h * 12288u;
            c[h][wh] = *reinterpret_cast<const uint4*>(base + ((j * 2u + wh) * 128u + m) * 16u);
            g[h][wh] = *reinterpret_cast<const uint4*>(base + 8192u + (wh * 128u + m) * 16u);
          }
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&raw_empty[rs])) : "memory");
      ++rit;
      // the row's block scale (and Q4_K min scale) times 2^6, folded into the operand
      const float d64 = kOperandScale * half_bits_to_float(scale_word & 0xFFFFu);
      const __half2 dd = __float2half2_rn(d64);
      Q4Scales sc4;
      if constexpr (kQ4) sc4 = q4_scales(hdr, j, d64, kOperandScale * half_bits_to_float(scale_word >> 16));
      uint32_t lo[16], hi[16];
      auto expand = [&](uint32_t h) {
#pragma unroll
        for (uint32_t wh = 0; wh < 2u; ++wh) {
          uint32_t(&l8)[8] = *reinterpret_cast<uint32_t(*)[8]>(&lo[8u * wh]);
          uint32_t(&h8)[8] = *reinterpret_cast<uint32_t(*)[8]>(&hi[8u * wh]);
          if constexpr (kQ4)
            expand_q4(c[h][wh], sc4.s[2u * h], sc4.k[2u * h], sc4.s[2u * h + 1u], sc4.k[2u * h + 1u], dd, l8, h8);
          else
            expand_q6(c[h][wh], g[h][wh], hdr, h, j, wh, dd, l8, h8);
        }
      };
      expand(0u);
#pragma unroll
      for (uint32_t h = 0; h < 2u; ++h) {
        const uint32_t as = ait % kAStages;
        if (!warp_wait_fast(&ab_empty[as], ((ait / kAStages) & 1u) ^ 1u, p.err, abort_flag)) {
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t tcol = tmem + lane_addr + kAColBase + 64u * as;
        if constexpr (kQ4) {  // group pair j: low group at columns 32 j.., high group at 32 j + 16..
          tmem_st16(tcol + 32u * j, lo);
          tmem_st16(tcol + 32u * j + 16u, hi);
          if (h == 0u) {  // the mins pairs of groups (2j, 2j+1, 4+2j, 5+2j), against the hi and the lo sums
            const uint32_t mv[4] = {sc4.mins[0], sc4.mins[1], sc4.mins[0], sc4.mins[1]};
            tmem_st4(tmem + lane_addr + kA2ColBase + 8u * as + 4u * j, mv);
          }
        } else {  // run pair j: low runs at columns 16 j.., high runs at 32 + 16 j..
          tmem_st16(tcol + 16u * j, lo);
          tmem_st16(tcol + 32u + 16u * j, hi);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&ab_full[as])) : "memory");
        ++ait;
        if (h == 0u) expand(1u);  // half 1 before its stage is waited for
      }
    }
    if (stop) *abort_flag = 1u;
  }

  // argmax candidates of this CTA -> the global keys (epilogue warps only)
  if (warp >= 2 && warp < 10) {
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const uint32_t t = threadIdx.x - 64u;
    if (p.argmax && t < (p.split ? static_cast<uint32_t>(N) / 2u : static_cast<uint32_t>(N)) && t < p.batch && cand[t])
      atomicMax(p.argmax + static_cast<size_t>(t) * p.arg_step, cand[t]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// -------------------------------------------------------- activation prep
// Batch row n, columns [kPrepCols*blockIdx.y, +kPrepCols) (one CTA): prologue,
// x -> fp16 in the K-major core-matrix layout of the activation stages, and
// (Q4_K) the fp32 32-group sums of the fp16 x as fp16 hi / lo.  Rows past the
// batch, or of stopped sequences, are written as zeros.  The RMS norm's sum
// runs over the whole row in every chunk (an L2-resident re-read).
__global__ void __launch_bounds__(256) tc_prep_kernel(const Prep p) {
  __shared__ float red[8];
  const uint32_t n = blockIdx.x, tid = threadIdx.x, lane = tid & 31u;
  // split stages: CTA n >= N/2 writes the fp16 remainders of batch row n - N/2
  const uint32_t nr = p.split ? n % (p.N / 2u) : n;
  const bool rem = p.split && n >= p.N / 2u;
  pdl_wait();
  pdl_launch_dependents();
  const bool live = nr < p.batch && (!p.running || p.running[static_cast<size_t>(nr) * p.run_step] != 0u);
  if (live && p.zero_y && !rem) {  // this chunk's share of the output row
    const uint32_t per = (p.zero_cols + gridDim.y - 1u) / gridDim.y;
    const uint32_t a = blockIdx.y * per, b = min(p.zero_cols, a + per);
    float* yr = p.zero_y + static_cast<size_t>(nr) * p.zero_stride;
    for (uint32_t c = a + tid; c < b; c += 256u) yr[c] = 0.f;
  }
  const float* xr = p.x + static_cast<size_t>(nr < p.batch ? nr : 0u) * p.x_stride;
  const float* zr = p.z ? p.z + static_cast<size_t>(nr < p.batch ? nr : 0u) * p.z_stride : nullptr;
  const uint32_t nch = p.cols / 8u;
  float inv = 1.f;
  if (live && p.prologue == kRmsNorm) {
    float s = 0.f;
    for (uint32_t c = tid; c < nch; c += 256u) {
      const float4 a = reinterpret_cast<const float4*>(xr)[2u * c];
      const float4 b = reinterpret_cast<const float4*>(xr)[2u * c + 1u];
      s += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    }
    s = warp_sum(s);
    if (lane == 0) red[tid >> 5] = s;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w];
    inv = rsqrtf(t / static_cast<float>(p.cols) + p.eps);
  }
  const uint32_t N = p.N;
  const uint32_t c_end = min(nch, (blockIdx.y + 1u) * (kPrepCols / 8u));
  for (uint32_t c = blockIdx.y * (kPrepCols / 8u) + tid; c < c_end; c += 256u) {  // a warp: 32 consecutive 8-chunks
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (live) {
      const float4 a = reinterpret_cast<const float4*>(xr)[2u * c];
      const float4 b = reinterpret_cast<const float4*>(xr)[2u * c + 1u];
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
      float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (zr) {
        const float4 za = reinterpret_cast<const float4*>(zr)[2u * c];
        const float4 zb = reinterpret_cast<const float4*>(zr)[2u * c + 1u];
        z[0] = za.x, z[1] = za.y, z[2] = za.z, z[3] = za.w, z[4] = zb.x, z[5] = zb.y, z[6] = zb.z, z[7] = zb.w;
      }
      if (p.prologue == kRmsNorm) {
        const float4 wa = reinterpret_cast<const float4*>(p.norm_w)[2u * c];
        const float4 wb = reinterpret_cast<const float4*>(p.norm_w)[2u * c + 1u];
        const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * inv * w[e];
      } else if (p.prologue == kHeadGate) {  // one 128-wide head = 16 chunks = half a warp
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) s += v[e] * v[e];
#pragma unroll
        for (int o = 8; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float hinv = rsqrtf(s / 128.0f + p.eps);
        const float4 wa = reinterpret_cast<const float4*>(p.norm_w)[2u * c];
        const float4 wb = reinterpret_cast<const float4*>(p.norm_w)[2u * c + 1u];
        const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * (((hinv * w[e]) * z[e]) * detector_sigmoid(z[e]));
      } else if (p.prologue == kSigmoidGate) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = v[e] * detector_sigmoid(z[e]);
      } else if (p.prologue == kSwiGLUIn) {  // x = gate, z = up: the SwiGLU activation of op 2 kind 3
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float gv = v[e], uv = z[e];
          const float amp = fabsf(gv) * fabsf(uv) * detector_sigmoid(gv);
          const float sgn = (gv > 0.f ? 1.f : gv < 0.f ? -1.f : 0.f) * (uv > 0.f ? 1.f : uv < 0.f ? -1.f : 0.f);
          v[e] = sgn * amp;
        }
      }
    }
    const uint32_t k = 8u * c, kb = k / 256u, h = (k / 128u) & 1u, kc = (k % 128u) / 8u;
    uint8_t* dst = p.xb + static_cast<size_t>(kb) * p.blk + (h ? N * 256u + (p.q4 ? N * 32u : 0u) : 0u) +
                   (n / 8u) * 2048u + kc * 128u + (n % 8u) * 16u;
    __half2 hv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      hv[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
      if (rem)  // the remainder x - fp16(x), itself rounded to fp16 (x = hi + lo to about 2^-22)
        hv[e] = __floats2half2_rn(v[2 * e] - __low2float(hv[e]), v[2 * e + 1] - __high2float(hv[e]));
    }
    *reinterpret_cast<uint4*>(dst) = make_uint4(h2_bits(hv[0]), h2_bits(hv[1]), h2_bits(hv[2]), h2_bits(hv[3]));
    if (p.q4) {  // 32-group sum of the fp16 x over 4 consecutive chunks (lanes 4i..4i+3)
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) s += __low2float(hv[e]) + __high2float(hv[e]);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if ((c & 3u) == 0u) {
        // K order of the mins product: the dequantizing thread j holds the mins of
        // groups (2j, 2j+1, 4+2j, 5+2j) in its four columns, against the hi sums
        // and then the lo sums: K = 8j + 4 part + 2 (g >> 2) + (g & 1), j = (g >> 1) & 1
        const uint32_t G = c / 4u, g8 = G % 8u;
        const __half hi = __float2half_rn(s);
        const __half lo = __float2half_rn(s - __half2float(hi));
        uint8_t* b2 = p.xb + static_cast<size_t>(G / 8u) * p.blk + N * 256u + (n / 8u) * 256u + (n % 8u) * 16u +
                      ((g8 >> 1) & 1u) * 128u;
        const uint32_t e = 2u * (g8 >> 2) + (g8 & 1u);
        reinterpret_cast<__half*>(b2)[e] = hi;
        reinterpret_cast<__half*>(b2)[4u + e] = lo;
      }
    }
  }
}

// act[r][c] = swiglu(gu[r][c], gu[r][F + c]) (op 2 kind 3's epilogue, for the
// callers that need the activation rows themselves).
__global__ void swiglu_rows_kernel(const float* __restrict__ gu, uint32_t rows, uint32_t F, uint32_t gu_stride,
                                   float* __restrict__ act, uint32_t act_stride) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(rows) * F) return;
  const uint32_t r = static_cast<uint32_t>(i / F), c = static_cast<uint32_t>(i % F);
  const float gv = gu[static_cast<size_t>(r) * gu_stride + c], uv = gu[static_cast<size_t>(r) * gu_stride + F + c];
  const float amp = fabsf(gv) * fabsf(uv) * detector_sigmoid(gv);
  const float sgn = (gv > 0.f ? 1.f : gv < 0.f ? -1.f : 0.f) * (uv > 0.f ? 1.f : uv < 0.f ? -1.f : 0.f);
  act[static_cast<size_t>(r) * act_stride + c] = sgn * amp;
}

// ------------------------------------------------------------- panel tiler
// grid (KB, rows / 128); one panel per CTA.
template <int FMT>
__global__ void __launch_bounds__(256) tile_tc_kernel(const uint8_t* __restrict__ src, uint32_t KB,
                                                      uint8_t* __restrict__ dst) {
  constexpr uint32_t BB = FMT == kQ4K ? kQ4KBytes : kQ6KBytes, PB = 128u * BB;
  const uint32_t kb = blockIdx.x, T = blockIdx.y;
  const uint8_t* rows = src + (static_cast<size_t>(T) * 128u * KB + kb) * BB;  // row r block: rows + r*KB*BB
  uint8_t* out = dst + (static_cast<size_t>(T) * KB + kb) * PB;
  for (uint32_t o = threadIdx.x; o < PB; o += blockDim.x) {
    uint32_t r, b;  // source row and byte within its block
    if constexpr (FMT == kQ4K) {
      if (o < 16384u) {  // each 4-byte word of codes as bytes (0, 2, 1, 3): the dequantizer's nibble order
        const uint32_t pl = o / 4096u, part = (o / 2048u) & 1u, i = o % 16u;
        const uint32_t src = (i & ~3u) | ((i & 1u) << 1) | ((i >> 1) & 1u);
        r = (o / 16u) & 127u;
        b = 16u + 32u * pl + 16u * part + src;
      } else {
        r = (o - 16384u) / 16u;
        b = o % 16u;
      }
    } else {
      if (o < 24576u) {
        const uint32_t h = o / 12288u, x = o % 12288u;
        if (x < 8192u) {
          const uint32_t jj = x / 4096u, part = (x / 2048u) & 1u;
          r = (x / 16u) & 127u;
          b = 64u * h + 32u * jj + 16u * part + x % 16u;
        } else {
          const uint32_t y = x - 8192u, part = y / 2048u;
          r = (y / 16u) & 127u;
          b = 128u + 32u * h + 16u * part + y % 16u;
        }
      } else if (o < 26624u) {
        r = (o - 24576u) / 16u;
        b = 192u + o % 16u;
      } else {
        r = (o - 26624u) / 2u;
        b = 208u + o % 2u;
      }
    }
    out[o] = rows[static_cast<size_t>(r) * KB * BB + b];
  }
}

}  // namespace tc

// ------------------------------------------------------------------- host
namespace {
template <int FMT, int N>
cudaError_t launch_n(const tc::Params& p0, const tc::Prep& pr, uint32_t grid, bool pdl, cudaStream_t s) {
  using C = tc::Cfg<FMT>;
  tc::Params p = p0;
  p.b_slot = (tc::blk_bytes(C::kQ4, N) + 1023u) / 1024u * 1024u;
  p.off_b = C::kRawStages * C::kPanel;
  p.off_b = (p.off_b + 1023u) / 1024u * 1024u;
  p.off_bar = p.off_b + p.slots * p.b_slot;
  p.off_misc = p.off_bar + 512u;
  uint32_t smem = p.off_misc + 16u + 8u * static_cast<uint32_t>(N);
  smem = smem < tc::kMinSmem ? tc::kMinSmem : smem;
  auto kernel = tc::tc_gemm_kernel<FMT, N>;
  // once per (kernel, device), under a lock: host threads may make their first
  // calls at the same time; the flag is published with release order
  static std::mutex attr_mutex;
  static std::atomic<int> attr_done[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(attr_mutex);
    if (!attr_done[dev].load(std::memory_order_relaxed)) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
      if (e != cudaSuccess) return e;
      attr_done[dev].store(1, std::memory_order_release);
    }
  }
  if (smem > 227u * 1024u) return cudaErrorInvalidConfiguration;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pr.N, (pr.cols + tc::kPrepCols - 1u) / tc::kPrepCols);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, tc::tc_prep_kernel, pr);
  if (e == cudaSuccess) {
    attr[0].val.programmaticStreamSerializationAllowed = 1;  // overlaps its set-up with the prep kernel
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(tc::kThreads);
    cfg.dynamicSmemBytes = smem;
    e = cudaLaunchKernelEx(&cfg, kernel, p);
  }
  if (e != cudaSuccess) (void)cudaGetLastError();  // a refused launch is reported here, not to the next call
  return e;
}

template <int FMT>
cudaError_t launch_fmt(const tc::Params& p, const tc::Prep& pr, uint32_t grid, bool pdl, cudaStream_t s) {
  switch (pr.N) {
    case 16: return launch_n<FMT, 16>(p, pr, grid, pdl, s);
    case 32: return launch_n<FMT, 32>(p, pr, grid, pdl, s);
    case 64: return launch_n<FMT, 64>(p, pr, grid, pdl, s);
    case 128: return launch_n<FMT, 128>(p, pr, grid, pdl, s);  // split stages of 64 batch rows
    default: return cudaErrorInvalidValue;
  }
}

uint32_t tile_n(uint32_t rows) { return rows <= 16u ? 16u : rows <= 32u ? 32u : 64u; }
}  // namespace

size_t tc_workspace_bytes(int fmt, uint32_t batch, uint32_t cols, bool split) {
  const bool q4 = fmt == kQ4KPanel || fmt == kQ4K;
  const uint32_t N = tile_n(batch < kTcMaxN ? batch : kTcMaxN) * (split ? 2u : 1u);
  return static_cast<size_t>(cols / 256u) * tc::blk_bytes(q4, N);
}

cudaError_t launch_tc_gemm(const TcGemmArgs& a, cudaStream_t s) {
  if (a.fmt != kQ4KPanel && a.fmt != kQ6KPanel) return cudaErrorInvalidValue;
  const bool q4 = a.fmt == kQ4KPanel;
  if (!a.w0 || !a.x || !a.xb || a.rows == 0 || a.rows % tc::kTileRows || a.cols == 0 || a.cols % 256u ||
      a.batch == 0 || a.batch > kMaxBatch || (!a.y && !a.argmax))
    return cudaErrorInvalidValue;
  if ((a.prologue == kHeadGate || a.prologue == kSigmoidGate || a.prologue == kSwiGLUIn) && !a.z)
    return cudaErrorInvalidValue;
  if ((a.prologue == kRmsNorm || a.prologue == kHeadGate) && !a.norm_w) return cudaErrorInvalidValue;
  if (a.prologue == kHeadGate && a.cols % 128u) return cudaErrorInvalidValue;
  if (a.epilogue != kStore && a.epilogue != kAccumulate) return cudaErrorInvalidValue;
  if (a.xb_bytes < tc_workspace_bytes(a.fmt, a.batch, a.cols, a.split)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.w0) | reinterpret_cast<uintptr_t>(a.w1) | reinterpret_cast<uintptr_t>(a.xb) |
       reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.z)) & 15u)
    return cudaErrorInvalidValue;
  if (a.x_stride % 4u || (a.z && (a.z_stride ? a.z_stride : a.x_stride) % 4u)) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint32_t nmat = a.w1 ? 2u : 1u, ntiles = nmat * (a.rows / tc::kTileRows), KB = a.cols / 256u;
  // Work split.  Without an argmax every CTA takes an equal contiguous range of
  // the panels in tile-major order, activations streamed through the slots;
  // partial sums land atomically (residual products add into y, stores into
  // rows the prep kernel zeroes).  The argmax needs whole sums: whole tiles per
  // CTA.
  const bool whole = a.argmax != nullptr || !a.y;
  const uint32_t total = ntiles * KB;
  const uint32_t grid = whole ? (ntiles < static_cast<uint32_t>(sms) ? ntiles : static_cast<uint32_t>(sms))
                              : (total < static_cast<uint32_t>(sms) ? total : static_cast<uint32_t>(sms));
  // batch rows run in launches of at most kTcMaxN (each streams the weights once)
  for (uint32_t b0 = 0; b0 < a.batch; b0 += kTcMaxN) {
    const uint32_t nb = a.batch - b0 < kTcMaxN ? a.batch - b0 : kTcMaxN;
    tc::Prep pr = {};
    pr.x = a.x + static_cast<size_t>(b0) * a.x_stride;
    pr.x_stride = a.x_stride;
    const uint32_t zs = a.z_stride ? a.z_stride : a.x_stride;
    pr.z = a.z ? a.z + static_cast<size_t>(b0) * zs : nullptr;
    pr.z_stride = zs;
    pr.norm_w = a.norm_w;
    pr.eps = a.eps;
    pr.prologue = a.prologue;
    pr.cols = a.cols;
    pr.batch = nb;
    pr.N = tile_n(nb) * (a.split ? 2u : 1u);  // split: hi and lo stages of every row
    pr.split = a.split;
    const uint32_t rstep = a.running_step ? a.running_step : 1u;
    pr.running = a.running ? a.running + static_cast<size_t>(b0) * rstep : nullptr;
    pr.run_step = rstep;
    pr.xb = a.xb;
    pr.blk = tc::blk_bytes(q4, pr.N);
    pr.q4 = q4;
    if (!whole && a.epilogue == kStore) {
      pr.zero_y = a.y + static_cast<size_t>(b0) * a.y_stride;
      pr.zero_cols = nmat * a.rows;
      pr.zero_stride = a.y_stride;
    }
    tc::Params p = {};
    p.w[0] = a.w0;
    p.w[1] = a.w1 ? a.w1 : a.w0;
    p.nmat = nmat;
    p.rows = a.rows;
    p.KB = a.cols / 256u;
    p.ntiles = ntiles;
    p.slots = 4u * 64u / pr.N;
    p.width = KB;
    p.total = total;
    p.whole_tiles = whole ? 1u : 0u;
    p.split = a.split ? 1u : 0u;

    p.xb = a.xb;
    p.blk = pr.blk;
    p.batch = nb;
    p.y = a.y ? a.y + static_cast<size_t>(b0) * a.y_stride : nullptr;
    p.y_stride = a.y_stride;
    p.epilogue = a.epilogue;
    const uint32_t astep = a.argmax_step ? a.argmax_step : 1u;
    p.argmax = a.argmax ? a.argmax + static_cast<size_t>(b0) * astep : nullptr;
    p.arg_step = astep;
    p.running = pr.running;
    p.run_step = rstep;
    p.err = a.err;
    e = q4 ? launch_fmt<kQ4K>(p, pr, grid, a.pdl || b0 > 0, s) : launch_fmt<kQ6K>(p, pr, grid, a.pdl || b0 > 0, s);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_swiglu_rows(const float* gu, uint32_t rows, uint32_t F, uint32_t gu_stride, float* act,
                               uint32_t act_stride, cudaStream_t s) {
  if (!gu || !act || rows == 0 || F == 0) return cudaErrorInvalidValue;
  const size_t n = static_cast<size_t>(rows) * F;
  tc::swiglu_rows_kernel<<<static_cast<uint32_t>((n + 255) / 256), 256, 0, s>>>(gu, rows, F, gu_stride, act, act_stride);
  return cudaGetLastError();
}

cudaError_t launch_tile_tc(int fmt, const uint8_t* src, uint32_t rows, uint32_t cols, uint8_t* dst, cudaStream_t s) {
  if ((fmt != kQ4K && fmt != kQ6K) || !src || !dst || src == dst || rows == 0 || rows % tc::kTileRows || cols == 0 ||
      cols % 256u)
    return cudaErrorInvalidValue;
  const dim3 grid(cols / 256u, rows / tc::kTileRows);
  if (fmt == kQ4K)
    tc::tile_tc_kernel<kQ4K><<<grid, 256, 0, s>>>(src, cols / 256u, dst);
  else
    tc::tile_tc_kernel<kQ6K><<<grid, 256, 0, s>>>(src, cols / 256u, dst);
  return cudaGetLastError();
}

}  // namespace rta
