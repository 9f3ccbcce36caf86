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
// so  sum_k w_k x_k = d * sum_k A_k x_k - dmin * sum_G m_G X_G  with the exact
// integers A_k = sc*q (Q4_K, <= 945) or sc*(q-32) (Q6_K, |A| <= 4096; fp16
// holds them exactly up to 2048 and rounds to even above) and the group sums
// X_G.  The tensor cores form sum A_k x_k per block in fp32 (A fp16 in tensor
// memory, x rounded once to fp16), the mins term is one more K=16 MMA per
// block against the group sums of the same fp16 x (fp32 sums split into two
// fp16 halves, so the mins cancel against exactly what the codes see), and
// the epilogue applies the fp32 block scales d / dmin and sums the blocks in
// fp32.  The only rounding beyond fp32 accumulation is x -> fp16.
//
// Weights use the "panel" layout of this library (formats 212 / 214, made by
// launch_tile_tc): per 128-row tile and 256-wide block column one contiguous
// panel of the same bytes, ordered so that the dequantizing thread of row m
// reads its bytes with conflict-free 16-byte shared loads:
//   Q4_K panel (18432 B): codes [pl 4][part 2][row 128][16 B] = GGUF bytes
//     16 + 32*pl + 16*part .. +15 of the row; then headers [row 128][16 B]
//     (d, dmin, 12 packed 6-bit scales and mins).
//   Q6_K panel (26880 B): per half h (2): ql [j 2][part 2][row 128][16 B] =
//     GGUF ql bytes 64h + 32j + 16part .. +15, then qh [part 2][row 128][16 B]
//     = qh bytes 128 + 32h + 16part .. +15; then scales [row 128][16 int8],
//     then d [row 128][fp16].
//
// One persistent CTA per SM (608 threads) walks (128-row tile, K slice) units:
//   warp 0      bulk-copies each tile's panels (one copy per block column),
//               from kernel start (weights do not depend on earlier kernels)
//   warp 18     bulk-copies the activation stage of each 128-wide K step, after
//               griddepcontrol.wait (written by the preceding prep kernel)
//   warps 10-17 dequantize the panel into tensor memory (A operand; thread =
//               row, tcgen05.st), two warps per 32-lane quarter (warp % 4)
//   warp 1      issues tcgen05.mma kind::f16 M=128 N=batch K=16 (A from tensor
//               memory, B from shared memory) into one of two fp32 block
//               accumulators, and commits stage releases to mbarriers
//   warps 2-9   read the block accumulators (tcgen05.ld; thread = row, each
//               warp half of the batch columns), scale and sum them per row in
//               registers, and run the store / residual / argmax epilogue at
//               the end of the tile
// Every wait is bounded (RTA_WAIT_NS): a stuck pipeline flags
// RTA_DEVERR_TIMEOUT, drains its copies and MMAs and frees tensor memory.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "rta_device.cuh"
#include "rta_internal.h"

namespace rta {
namespace tc {

constexpr uint32_t kThreads = 608;  // 19 warps
constexpr uint32_t kTileRows = 128;
constexpr uint32_t kQ4KPanel = 128u * kQ4KBytes, kQ6KPanel = 128u * kQ6KBytes;  // 18432, 26880
constexpr uint32_t kAStages = 3;  // tensor-memory A stages
// Activation ring: the same depth as the tensor-memory A ring, so one barrier
// pair per stage serves both (A and B of a half block are ready and released together).
__host__ __device__ constexpr uint32_t b_stages(uint32_t) { return kAStages; }
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
  uint32_t ksplit;  // K slices per tile: work unit = (tile, slice); > 1 only for the residual epilogue
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
  uint32_t off_b, off_bar, off_misc, b_stage;
};

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
__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, __half2 b) { return h2_bits(__hsub2(bits_h2(a), b)); }

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

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
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

// ------------------------------------------------------------- dequantizers
// Q4_K header word w (bytes 4..15 of the block: scales / mins, 6 bits each).
__device__ __forceinline__ void q4_scale_min(const uint4& h, uint32_t G, uint32_t& sc, uint32_t& mn) {
  auto byte = [&](uint32_t i) -> uint32_t {  // header byte i (0..15)
    const uint32_t w = i < 4u ? h.x : i < 8u ? h.y : i < 12u ? h.z : h.w;
    return (w >> (8u * (i & 3u))) & 0xFFu;
  };
  if (G < 4u) {
    sc = byte(4u + G) & 63u;
    mn = byte(8u + G) & 63u;
  } else {
    const uint32_t mixed = byte(12u + G - 4u);
    sc = (mixed & 15u) | ((byte(G) >> 6) << 4);
    mn = (mixed >> 4) | ((byte(4u + G) >> 6) << 4);
  }
}

// Code bytes of row m that one dequantizing thread (j) needs for one half
// block column (h): loaded for both halves as soon as the panel lands, so the
// shared-memory latency overlaps the previous half's arithmetic.
struct Q4Words {
  uint4 c0, c1;  // GGUF code bytes 16 + 32*pl .. +31, pl = 2h + j
};
struct Q6Words {
  uint4 l0, l1;  // ql bytes 64h + 32j .. +31
  uint4 g0, g1;  // qh bytes 128 + 32h .. +31
};
__device__ __forceinline__ Q4Words load_q4(const uint8_t* panel, uint32_t m, uint32_t h, uint32_t j) {
  const uint32_t pl = 2u * h + j;
  return {*reinterpret_cast<const uint4*>(panel + ((pl * 2u + 0u) * 128u + m) * 16u),
          *reinterpret_cast<const uint4*>(panel + ((pl * 2u + 1u) * 128u + m) * 16u)};
}
__device__ __forceinline__ Q6Words load_q6(const uint8_t* panel, uint32_t m, uint32_t h, uint32_t j) {
  const uint8_t* base = panel + h * 12288u;
  return {*reinterpret_cast<const uint4*>(base + ((j * 2u + 0u) * 128u + m) * 16u),
          *reinterpret_cast<const uint4*>(base + ((j * 2u + 1u) * 128u + m) * 16u),
          *reinterpret_cast<const uint4*>(base + 8192u + m * 16u),
          *reinterpret_cast<const uint4*>(base + 8192u + (128u + m) * 16u)};
}

// Row m's 64 coefficients 128h + 64j .. +63 of one Q4_K panel -> 32 tensor-
// memory columns (fp16 pairs sc*q), plus (h == 0, j == 0) the 8 mins columns.
// Q4_K operand: the codes centred on 8, sc*(q-8) (exact), times 2^6 d (one
// rounding); the mins term carries 2^6 (8 d sc - dmin m) per group, so the two
// rounded terms stay small next to the weight they sum to.
__device__ __forceinline__ void dequant_q4(const Q4Words& cw, const uint4& hdr, uint32_t h, uint32_t j, uint32_t tcol,
                                           uint32_t a2col, __half2 dd, float d64, float dmin64) {
  const uint32_t pl = 2u * h + j;
  uint32_t sc0, mn0, sc1, mn1;
  q4_scale_min(hdr, 2u * pl, sc0, mn0);
  q4_scale_min(hdr, 2u * pl + 1u, sc1, mn1);
  // low nibbles hold 1024 + q after the 0x64 exponent byte: (1024+q)*sc - 1024*sc;
  // high nibbles hold 1024 + 16q: (1024+16q)*(sc/16) - 64*sc.  Both exact.
  const __half2 s0 = __float2half2_rn(static_cast<float>(sc0)), k0 = __float2half2_rn(-1024.f * sc0);
  const __half2 s1 = __float2half2_rn(static_cast<float>(sc1) * 0.0625f), k1 = __float2half2_rn(-64.f * sc1);
  const __half2 e0 = __float2half2_rn(8.f * sc0), e1 = __float2half2_rn(8.f * sc1);  // centre: q -> q - 8
  const uint32_t words[8] = {cw.c0.x, cw.c0.y, cw.c0.z, cw.c0.w, cw.c1.x, cw.c1.y, cw.c1.z, cw.c1.w};
  uint32_t lo[16], hi[16];
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t p01 = __byte_perm(words[w], 0x64646464u, 0x5140u);
    const uint32_t p23 = __byte_perm(words[w], 0x64646464u, 0x5342u);
    lo[2 * w] = hmul2_bits(hsub2_bits(hfma2_bits(p01 & 0xFF0FFF0Fu, s0, k0), e0), dd);
    lo[2 * w + 1] = hmul2_bits(hsub2_bits(hfma2_bits(p23 & 0xFF0FFF0Fu, s0, k0), e0), dd);
    hi[2 * w] = hmul2_bits(hsub2_bits(hfma2_bits(p01 & 0xFFF0FFF0u, s1, k1), e1), dd);
    hi[2 * w + 1] = hmul2_bits(hsub2_bits(hfma2_bits(p23 & 0xFFF0FFF0u, s1, k1), e1), dd);
  }
  tmem_st16(tcol + 32u * j, lo);
  tmem_st16(tcol + 32u * j + 16u, hi);
  if (a2col != 0u) {  // mins of the 8 groups, twice (against the hi and lo halves of the group sums)
    uint32_t mv[8];
#pragma unroll
    for (uint32_t p = 0; p < 4u; ++p) {
      uint32_t sa, ma, sb, mb;
      q4_scale_min(hdr, 2u * p, sa, ma);
      q4_scale_min(hdr, 2u * p + 1u, sb, mb);
      mv[p] = mv[4 + p] = h2_bits(__floats2half2_rn(8.f * d64 * static_cast<float>(sa) - dmin64 * static_cast<float>(ma),
                                                     8.f * d64 * static_cast<float>(sb) - dmin64 * static_cast<float>(mb)));
    }
    tmem_st8(a2col, mv);
  }
}

// Row m's coefficients 128h + 32j + 0..31 and 128h + 64 + 32j + 0..31 of one
// Q6_K panel -> tensor-memory columns 16j.. and 32 + 16j.. (fp16 sc*(q-32)).
// Each fp16 pair is assembled by one bit-select of two byte permutes: the
// nibble (at bits 4-7) and the 0x64 exponent byte from the ql permute, the
// two high bits (at bits 8-9) from the permute of the pre-shifted qh word:
// 0x6400 | 16q = 1024 + 16q, then (1024 + 16q)*(sc/16) - 96*sc = sc*(q-32).
__device__ __forceinline__ void dequant_q6(const Q6Words& cw, const uint4& s4, uint32_t h, uint32_t j,
                                           uint32_t tcol, __half2 dd) {
  const uint32_t qlw[8] = {cw.l0.x, cw.l0.y, cw.l0.z, cw.l0.w, cw.l1.x, cw.l1.y, cw.l1.z, cw.l1.w};
  const uint32_t qhw[8] = {cw.g0.x, cw.g0.y, cw.g0.z, cw.g0.w, cw.g1.x, cw.g1.y, cw.g1.z, cw.g1.w};
  // int8 scales 8h + 2j + u (low run) and 8h + 4 + 2j + u (high run), u = 0, 1:
  // bytes 2j + u of word h*2 and of word h*2 + 1
  const uint32_t wl = h ? s4.z : s4.x, wh = h ? s4.w : s4.y;
  __half2 sl[2], kl[2], sh[2], kh[2];
#pragma unroll
  for (uint32_t u = 0; u < 2u; ++u) {
    const float a = static_cast<float>(static_cast<int8_t>((wl >> (8u * (2u * j + u))) & 0xFFu));
    const float b = static_cast<float>(static_cast<int8_t>((wh >> (8u * (2u * j + u))) & 0xFFu));
    sl[u] = __float2half2_rn(a * 0.0625f);
    kl[u] = __float2half2_rn(-96.f * a);
    sh[u] = __float2half2_rn(b * 0.0625f);
    kh[u] = __float2half2_rn(-96.f * b);
  }
  constexpr uint32_t kSel = 0xFCF0FCF0u;  // bits taken from the ql permute
  uint32_t lo[16], hi[16];
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t qs = qlw[w] << 4;               // low-run nibbles to bits 4-7 of each byte
    const uint32_t hl = qhw[w] >> (2u * j);        // low-run high bits to bits 0-1 of each byte
    const uint32_t hh = qhw[w] >> (4u + 2u * j);   // high-run high bits to bits 0-1 of each byte
    const uint32_t u = static_cast<uint32_t>(w) / 4u;  // first / second 16 coefficients of the run
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const uint32_t sel_l = pr == 0 ? 0x5140u : 0x5342u;  // bytes (2pr, 2pr+1) -> low byte of each half
      const uint32_t sel_h = pr == 0 ? 0x1404u : 0x3424u;  // the same bytes -> high byte of each half
      const uint32_t al = __byte_perm(qs, 0x64646464u, sel_l), ah = __byte_perm(qlw[w], 0x64646464u, sel_l);
      const uint32_t bl = __byte_perm(hl, 0u, sel_h), bh = __byte_perm(hh, 0u, sel_h);
      lo[2 * w + pr] = hmul2_bits(hfma2_bits((al & kSel) | (bl & ~kSel), sl[u], kl[u]), dd);
      hi[2 * w + pr] = hmul2_bits(hfma2_bits((ah & kSel) | (bh & ~kSel), sh[u], kh[u]), dd);
    }
  }
  tmem_st16(tcol + 16u * j, lo);
  tmem_st16(tcol + 32u + 16u * j, hi);
}

// ---------------------------------------------------------------- the kernel
template <int FMT, int N>
__global__ void __maxnreg__(96) tc_gemm_kernel(const Params p) {  // 19 warps: <= 5 per sub-partition x 96 x 32 <= 16384
  using C = Cfg<FMT>;
  constexpr bool kQ4 = C::kQ4;
  constexpr uint32_t kPanel = C::kPanel, kRawS = C::kRawStages;
  constexpr uint32_t kDStride = static_cast<uint32_t>(N);  // tensor-memory columns of one accumulator
  constexpr uint32_t kBStages = b_stages(N);
  static_assert(2u * kDStride <= kAColBase, "accumulators overlap the A stages");
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + p.off_bar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = raw_full + kRawS;
  static_assert(kBStages == kAStages, "one barrier pair per (A, B) stage");
  // stage s of a half block: full once the 8 dequantizing warps have written A
  // and the activation copy has landed (8 arrivals + the stager's expect-tx
  // arrival), empty once the MMAs that read both have completed (one commit)
  uint64_t* ab_full = raw_empty + kRawS;
  uint64_t* ab_empty = ab_full + kAStages;
  uint64_t* d_full = ab_empty + kAStages;
  uint64_t* d_empty = d_full + 2;
  uint64_t* drain = d_empty + 2;
  uint32_t* misc = reinterpret_cast<uint32_t*>(smem + p.off_misc);
  volatile uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(misc + 4);  // [N] argmax candidates

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
  // work units (tile, K slice), walked in the same order by every role
  const uint32_t nunits = p.ntiles * p.ksplit;
  const uint32_t my_tiles = blockIdx.x < nunits ? (nunits - blockIdx.x + gridDim.x - 1u) / gridDim.x : 0u;
  const uint32_t tiles_per_mat = p.rows / kTileRows;
  auto unit = [&](uint32_t i, uint32_t& t, uint32_t& kb0, uint32_t& kb1) {
    const uint32_t u = blockIdx.x + i * gridDim.x, sl = u % p.ksplit;
    t = u / p.ksplit;
    kb0 = sl * p.KB / p.ksplit;
    kb1 = (sl + 1u) * p.KB / p.ksplit;
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
    for (uint32_t i = 0; i < my_tiles && early < kRawS; ++i) {
      uint32_t t, kb0, kb1;
      unit(i, t, kb0, kb1);
      const uint32_t mat = t / tiles_per_mat, mt = t % tiles_per_mat;
      const uint8_t* wbase = (mat ? p.w[1] : p.w[0]) + static_cast<size_t>(mt) * p.KB * kPanel;
      for (uint32_t kb = kb0; kb < kb1 && early < kRawS; ++kb, ++early) {
        mbar_expect_tx(&raw_full[early], kPanel);
        bulk_g2s_stream(raw + early * kPanel, wbase + static_cast<size_t>(kb) * kPanel, kPanel, &raw_full[early],
                        policy);
      }
    }
    for (uint32_t s = 0; s < kAStages; ++s) {
      mbar_init(&ab_full[s], 9);
      mbar_init(&ab_empty[s], 1);
    }
    for (uint32_t s = 0; s < 2; ++s) {
      mbar_init(&d_full[s], 1);
      mbar_init(&d_empty[s], 8);
    }
    mbar_init(drain, 1);
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
  const uint32_t b_bytes1 = static_cast<uint32_t>(N) * 256u;

  if (warp == 0) {
    // ----------------------------------------------- weight panel producer
    // Weights never depend on earlier kernels: their copies start at once, so
    // the dequantizers fill tensor memory while the prep kernel still runs.
    if (lane == 0) {
      const uint64_t policy = evict_first_policy();
      uint32_t rit = 0;  // copies issued into the raw ring
      bool stop = false;
      for (uint32_t i = 0; i < my_tiles && !stop; ++i) {
        uint32_t t, kb0, kb1;
        unit(i, t, kb0, kb1);
        const uint32_t mat = t / tiles_per_mat, mt = t % tiles_per_mat;
        const uint8_t* wbase = (mat ? p.w[1] : p.w[0]) + static_cast<size_t>(mt) * p.KB * kPanel;
        for (uint32_t kb = kb0; kb < kb1 && !stop; ++kb) {
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
          bulk_g2s_stream(raw + rs * kPanel, wbase + static_cast<size_t>(kb) * kPanel, kPanel, &raw_full[rs], policy);
          ++rit;
        }
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
    // ------------------------------------------- activation stage producer
    if (lane == 0) {
      uint32_t bit = 0;  // copies issued into the activation ring
      bool stop = false;
      pdl_wait();  // the activation stages are written by the preceding prep kernel
      for (uint32_t i = 0; i < my_tiles && !stop; ++i) {
        uint32_t t, kb0, kb1;
        unit(i, t, kb0, kb1);
        for (uint32_t kb = kb0; kb < kb1 && !stop; ++kb)
          for (uint32_t h = 0; h < 2u; ++h) {
            const uint32_t bs = bit % kBStages;
            if (*abort_flag || !mbar_wait(&ab_empty[bs], ((bit / kBStages) & 1u) ^ 1u, p.err)) {
              stop = true;
              break;
            }
            const uint32_t bytes = h == 0 ? b_bytes0 : b_bytes1;
            const uint32_t off = kb * p.blk + (h == 0 ? 0u : b_bytes0);
            mbar_expect_tx(&ab_full[bs], bytes);
            bulk_g2s(bst + bs * p.b_stage, p.xb + off, bytes, &ab_full[bs]);
            ++bit;
          }
      }
      if (stop) {
        *abort_flag = 1u;
        for (uint32_t s = 0; s < kBStages; ++s) {
          const uint32_t n = bit / kBStages + (s < bit % kBStages ? 1u : 0u);
          if (n) (void)mbar_wait(&ab_full[s], (n - 1u) & 1u, nullptr);  // bounded: ends after its limit
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(N);
      uint32_t ait = 0, bit = 0;
      bool stop = false;
      const uint32_t b0 = smem_u32(bst);
      for (uint32_t i = 0; i < my_tiles && !stop; ++i) {
        uint32_t t, kb0, kb1;
        unit(i, t, kb0, kb1);
        // one accumulator per unit (block scales are in the operand), double-buffered by unit
        const uint32_t buf = i & 1u;
        if (*abort_flag || !mbar_wait(&d_empty[buf], ((i >> 1) & 1u) ^ 1u, p.err)) {
          stop = true;
          break;
        }
        tc_fence_after();
        const uint32_t d1 = tmem + buf * kDStride;
        for (uint32_t kb = kb0; kb < kb1 && !stop; ++kb) {
          for (uint32_t h = 0; h < 2u; ++h) {
            const uint32_t as = ait % kAStages, bs = as;  // the rings advance together (one stage per half)
            if (*abort_flag || !mbar_wait(&ab_full[as], (ait / kAStages) & 1u, p.err)) {
              stop = true;
              break;
            }
            tc_fence_after();
            const uint32_t acol = tmem + kAColBase + 64u * as;
            const uint32_t bsa = b0 + bs * p.b_stage;
            const bool first = kb == kb0 && h == 0u;
#pragma unroll
            for (uint32_t kk = 0; kk < 8u; ++kk)
              mma_ts(d1, acol + 8u * kk, smem_desc(bsa + 256u * kk, 128u, 2048u), idesc,
                     (first && kk == 0u) ? 0u : 1u);
            if (kQ4 && h == 0u)  // mins term: [c_G, c_G] x [X_G hi, X_G lo], c_G = 2^6 (8 d sc - dmin m), same accumulator
              mma_ts(d1, tmem + kA2ColBase + 8u * as, smem_desc(bsa + static_cast<uint32_t>(N) * 256u, 128u, 256u),
                     idesc, 1u);
            mma_commit(&ab_empty[as]);
            ++ait;
            ++bit;
          }
        }
        if (!stop) mma_commit(&d_full[buf]);
      }
      if (stop) *abort_flag = 1u;
      mma_commit(drain);  // every MMA issued above has completed once this arrives
      (void)mbar_wait(drain, 0u, nullptr);
    }
    __syncwarp();
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------- epilogue
    constexpr int NH = N / 2;  // batch columns of this warp
    const uint32_t q = warp & 3u, m = 32u * q + lane, c0 = (warp - 2u) >> 2;  // columns c0*NH ..
    const uint32_t lane_addr = (32u * q) << 16;
    pdl_wait();  // residual targets and running flags are written by earlier kernels
    bool stop = false;
    for (uint32_t i = 0; i < my_tiles && !stop; ++i) {
      uint32_t t, kb0, kb1;
      unit(i, t, kb0, kb1);
      const uint32_t mat = t / tiles_per_mat, mt = t % tiles_per_mat;
      // the unit's whole sum (block scales were folded into the operand): one drain per unit
      const uint32_t buf = i & 1u;
      if (!warp_wait(&d_full[buf], (i >> 1) & 1u, p.err, abort_flag)) {
        stop = true;
        break;
      }
      tc_fence_after();
      float acc[NH];
      const uint32_t dcol = tmem + lane_addr + buf * kDStride + c0 * NH;
#pragma unroll
      for (int c = 0; c < NH / 8; ++c) {
        float v[8];
        tmem_ld8(dcol + 8u * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[8 * c + e] = v[e] * (1.0f / kOperandScale);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&d_empty[buf])) : "memory");
      const uint32_t R0 = mat * p.rows + mt * kTileRows, R = R0 + m;  // output rows of the tile, this thread's
#pragma unroll
      for (int i = 0; i < NH; ++i) {
        const uint32_t n = c0 * NH + static_cast<uint32_t>(i);
        if (n >= p.batch) break;
        if (p.running && p.running[static_cast<size_t>(n) * p.run_step] == 0u) continue;  // stopped sequence
        if (p.y) {
          // a warp's 32 rows of one batch column are one 128-byte line: scalar
          // atomics of split partial sums cost one L2 line operation per warp
          // instruction, as many as 16-byte vector or 512-byte bulk reductions
          float* yp = p.y + static_cast<size_t>(n) * p.y_stride + R;
          if (p.ksplit > 1u)  // partial sum of one K slice (into the residual, or into rows the prep zeroed)
            atomicAdd(yp, acc[i]);
          else if (p.epilogue == kAccumulate)
            *yp += acc[i];
          else
            *yp = acc[i];
        }
        if (p.argmax) {
          unsigned long long key = pack_argmax(acc[i], R);
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
          }
          if (lane == 0) atomicMax(&cand[n], key);
        }
      }
    }
    if (stop) *abort_flag = 1u;
  } else if (warp >= 10 && warp < 18) {
    // ---------------------------------------------------------- dequantizers
    const uint32_t q = warp & 3u, j = (warp - 10u) >> 2, m = 32u * q + lane;
    const uint32_t lane_addr = (32u * q) << 16;
    uint32_t rit = 0, ait = 0;
    bool stop = false;
    for (uint32_t i = 0; i < my_tiles && !stop; ++i) {
      uint32_t t, kb0, kb1;
      unit(i, t, kb0, kb1);
      for (uint32_t kb = kb0; kb < kb1 && !stop; ++kb) {
        const uint32_t rs = rit % kRawS;
        if (!warp_wait(&raw_full[rs], (rit / kRawS) & 1u, p.err, abort_flag)) {
          stop = true;
          break;
        }
        const uint8_t* panel = raw + rs * kPanel;
        // everything this thread needs from the panel, then the panel is released
        uint4 hdr;  // Q4_K block header / Q6_K int8 scales of row m
        uint32_t scale_word;
        Q4Words c4[2];
        Q6Words c6[2];
        if constexpr (kQ4) {
          hdr = *reinterpret_cast<const uint4*>(panel + 16384u + 16u * m);
          scale_word = hdr.x;  // d, dmin
          c4[0] = load_q4(panel, m, 0u, j);
          c4[1] = load_q4(panel, m, 1u, j);
        } else {
          hdr = *reinterpret_cast<const uint4*>(panel + 24576u + 16u * m);
          scale_word = *reinterpret_cast<const unsigned short*>(panel + 26624u + 2u * m);  // d
          c6[0] = load_q6(panel, m, 0u, j);
          c6[1] = load_q6(panel, m, 1u, j);
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&raw_empty[rs])) : "memory");
        ++rit;
        // the row's block scale (and Q4_K min scale) times 2^6, folded into the operand
        const float d64 = kOperandScale * half_bits_to_float(scale_word & 0xFFFFu);
        const float dmin64 = kOperandScale * half_bits_to_float(scale_word >> 16);  // Q4_K only
        const __half2 dd = __float2half2_rn(d64);
        for (uint32_t h = 0; h < 2u; ++h) {
          const uint32_t as = ait % kAStages;
          if (!warp_wait(&ab_empty[as], ((ait / kAStages) & 1u) ^ 1u, p.err, abort_flag)) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint32_t tcol = tmem + lane_addr + kAColBase + 64u * as;
          if constexpr (kQ4) {
            const uint32_t a2 = (h == 0u && j == 0u) ? tmem + lane_addr + kA2ColBase + 8u * as : 0u;
            dequant_q4(c4[h], hdr, h, j, tcol, a2, dd, d64, dmin64);
          } else {
            dequant_q6(c6[h], hdr, h, j, tcol, dd);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&ab_full[as])) : "memory");
          ++ait;
        }
      }
    }
    if (stop) *abort_flag = 1u;
  }

  // argmax candidates of this CTA -> the global keys (epilogue warps only)
  if (warp >= 2 && warp < 10) {
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const uint32_t t = threadIdx.x - 64u;
    if (p.argmax && t < static_cast<uint32_t>(N) && t < p.batch && cand[t])
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
  pdl_wait();
  pdl_launch_dependents();
  const bool live = n < p.batch && (!p.running || p.running[static_cast<size_t>(n) * p.run_step] != 0u);
  if (live && p.zero_y) {  // this chunk's share of the output row
    const uint32_t per = (p.zero_cols + gridDim.y - 1u) / gridDim.y;
    const uint32_t a = blockIdx.y * per, b = min(p.zero_cols, a + per);
    float* yr = p.zero_y + static_cast<size_t>(n) * p.zero_stride;
    for (uint32_t c = a + tid; c < b; c += 256u) yr[c] = 0.f;
  }
  const float* xr = p.x + static_cast<size_t>(n < p.batch ? n : 0u) * p.x_stride;
  const float* zr = p.z ? p.z + static_cast<size_t>(n < p.batch ? n : 0u) * p.z_stride : nullptr;
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
    for (int e = 0; e < 4; ++e) hv[e] = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(dst) = make_uint4(h2_bits(hv[0]), h2_bits(hv[1]), h2_bits(hv[2]), h2_bits(hv[3]));
    if (p.q4) {  // 32-group sum of the fp16 x over 4 consecutive chunks (lanes 4i..4i+3)
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) s += __low2float(hv[e]) + __high2float(hv[e]);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if ((c & 3u) == 0u) {
        const uint32_t G = c / 4u, g8 = G % 8u;
        const __half hi = __float2half_rn(s);
        const __half lo = __float2half_rn(s - __half2float(hi));
        uint8_t* b2 = p.xb + static_cast<size_t>(G / 8u) * p.blk + N * 256u + (n / 8u) * 256u + (n % 8u) * 16u;
        reinterpret_cast<__half*>(b2)[g8] = hi;
        reinterpret_cast<__half*>(b2 + 128u)[g8] = lo;
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
      if (o < 16384u) {
        const uint32_t pl = o / 4096u, part = (o / 2048u) & 1u;
        r = (o / 16u) & 127u;
        b = 16u + 32u * pl + 16u * part + o % 16u;
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
  p.b_stage = (static_cast<uint32_t>(N) * 256u + (C::kQ4 ? static_cast<uint32_t>(N) * 32u : 0u) + 1023u) / 1024u * 1024u;
  p.off_b = C::kRawStages * C::kPanel;
  p.off_b = (p.off_b + 1023u) / 1024u * 1024u;
  p.off_bar = p.off_b + tc::b_stages(N) * p.b_stage;
  p.off_misc = p.off_bar + 512u;
  uint32_t smem = p.off_misc + 16u + 8u * static_cast<uint32_t>(N);
  smem = smem < tc::kMinSmem ? tc::kMinSmem : smem;
  auto kernel = tc::tc_gemm_kernel<FMT, N>;
  static int attr_done[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[dev] = 1;
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
    default: return cudaErrorInvalidValue;
  }
}

uint32_t tile_n(uint32_t rows) { return rows <= 16u ? 16u : rows <= 32u ? 32u : 64u; }
}  // namespace

size_t tc_workspace_bytes(int fmt, uint32_t batch, uint32_t cols) {
  const bool q4 = fmt == kQ4KPanel || fmt == kQ4K;
  const uint32_t N = tile_n(batch < kTcMaxN ? batch : kTcMaxN);
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
  if (a.xb_bytes < tc_workspace_bytes(a.fmt, a.batch, a.cols)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(a.w0) | reinterpret_cast<uintptr_t>(a.w1) | reinterpret_cast<uintptr_t>(a.xb) |
       reinterpret_cast<uintptr_t>(a.x) | reinterpret_cast<uintptr_t>(a.z)) & 15u)
    return cudaErrorInvalidValue;
  if (a.x_stride % 4u || (a.z && (a.z_stride ? a.z_stride : a.x_stride) % 4u)) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint32_t nmat = a.w1 ? 2u : 1u, ntiles = nmat * (a.rows / tc::kTileRows), KB = a.cols / 256u;
  // K splits: each CTA walks its share of (tile, K slice) units; the slice
  // count minimises the block columns of the busiest CTA plus one block of
  // fixed cost per unit.  Partial sums land atomically (residual products add
  // into y, stores into rows the prep kernel zeroes); the argmax needs whole sums.
  uint32_t ksplit = 1;
  if (!a.argmax && a.y) {
    uint64_t best = ~0ull;
    for (uint32_t ks = 1; ks <= 8u && ks <= KB; ++ks) {
      const uint64_t units = static_cast<uint64_t>(ntiles) * ks;
      const uint64_t per_cta = (units + sms - 1) / sms;
      const uint64_t cost = per_cta * ((KB + ks - 1) / ks + 1);
      if (cost < best) best = cost, ksplit = ks;
    }
  }
  const uint32_t units = ntiles * ksplit;
  const uint32_t grid = units < static_cast<uint32_t>(sms) ? units : static_cast<uint32_t>(sms);
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
    pr.N = tile_n(nb);
    const uint32_t rstep = a.running_step ? a.running_step : 1u;
    pr.running = a.running ? a.running + static_cast<size_t>(b0) * rstep : nullptr;
    pr.run_step = rstep;
    pr.xb = a.xb;
    pr.blk = tc::blk_bytes(q4, pr.N);
    pr.q4 = q4;
    if (ksplit > 1u && a.epilogue == kStore) {
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
    p.ksplit = ksplit;

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
