// rta_internal.h -- internal C++ interface between the CUDA kernels, the
// decode engine and the C-ABI layer (capi.cu).  Not installed; the public
// boundary is include/rta.h.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <string>

#include "rta_device.cuh"

struct rta_team;  // team.cu (include/rta.h: typedef struct rta_team rta_team)

namespace rta {

constexpr int kF32 = 0, kF16 = 1, kBF16 = 30, kQ4K = 12, kQ6K = 14;  // export.py FORMATS codes
// Tiled re-layouts of Q4_K / Q6_K matrices (same bytes, GEMV-friendly order;
// see launch_tile_weights).  Codes of this library, not of the exporter.
constexpr int kTiledOffset = 100, kQ4KTiled = kQ4K + kTiledOffset, kQ6KTiled = kQ6K + kTiledOffset;
// Panel re-layouts for the tensor-core batched path (qgemm.cu): per 128-row
// tile and 256-wide block column one contiguous panel of the same bytes.
constexpr int kPanelOffset = 200, kQ4KPanel = kQ4K + kPanelOffset, kQ6KPanel = kQ6K + kPanelOffset;
constexpr uint32_t kQ4KBytes = 144, kQ6KBytes = 210;
constexpr uint32_t kMaxBatch = 256;  // GEMV batch rows per call (run as launches of up to 8 rows)

inline uint32_t block_bytes(int fmt) {
  return fmt == kQ4K || fmt == kQ4KTiled || fmt == kQ4KPanel ? kQ4KBytes : kQ6KBytes;
}

// Record the thread-local text returned by rta_last_error() (capi.cu).
void set_last_error(const std::string& msg);

// ---------------------------------------------------------------- quant.cu
cudaError_t launch_quantize(int fmt, const float* src, size_t nblocks, uint8_t* dst, cudaStream_t s);
cudaError_t launch_random_quantize(int fmt, uint64_t seed, float sigma, uint64_t first_block, size_t nblocks,
                                   uint8_t* dst, cudaStream_t s);
cudaError_t launch_random_normal(uint64_t seed, float sigma, float mean, size_t n, float* dst, cudaStream_t s);
cudaError_t launch_random_normal_half(uint64_t seed, float sigma, size_t n, __half* dst, cudaStream_t s);
cudaError_t launch_dequantize(int fmt, const uint8_t* src, size_t nblocks, float* dst, cudaStream_t s);
// History packets (kvh Q4_K keys + kvh Q6_K values per position) from fp32
// K / V rows [rows][kvh][256], and seeded random packets for throughput runs.
cudaError_t launch_pack_history(const float* k, const float* v, uint32_t rows, uint32_t kvh, uint8_t* dst,
                                cudaStream_t s);
cudaError_t launch_random_packets(uint64_t seed, size_t rows, uint32_t kvh, uint8_t* dst, cudaStream_t s);

// ----------------------------------------------------------------- gemv.cu
// Activation prologue applied (per CTA) before the int16 activation split.
enum Prologue : int {
  kPlain = 0,      // x as given
  kRmsNorm = 1,    // x * inversesqrt(mean(x^2) + eps) * norm_w
  kHeadGate = 2,   // per 128-wide head: x * inversesqrt(mean_head(x^2)+eps) * norm_w * z * sigmoid(z)
  kSigmoidGate = 3, // x * sigmoid(z)
  kSwiGLUIn = 4     // swiglu(x, z): the gate / up outputs of the batched path (qgemm.cu only)
};
enum Epilogue : int {
  kStore = 0,      // y = W x
  kAccumulate = 1, // y += W x  (residual stream)
  kSwiGLU = 2      // y = swiglu(W0 x, W1 x)
};
struct GemvArgs {
  int fmt = kQ4K;             // kQ4K or kQ6K
  const uint8_t* w0 = nullptr;
  const uint8_t* w1 = nullptr;  // second matrix (SwiGLU up); same shape as w0
  uint32_t rows = 0, cols = 0;  // output rows (multiple of 16), input cols (multiple of 256)
  const float* x = nullptr;
  uint32_t x_stride = 0, batch = 1;
  int prologue = kPlain;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  const float* z = nullptr;     // gate input for kHeadGate / kSigmoidGate
  uint32_t z_stride = 0;        // floats between batch rows of z (0: x_stride)
  int epilogue = kStore;
  float* y = nullptr;
  uint32_t y_stride = 0;
  // optional argmax over the rows of batch row b (vocabulary readout):
  unsigned long long* argmax = nullptr;  // [batch] packed (order key, ~id); null = none
  uint32_t argmax_step = 1;              // u64 elements between batch rows' argmax keys
  uint32_t* err = nullptr;               // device error word (may be null)
  const uint32_t* running = nullptr;     // optional per-row device flags: 0 -> that row is skipped
  uint32_t running_step = 1;             // u32 elements between batch rows' flags
  bool pdl = false;                      // launch with programmatic stream serialization
};
cudaError_t launch_gemv(const GemvArgs& a, cudaStream_t s);
// Re-lay a [rows x cols] Q4_K / Q6_K matrix (rows % 16 == 0) out of GGUF row
// order into the tiled order the kTiled formats name (dst != src, same size).
cudaError_t launch_tile_weights(int fmt, const uint8_t* src, uint32_t rows, uint32_t cols, uint8_t* dst,
                                cudaStream_t s);
// ---------------------------------------------------------------- qgemm.cu
// Batched product on the tensor cores with panel-layout weights (kQ4KPanel /
// kQ6KPanel, rows % 128 == 0): a prep launch (prologue, x -> fp16 stages) and
// the persistent tcgen05 kernel per kTcMaxN batch rows.  w1 (optional) is a
// second matrix whose rows follow w0's in y (the gate / up pair).
constexpr uint32_t kTcMaxN = 64;
struct TcGemmArgs {
  int fmt = kQ4KPanel;
  const uint8_t* w0 = nullptr;
  const uint8_t* w1 = nullptr;
  uint32_t rows = 0, cols = 0;  // rows per matrix (multiple of 128), cols (multiple of 256)
  const float* x = nullptr;
  uint32_t x_stride = 0, batch = 1;
  int prologue = kPlain;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  const float* z = nullptr;
  uint32_t z_stride = 0;
  int epilogue = kStore;  // kStore or kAccumulate
  float* y = nullptr;
  uint32_t y_stride = 0;
  unsigned long long* argmax = nullptr;
  uint32_t argmax_step = 1;
  uint32_t* err = nullptr;
  const uint32_t* running = nullptr;
  uint32_t running_step = 1;
  uint8_t* xb = nullptr;  // workspace of tc_workspace_bytes(fmt, batch, cols, split) bytes
  size_t xb_bytes = 0;
  bool pdl = false;
  // Activations as two fp16 operands (x = fp16(x) + fp16(x - fp16(x))): the
  // products then carry only the weight operand's rounding, at twice the MMA
  // columns.
  bool split = false;
};
size_t tc_workspace_bytes(int fmt, uint32_t batch, uint32_t cols, bool split = false);
cudaError_t launch_tc_gemm(const TcGemmArgs& a, cudaStream_t s);
// act[r][c] = swiglu(gu[r][c], gu[r][F + c]) for r < rows, c < F.
cudaError_t launch_swiglu_rows(const float* gu, uint32_t rows, uint32_t F, uint32_t gu_stride, float* act,
                               uint32_t act_stride, cudaStream_t s);
// GGUF rows of a Q4_K / Q6_K matrix (rows % 128 == 0) -> panel layout.
cudaError_t launch_tile_tc(int fmt, const uint8_t* src, uint32_t rows, uint32_t cols, uint8_t* dst, cudaStream_t s);
// Dense F32 GEMV for the tiny recurrent alpha/beta projections.
cudaError_t launch_gemv_f32(const float* W, uint32_t rows, uint32_t cols, const float* x, uint32_t x_stride,
                            uint32_t batch, float* y, uint32_t y_stride, cudaStream_t s);

// ----------------------------------------------------------- gemv_dense.cu
// F32 / F16 / BF16 matrices (export.py format codes 0 / 1 / 30), row-major:
// the same GemvArgs contract as launch_gemv (which forwards them here).
bool dense_format(int fmt);
uint32_t dense_bytes(int fmt);  // bytes per coefficient
cudaError_t launch_gemv_dense(const GemvArgs& a, cudaStream_t s);

// ----------------------------------------------------------------- team.cu
// The decode engine's tensor-parallel mode drives the team exchanges from its
// own graphs (every rank records the same exchanges in the same order).
uint32_t team_rank(const rta_team* t);
uint32_t team_world(const rta_team* t);
bool team_ready(const rta_team* t);
size_t team_capacity_words(const rta_team* t);
uint32_t* team_error_word(rta_team* t);
// Every exchange a handle records uses team_blocks(largest exchange in words)
// blocks, which keeps the slot parity of each call the same in every block.
uint32_t team_blocks(size_t words);
// out = addend + sum over ranks of partial (rank order; same bits everywhere).
// With `running` (u32 flags `run_step` apart, one per row of `width` floats),
// rows of sequences that sat the step out keep out = addend.
cudaError_t team_allreduce(rta_team* t, const float* partial, const float* addend, float* out, size_t n,
                           uint32_t blocks, cudaStream_t s, const uint32_t* running = nullptr,
                           uint32_t run_step = 0, uint32_t width = 0);
// the same sum as a reduce-scatter + all-gather in one launch (two flag rounds,
// 2 (world - 1) / world of the contribution sent instead of world - 1 times it)
cudaError_t team_allreduce2(rta_team* t, const float* partial, const float* addend, float* out, size_t n,
                            uint32_t blocks, cudaStream_t s, const uint32_t* running = nullptr,
                            uint32_t run_step = 0, uint32_t width = 0);
// state rows of every rank r, [row_start[r], row_start[r + 1]) x width, += that
// rank's delta rows (row_start has world + 1 entries); rows of sequences that
// sat the step out (running flag 0) are left as they are
cudaError_t team_gather_add(rta_team* t, const float* delta, float* state, uint32_t width,
                            const uint32_t* row_start, uint32_t blocks, cudaStream_t s,
                            const uint32_t* running = nullptr, uint32_t run_step = 0);
// packed argmax keys (local ids from id_base) -> the largest over the ranks, in place
cudaError_t team_allmax_keys(rta_team* t, unsigned long long* keys, uint32_t n, uint32_t stride, uint32_t id_base,
                             uint32_t blocks, cudaStream_t s);

}  // namespace rta
