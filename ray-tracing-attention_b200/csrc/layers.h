// layers.h -- parameter blocks of the per-token kernels in layers.cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace rta {

constexpr uint32_t kMaxOut = 4096;  // token ids kept per generate call

// Device-resident control block of one sequence (the role of the reference's
// control[] words: token, count, running flag, stop ids, error word).
struct Control {
  unsigned long long argkey;    // packed (order key, ~id) written by the readout's atomicMax
  unsigned long long best_key;  // last consumed key (winner value)
  uint32_t pos_next;            // next absolute position to process
  uint32_t pos_cur;             // position processed by the current step
  uint32_t running;             // 1 while generating (0 after a stop id / error)
  uint32_t n_out;               // ids emitted by this generate call
  uint32_t stops[2];
  uint32_t err;
  uint32_t prompt_len;          // prefill: prompt ids of this sequence
  uint32_t ids[kMaxOut];
};

enum EmbedMode : int { kEmbedPrefill = 0, kEmbedDecode = 1 };
struct EmbedParams {
  const uint8_t* table = nullptr;  // token_embd rows (Q4_K / Q6_K)
  int fmt = 14;
  uint32_t D = 0, row_bytes = 0, vocab = 0;
  Control* ctrl = nullptr;           // [nseq] control blocks
  const uint32_t* prompt = nullptr;  // [nseq][prompt_stride] prefill ids by absolute position
  uint32_t prompt_stride = 0;
  int mode = kEmbedDecode;
  float* state = nullptr;            // [nseq][D]
  uint32_t nseq = 1;
};

struct PrepParams {
  const float* qkvg = nullptr;   // [q (heads*hd) | k (kvh*hd) | v (kvh*hd) | gate]
  const float* qnorm = nullptr;  // [heads][hd]
  const float* knorm = nullptr;  // [heads][hd] (tiled per query head)
  const float* inv_freq = nullptr;
  float eps = 1e-6f;
  uint32_t heads = 16, kvh = 4, hd = 256, group = 4, rotary = 0, qk_norm = 1;
  uint32_t q_width = 0, kv_width = 0;
  float* qout = nullptr;
  __half* kcache = nullptr;  // this layer: [nseq][kvh][capacity][hd]
  __half* vcache = nullptr;
  uint32_t capacity = 0;
  const uint32_t* pos = nullptr;      // sequence z reads pos[z * ctrl_step]
  const uint32_t* running = nullptr;  // likewise
  uint32_t nseq = 1, ctrl_step = 0;
  size_t qkvg_seq = 0;                // floats between sequences' projections
  // non-null: append the reference's history packet (kvh Q4_K keys + kvh Q6_K
  // values, packet_bytes(kvh) per position) to this ring instead of fp16 K/V
  uint8_t* packets = nullptr;         // this layer: [nseq][capacity][packet]
  // 1: sequence z writes ring z; 0: every z writes the one ring (the rows of a
  // prefill chunk are consecutive positions of one sequence)
  uint32_t ring_seq = 1;
};

// Prefill chunk (C consecutive prompt positions of one sequence as C rows):
// chunk_begin embeds prompt ids pos_next .. pos_next + C - 1 into rows and writes
// each row's (position, live) pair; chunk_end copies the last live row into the
// sequence's residual row and advances its positions.
struct ChunkParams {
  const uint8_t* table = nullptr;  // token_embd rows
  int fmt = 14;
  uint32_t D = 0, row_bytes = 0, vocab = 0, C = 0;
  Control* ctrl = nullptr;            // the sequence's control block
  const uint32_t* prompt = nullptr;   // prompt ids by absolute position
  uint32_t* rowctl = nullptr;         // [C][2]: position, live
  float* rows = nullptr;              // [C][D] residual rows of the chunk
  float* state = nullptr;             // [D] the sequence's residual row
};

struct GdnParams {
  const float* x = nullptr;          // residual stream [D] (input of the layer)
  const float* attn_norm = nullptr;  // [D]
  float eps = 1e-6f;
  const float* wa = nullptr;         // [H][D] alpha projection (F32)
  const float* wb = nullptr;         // [H][D] beta projection (F32)
  const float* a_log = nullptr;      // [H]
  const float* dt_bias = nullptr;    // [H]
  const float* proj = nullptr;       // [q (K) | k (K) | v (S) | z (S)] raw projections
  const float* conv_w = nullptr;     // [3S][4]
  float* conv_state = nullptr;       // [2][3S][3] double-buffered by position parity
  float* rec = nullptr;              // [H][128][128] (value, key)
  float* out = nullptr;              // [S] detector output (before the gated norm)
  uint32_t D = 0, H = 0, KH = 0;
  const uint32_t* pos = nullptr;      // sequence z reads pos[z * ctrl_step]
  const uint32_t* running = nullptr;  // likewise
  uint32_t* err = nullptr;            // device error words, sequence z's at err[z * err_step] (bounded staging waits)
  uint32_t err_step = 0;
  uint32_t nseq = 1, ctrl_step = 0;
  size_t proj_seq = 0;                // floats between sequences' projections
  size_t conv_seq = 0, rec_seq = 0;   // floats between sequences' conv history / recurrent state
};

// Prefill capture (the reference's debug prefill, optical_resident.cpp:481
// audit copy and the final state copy): the residual row of the position the
// step processes, copied to dst + pos * D, or (norm_w set) written after the
// final RMSNorm, op 1 index 2 of resident_math.comp:33-38.
struct CaptureParams {
  const float* state = nullptr;  // [D] (one sequence)
  float* dst = nullptr;          // [capacity][D]
  const Control* ctrl = nullptr;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  uint32_t D = 0, capacity = 0;
};

// The recurrent layer over the rows of a prefill chunk (consecutive positions of
// one sequence): a parallel pre-pass forms every row's gates, convolved and
// normalised q / k and convolved v (nothing there depends on the recurrent
// state: the convolution reads earlier rows' raw projections), then a scan
// walks the rows in order on each CTA's value rows held in registers.
struct GdnChunkParams {
  GdnParams g;                 // x / proj rows (g.proj_seq floats apart), weights, conv_state, rec, out rows
  const uint32_t* rowctl = nullptr;  // [C][2]: position, live (live rows are a prefix)
  uint32_t C = 0;
  float* gates = nullptr;      // [C][H][2] decay, beta
  float* qk = nullptr;         // [C][H][2][128] normalised q (scaled by 1/sqrt(128)), k
  float* vc = nullptr;         // [C][H][128] convolved v
};
cudaError_t launch_gdn_chunk(const GdnChunkParams& p, cudaStream_t s, bool pdl);

cudaError_t launch_embed(const EmbedParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_chunk_begin(const ChunkParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_chunk_end(const ChunkParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_capture_row(const CaptureParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_attn_prep(const PrepParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_gdn(const GdnParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_gather_rows(const uint8_t* src, const uint32_t* map, uint32_t rows, uint32_t row_bytes,
                               uint8_t* dst, cudaStream_t s);

}  // namespace rta
