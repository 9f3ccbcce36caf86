/*
 * rta.h -- C-ABI of librta_cuda.so, the B200 (sm_100a) backend for the decode
 * path of Ray Tracing Attention (Winamin/Ray-Tracing-Attention).
 *
 * Two layers, both plain C types (no torch, no C++):
 *
 *  1. Decode-path operators on caller-owned DEVICE pointers.  They allocate
 *     nothing; where an operator needs device scratch the caller passes a
 *     workspace sized by the matching *_workspace_bytes() query.  `stream` is a
 *     cudaStream_t (NULL = legacy default stream).  Calls are asynchronous.
 *
 *  2. A resident-model handle (rta_open ... rta_close) that owns all device
 *     memory of one model on one GPU and serves the operations of the
 *     reference's native worker protocol (ray_tracing/native/src/
 *     optical_resident.cpp:969): generate (op 2), prefill (op 1), vocabulary
 *     (op 4), mlp (op 6), attention (op 14), resources (op 8), grow (op 10).
 *     Host buffers in, host buffers out; a handle is single-threaded.
 *
 * Host threads may call the operators, and use different handles, at the same
 * time: each kernel's one-time set-up on a device (shared-memory limits,
 * occupancy) is synchronised, so first calls that arrive together are safe.
 *
 * Every function returns an rta_status and never aborts the process.
 * Format codes are the exporter's (ray_tracing/compiler/export.py:12):
 * 0 F32, 1 F16, 30 BF16, 12 Q4_K, 14 Q6_K.
 */
#ifndef RTA_H
#define RTA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define RTA_API __attribute__((visibility("default")))
#else
#define RTA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int rta_status;
enum {
  RTA_OK = 0,
  RTA_E_ARG = 1,          /* invalid argument, shape or format */
  RTA_E_ASSET = 2,        /* unreadable or inconsistent model payload */
  RTA_E_CUDA = 3,         /* CUDA runtime error (see rta_last_error) */
  RTA_E_DEVICE_CHECK = 4, /* a kernel set the device error word (mirrors control[3]) */
  RTA_E_TIMEOUT = 5,      /* a bounded device-side wait or host deadline expired */
  RTA_E_STATE = 6         /* call not valid in the handle's current state */
};
enum { RTA_F32 = 0, RTA_F16 = 1, RTA_BF16 = 30, RTA_Q4_K = 12, RTA_Q6_K = 14 };
/* Tiled re-layouts of Q4_K / Q6_K matrices made by rta_tile_weights: the same
 * bytes in the order the decode GEMV streams them.  Codes of this library (no
 * counterpart in the exporter's format table); accepted by the GEMV operators
 * (rta_gemv, rta_gemv_swiglu, rta_mlp_swiglu, rta_readout) in place of 12 / 14. */
enum { RTA_Q4_K_TILED = 112, RTA_Q6_K_TILED = 114 };
/* Panel re-layouts made by rta_panel_weights for the tensor-core batched
 * product (rta_gemm_tc): per 128-row tile and 256-column block one contiguous
 * panel of the same bytes, ordered for the dequantizing threads. */
enum { RTA_Q4_K_PANEL = 212, RTA_Q6_K_PANEL = 214 };

/* Text of the last error raised on this thread (never NULL). */
RTA_API const char* rta_last_error(void);
/* Library build identity, e.g. "rta_cuda sm_100a". */
RTA_API const char* rta_version(void);

/* ------------------------------------------------------------------ 1. operators */

/* Quantize nblocks x 256 fp32 values into Q4_K (144 B) / Q6_K (210 B) blocks
 * with the reference's packet quantizer
 * (ray_tracing/native/shaders/resident_history_quant.glsl:9-41). */
RTA_API rta_status rta_quantize(int format, const float* src, size_t nblocks, void* dst_blocks, void* stream);

/* Synthetic weights: nblocks x 256 values sigma * N from a counter-based
 * generator keyed by (seed, global coefficient index), quantized as above.  N
 * is an Irwin-Hall sum of eight 16-bit uniforms from two splitmix64 outputs,
 * centred and scaled to unit variance (tails end at about 4.9 sigma): integer
 * arithmetic and exactly rounded multiplies only, so a host restatement
 * reproduces every value bit for bit. */
RTA_API rta_status rta_synthetic_blocks(int format, uint64_t seed, float sigma, uint64_t first_block, size_t nblocks,
                                void* dst_blocks, void* stream);

/* Synthetic fp32 values mean + sigma * N, same generator. */
RTA_API rta_status rta_synthetic_normal(uint64_t seed, float sigma, float mean, size_t n, float* dst, void* stream);

/* Decode packed blocks to fp32, bit-exact with ggufValue
 * (ray_tracing/native/shaders/resident_quant.glsl:6-20). */
RTA_API rta_status rta_dequantize(int format, const void* blocks, size_t nblocks, float* dst, void* stream);

/* Re-lay a row-major [rows x cols] Q4_K / Q6_K matrix (rows % 16 == 0,
 * cols % 256 == 0) into the tiled order of RTA_Q4_K_TILED / RTA_Q6_K_TILED:
 * for each 16-row tile and 256-column block the 16 blocks become one
 * contiguous tile, codes in tensor-core fragment order.  dst (same byte size,
 * 16-byte aligned) must not overlap src.  The engine applies this once to
 * every resident matrix at load (the reference keeps its payloads in GGUF
 * order, optical_resident.cpp:139-153). */
RTA_API rta_status rta_tile_weights(int format, const void* src, uint32_t rows, uint32_t cols, void* dst,
                                    void* stream);

/* Re-lay a row-major [rows x cols] Q4_K / Q6_K matrix (rows % 128 == 0,
 * cols % 256 == 0) into the panel order of RTA_Q4_K_PANEL / RTA_Q6_K_PANEL
 * (same byte size; dst 16-byte aligned, not overlapping src). */
RTA_API rta_status rta_panel_weights(int format, const void* src, uint32_t rows, uint32_t cols, void* dst,
                                     void* stream);

/* Batched product on the tensor cores (tcgen05), for batches of 16 rows or
 * more: y[b][r] (+)= sum_c W[r][c] x[b][c] with W in panel order
 * (RTA_Q4_K_PANEL / RTA_Q6_K_PANEL), rows % 128 == 0, cols % 256 == 0,
 * 1 <= batch <= 256.  Both operands are fp16: x rounded once, each weight
 * rounded once after its block scale is applied (about 3e-4 relative L2 from
 * the exact product at random weights); accumulation is fp32.  `flags`
 * (formerly accumulate; 0 / 1 keep their meaning): RTA_GEMM_ACCUMULATE adds
 * into y; RTA_GEMM_SPLIT_ACTIVATIONS takes x as two fp16 operands,
 * fp16(x) + fp16(x - fp16(x)), leaving only the weight rounding.  When argmax
 * is not NULL the row of the largest y[b][.] (ties -> lowest row) and its
 * value (best, may be NULL) are returned per batch row, and y may be NULL
 * (vocabulary readout).  workspace: rta_gemm_tc_workspace_bytes(format,
 * batch, cols) bytes (enough for either mode).  Replaces op 2 of
 * ray_tracing/native/shaders/resident_math.comp:39-75 and the readout ops
 * 16/17/23 (:117-130) for batched rows. */
enum { RTA_GEMM_ACCUMULATE = 1, RTA_GEMM_SPLIT_ACTIVATIONS = 2 };
RTA_API size_t rta_gemm_tc_workspace_bytes(int format, uint32_t batch, uint32_t cols);
RTA_API rta_status rta_gemm_tc(int format, const void* w, uint32_t rows, uint32_t cols, const float* x,
                               uint32_t batch, float* y, int flags, uint32_t* argmax, float* best,
                               void* workspace, size_t workspace_bytes, void* stream);

/* SwiGLU MLP on the tensor cores: y (+)= Wd swiglu(Wg x, Wu x) with the three
 * matrices in panel order (middle % 256 == 0, hidden % 256 == 0), 1 <= batch
 * <= 256.  Gate and up run as one launch; SwiGLU is applied while the down
 * projection stages its activation (act, [batch][middle], may be NULL; when
 * given it receives the activation rows).  workspace:
 * rta_mlp_tc_workspace_bytes(format, batch, hidden, middle) bytes.  Replaces
 * executeMLP (optical_resident.cpp:484-491: op 2 kind 3 then kind 4) for
 * batched rows. */
RTA_API size_t rta_mlp_tc_workspace_bytes(int format, uint32_t batch, uint32_t hidden, uint32_t middle);
RTA_API rta_status rta_mlp_tc(int format, const void* w_gate, const void* w_up, const void* w_down, uint32_t hidden,
                              uint32_t middle, const float* x, uint32_t batch, float* act, float* y, int accumulate,
                              void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------- 1b. tensor-parallel peer exchange
 *
 * The reference has no collective (one worker, one GPU).  For the MLP and the
 * vocabulary readout split over the GPUs of one box (one process per GPU), a
 * team gives every rank an exchange buffer that the other ranks write through
 * NVLink peer memory; each exchange is one kernel launch with bounded waits.
 * Set-up: every rank calls rta_team_create on its own device, the caller
 * passes the world handles (rta_team_handle_bytes() each, rank order) to every
 * rank by any host means, and every rank calls rta_team_connect.  All ranks
 * must then make the same exchange calls in the same order.  Tear-down:
 * rta_team_disconnect on every rank, a host barrier, rta_team_destroy.  A rank
 * whose peers do not arrive within about a second records RTA_DEVERR_TIMEOUT
 * (read by rta_team_error) instead of hanging. */
typedef struct rta_team rta_team;
RTA_API size_t rta_team_handle_bytes(void);
/* capacity_bytes: the largest contribution of one rank to one exchange
 * (<= 2 MiB); handle: rta_team_handle_bytes() bytes out (unused at world 1). */
RTA_API rta_status rta_team_create(uint32_t rank, uint32_t world, size_t capacity_bytes, rta_team** team,
                                   void* handle);
RTA_API rta_status rta_team_connect(rta_team* team, const void* handles);
/* out[i] = addend[i] + sum over ranks of partial[i] (rank order, so every
 * rank gets the same bits); addend may be NULL; n % 4 == 0; 16-byte aligned
 * device buffers; out may alias partial or addend.  The sum of the row-split
 * MLP's partial down projections (the residual as addend). */
RTA_API rta_status rta_team_allreduce_f32(rta_team* team, const float* partial, const float* addend, float* out,
                                          size_t n, void* stream);
/* Best row over the ranks' local argmax (ids local to each rank's vocabulary
 * rows, which start at id_base; 0xffffffff = none): largest value, ties ->
 * lowest global id, as ops 16/17 of resident_math.comp:117-127.  best_out may
 * be NULL; batch <= 1024. */
RTA_API rta_status rta_team_argmax(rta_team* team, const uint32_t* ids, const float* best, uint32_t id_base,
                                   uint32_t batch, uint32_t* argmax, float* best_out, void* stream);
/* Synchronizes `stream`, returns and clears the team's device error word. */
RTA_API rta_status rta_team_error(rta_team* team, void* stream, uint32_t* error_word);
RTA_API rta_status rta_team_disconnect(rta_team* team);
RTA_API void rta_team_destroy(rta_team* team);

/* y[b][r] (+)= sum_c W[r][c] x[b][c]; W row-major Q4_K or Q6_K (or their tiled
 * re-layouts), or dense F32 / F16 / BF16 (the exporter's codes 0 / 1 / 30,
 * 16-byte aligned rows), rows % 16 == 0, cols % 256 == 0, 1 <= batch <= 32.
 * The same formats are accepted by rta_gemv_swiglu, rta_mlp_swiglu and
 * rta_readout, and by the model handle for every projection, the embedding
 * and the output rows.  Replaces op 2 of
 * ray_tracing/native/shaders/resident_math.comp:39-75 (kinds 0-2, 4-6, 8)
 * over ggufValue (resident_quant.glsl:6-20). */
RTA_API rta_status rta_gemv(int format, const void* w, uint32_t rows, uint32_t cols, const float* x, uint32_t batch,
                    float* y, int accumulate, void* stream);

/* Fused gate+up projection with the SwiGLU epilogue (op 2 kind 3,
 * ray_tracing/native/shaders/resident_math.comp:54,58,71):
 * act[b][r] = swiglu(Wg[r] . x[b], Wu[r] . x[b]), rows % 16 == 0, cols % 256 == 0. */
RTA_API rta_status rta_gemv_swiglu(int format, const void* w_gate, const void* w_up, uint32_t rows, uint32_t cols,
                                   const float* x, uint32_t batch, float* act, void* stream);

/* SwiGLU MLP: act = swiglu(Wg x, Wu x) [batch][middle]; y (+)= Wd act [batch][hidden].
 * swiglu(g,u) = sign(g)sign(u)|g||u|sigmoid(g).  Replaces executeMLP
 * (optical_resident.cpp:484-491: op 2 kind 3 then kind 4). */
RTA_API rta_status rta_mlp_swiglu(int format, const void* w_gate, const void* w_up, const void* w_down, uint32_t hidden,
                          uint32_t middle, const float* x, uint32_t batch, float* act, float* y, int accumulate,
                          void* stream);

/* Vocabulary readout: logits[b][w] = sum_c W[w][c] x[b][c] and the argmax per
 * row (ties -> lowest id).  1 <= batch <= 64.  logits and best may be NULL.
 * workspace: rta_readout_workspace_bytes(batch) bytes.  Replaces ops 16/17/23
 * (ray_tracing/native/shaders/resident_math.comp:117-130). */
RTA_API size_t rta_readout_workspace_bytes(uint32_t batch);
RTA_API rta_status rta_readout(int format, const void* w, uint32_t vocab, uint32_t hidden, const float* x, uint32_t batch,
                       float* logits, uint32_t* argmax, float* best, void* workspace, void* stream);

/* GQA causal decode attention for one query position over an fp16 K/V cache.
 *   q    [heads][head_dim] fp32 (already normed / rotated)
 *   k, v fp16, element (position p, kv head h, dim d) at
 *        (p * pos_stride + h * kv_stride) * head_dim + d   (in halves)
 *        i.e. the layout [L][kv_heads][head_dim] has pos_stride = kv_heads, kv_stride = 1.
 *   attends to positions [max(0, time-capacity+1), time] (slot p % capacity).
 *   gate [heads][head_dim] or NULL: out *= sigmoid(gate)
 *   out  [heads][head_dim];  phys [heads][2] = (max + 20, Z) or NULL.
 * head_dim must be 256, heads == 4 * kv_heads and 1 <= splits <= 1024 (history
 * splits per KV head, merged after).  Replaces the S_t/R_t detector
 * (ray_tracing/native/shaders/resident_ray.comp:97-117 and
 *  resident_detector_ordered_{scores,normalize,value}.comp). */
RTA_API size_t rta_attention_workspace_bytes(uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t splits);
RTA_API uint32_t rta_attention_default_splits(uint32_t history, uint32_t kv_heads);
RTA_API rta_status rta_attention_decode_f16(const float* q, const void* k, const void* v, uint32_t time, uint32_t capacity,
                                    uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t pos_stride,
                                    uint32_t kv_stride, const float* gate, float* out, float* phys, uint32_t splits,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of rta_attention_decode_f16 (no counterpart in the
 * reference; it exists for callers that may not allocate device memory while
 * decoding, e.g. inside another framework's allocator or a latency-critical
 * serving loop).  The split records live in a fixed array inside the library's
 * device image (about 1 MiB per GPU that loads the library, held until the
 * process exits) instead of a caller workspace, so heads * splits must not
 * exceed 1024 (RTA_E_ARG otherwise; k / v not 16-byte aligned are RTA_E_ARG
 * too, before anything is launched).  The call allocates and frees nothing.
 * The first call on a device looks up the array's device address (set-up); make
 * that first call before any stream capture.  The address is kept per device
 * and CUDA context: after a device reset, or with another context current on
 * the device, the next call looks it up again (again outside any capture).  All
 * calls share the array: calls
 * that overlap on the GPU (different streams, or different threads on one
 * device) race and must be serialised by the caller.  device_error: optional
 * caller-owned device word, zeroed by the call, that receives the device error
 * bits (timeouts, non-finite output). */
RTA_API rta_status rta_attention_decode_f16_noalloc(const float* q, const void* k, const void* v, uint32_t time,
                                                    uint32_t capacity, uint32_t heads, uint32_t kv_heads,
                                                    uint32_t head_dim, uint32_t pos_stride, uint32_t kv_stride,
                                                    const float* gate, float* out, float* phys, uint32_t splits,
                                                    uint32_t* device_error, void* stream);

/* Recurrent gated-delta layer for one token of `batch` sequences: ops 18
 * (gates), 19 (4-tap causal convolution + SiLU), 20 (L2 norms, convolution
 * roll) and 21 (delta-rule state update and readout) of
 * ray_tracing/native/shaders/resident_math.comp:131-148.  Device buffers:
 *   x [batch][hidden] the layer's input residual rows (RMS-normed here with
 *     attn_norm [hidden]); w_alpha, w_beta [heads][hidden] (F32 projections);
 *     a_log, dt_bias [heads];
 *   proj [batch][proj_stride] the raw in-projection rows [q (key_heads*128) |
 *     k (key_heads*128) | v (heads*128) | ...];
 *   conv_w [3*heads*128][4]; conv_state [batch][2][3*heads*128][3], double
 *     buffered by position parity: buffer (positions[z] & 1) holds the three
 *     previous taps and buffer (positions[z] & 1) ^ 1 receives the next ones;
 *   state [batch][heads][128 value][128 key] (recurrentOffset,
 *     resident_common.glsl:139), updated in place;
 *   out [batch][heads*128] the detector output before the gated RMSNorm
 *     (op 15, which the engine applies in the out-projection's prologue);
 *   positions [batch] each sequence's absolute position.
 * hidden <= 4096 and a multiple of 4; x, attn_norm, w_alpha, w_beta, conv_w
 * 16-byte aligned.  device_error: optional word, zeroed by the call. */
RTA_API rta_status rta_gated_delta_step(const float* x, const float* attn_norm, const float* w_alpha,
                                        const float* w_beta, const float* a_log, const float* dt_bias,
                                        const float* proj, uint32_t proj_stride, const float* conv_w,
                                        float* conv_state, float* state, float* out, const uint32_t* positions,
                                        uint32_t hidden, uint32_t heads, uint32_t key_heads, uint32_t batch,
                                        float eps, uint32_t* device_error, void* stream);

/* Device error word of the last operator call that had a workspace
 * (0 = clean); synchronizes `stream`. */
RTA_API rta_status rta_workspace_error(const void* workspace, size_t workspace_bytes, void* stream, uint32_t* error_word);


/* ------------------------------------------------------------ 2. resident model */

/* Model geometry: the fields of the compiler's ModelSpec
 * (ray_tracing/compiler/spec.py:9-26), normally read from model.json.
 * layer_kinds[l] = 1 for a full-attention layer, 2 for a recurrent layer. */
typedef struct rta_model_spec {
  uint32_t hidden_size, middle_size, vocabulary_size, depth;
  uint32_t attention_heads, kv_heads, attention_head_dim, rotary_dim;
  uint32_t state_heads, state_key_heads, state_head_dim;
  uint32_t attention_gate, qk_norm;
  float rope_theta, norm_epsilon;
  uint8_t layer_kinds[256];
} rta_model_spec;

typedef struct rta_model rta_model;

/* Text of the last rta_model_* error on this thread. */
RTA_API const char* rta_model_last_error(void);

/* Open a model from the exporter's payloads (ray_tracing/compiler/export.py:136-138):
 * params = the parameter words of optical_model.bin (after its 44-byte header),
 * matrices = geometry_weights.bin, basis = vocabulary.bin after its 16-byte
 * header.  Pointers may be host or device memory; the handle copies them to
 * `device` and owns all device memory from then on.  Replaces the worker
 * constructor Resident::Resident (optical_resident.cpp:118-220). */
RTA_API rta_status rta_model_open(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                                  const void* matrices, size_t matrix_bytes, const void* basis, size_t basis_bytes,
                                  uint32_t capacity, int device, rta_model** out);
/* Model flags. */
enum {
  /* Keep the attention history as the reference's packets (per position kv_heads
   * Q4_K key blocks then kv_heads Q6_K value blocks, 1416 B at 4 x 256;
   * resident_history_quant.glsl:9-41) instead of fp16 K/V. */
  RTA_MODEL_PACKET_HISTORY = 1,
  /* Prefill one prompt position per step (the decode step's kernels) instead of
   * the default chunks of 64 positions.  A single-sequence handle prefills in
   * chunks: the chunk's rows go through every matrix product as one batch (the
   * decode GEMV's exact integer products, one weight pass per 16 rows), the
   * attention rows over the sequence's one history ring (each row its own
   * causal window), and the recurrent layer as a parallel pre-pass (gates,
   * convolution, norms of every row) and a scan over the rows
   * (Resident::prefill's batched forward, optical_resident.cpp:672-676, which
   * forwards spans of its prefill batch). */
  RTA_MODEL_TOKEN_PREFILL = 2,
  /* Prefill chunks with their products on the tensor cores (tcgen05), from
   * panel-order copies of the Q4_K / Q6_K matrices made at open (about the
   * weights' size again in HBM): one weight pass per chunk; each activation
   * row enters as two fp16 operands (x = fp16(x) + fp16(x - fp16(x))), so the
   * products carry only the block-scaled weight operand's one fp16 rounding. */
  RTA_MODEL_TC_PREFILL = 4,
  /* The batched decode products on the tensor cores (16+ sequences) take each
   * activation row as two fp16 operands as above (twice the MMA columns)
   * instead of one fp16 rounding of x. */
  RTA_MODEL_SPLIT_ACTIVATIONS = 8,
  /* The decode caches of a single-sequence handle (the worker's `cache`
   * argument, optical_resident.cpp:118, :212-216):
   * - prefix boundaries (SharedHistoryCache, shared_history_cache.hpp:5-142):
   *   every prefill that computes positions saves the decode state at the
   *   prompt's end (residual row, recurrent and convolution states) and the
   *   attention history of the prompt in immutable 16-position blocks shared
   *   by every boundary whose ids agree up to a block's end;
   *   rta_model_finish_history saves the same at a generated reply's end.  A
   *   prefill whose ids extend a saved boundary restores it and computes only
   *   the remaining positions;
   * - the reply tree (ReplyTreeCache, reply_cache.hpp:6-68): every generated
   *   token is recorded under the 256-bit address of the state it was read
   *   from (a device digest of every live input of the decode step: residual
   *   row, recurrent and convolution states, the visible history rows with
   *   their positions, the position and the stop ids; OpticalPathKey,
   *   optical_path_key.hpp:7-91) and its position, with the successor state's
   *   address.  A generate call first follows the tree from the current
   *   address and replays the tokens it holds without computing them; the
   *   device state catches up (a saved boundary, then one step per token)
   *   only when a later call has to compute.  The tree holds 65536 nodes, the
   *   oldest overwritten first, and serves positions inside the ring.
   * The tokens are those of an uncached handle: a replayed token was computed
   * from a state with the same address.  Boundaries and blocks live in device
   * memory up to rta_model_cache_limit bytes (least recently used dropped
   * first). */
  RTA_MODEL_CACHE = 16
};
RTA_API rta_status rta_model_open_ex(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                                     const void* matrices, size_t matrix_bytes, const void* basis, size_t basis_bytes,
                                     uint32_t capacity, uint32_t sequences, uint32_t flags, int device,
                                     rta_model** out);
/* Same, reading the three payload files. */
RTA_API rta_status rta_model_open_files(const rta_model_spec* spec, const char* optical_model_bin,
                                        const char* geometry_bin, const char* vocabulary_bin, uint32_t capacity,
                                        int device, rta_model** out);
RTA_API rta_status rta_model_open_files_ex(const rta_model_spec* spec, const char* optical_model_bin,
                                           const char* geometry_bin, const char* vocabulary_bin, uint32_t capacity,
                                           uint32_t sequences, uint32_t flags, int device, rta_model** out);
RTA_API void rta_model_close(rta_model* model);

/* A handle that decodes `sequences` independent sequences side by side (a
 * ragged multi-sequence batch): one decode step produces one token for every
 * running sequence, each with its own history ring, recurrent state, position
 * and stop state.  Below 16 sequences the GEMVs stream the weights once per
 * up-to-16 sequences; from 16 sequences on, every matrix with a multiple of 128
 * rows is kept in panel order and its products run on the tensor cores
 * (rta_gemm_tc arithmetic: fp16 activations and block-scaled fp16 weights,
 * fp32 accumulation), so the
 * tokens then follow the single-sequence ones wherever the top-2 margin exceeds
 * that rounding.  No reference counterpart: the reference worker
 * serves one sequence per process (optical_resident.cpp:964-971).  The
 * single-sequence calls (rta_model_prefill / rta_model_generate) require
 * sequences == 1. */
RTA_API rta_status rta_model_open_batch(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                                        const void* matrices, size_t matrix_bytes, const void* basis,
                                        size_t basis_bytes, uint32_t capacity, uint32_t sequences, int device,
                                        rta_model** out);
/* A handle that decodes `sequences` sequences together with the other ranks of
 * `team` (one process per GPU, every rank opens its handle with the same
 * payloads, spec, capacity, sequence count and starts): the tensor-parallel
 * hybrid of the ragged batch.  Rank r runs the attention and recurrent layers
 * of sequences [sequence_starts[r], sequence_starts[r + 1]) (their histories
 * and recurrent states live on its GPU only), and a 1/world slice of every MLP
 * (gate / up rows and down-projection columns, the middle dimension divided in
 * units of 256, the first ranks one unit more) and of the vocabulary readout
 * (rows in units of 128) for all the sequences.  After every attention /
 * recurrent block the ranks add each other's block outputs to the residual
 * rows, after every MLP they sum their partial down projections (rank order,
 * the same bits on every rank), and after the readout they agree on each
 * sequence's best row: one peer-memory exchange kernel each, recorded in the
 * handle's step graphs, so every rank keeps identical residual rows and
 * emits identical tokens.  sequence_starts has world + 1 entries (0 first,
 * `sequences` last, every rank at least one sequence); the team must be
 * connected, hold sequences x hidden_size floats per exchange, and serve no
 * other exchange while the handle is open.  All ranks must make the same calls
 * (prefill_batch / seed_history / generate_batch) in the same order.  No
 * reference counterpart: the reference worker runs one sequence on one GPU
 * (optical_resident.cpp:964-971) with whole matrices per layer
 * (compiler/export.py:87-91). */
RTA_API rta_status rta_model_open_team(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                                       const void* matrices, size_t matrix_bytes, const void* basis,
                                       size_t basis_bytes, uint32_t capacity, uint32_t sequences,
                                       const uint32_t* sequence_starts, rta_team* team, uint32_t flags, int device,
                                       rta_model** out);
/* Prefill every sequence: ids[z * stride + i], i < lengths[z] (0 = idle
 * sequence); the sequences advance in lockstep, a shorter prompt sits out the
 * remaining steps. */
RTA_API rta_status rta_model_prefill_batch(rta_model* model, const uint32_t* ids, const uint32_t* lengths,
                                           uint32_t stride, const uint32_t stops[2], double* gpu_ms);
/* Throughput runs: fill every history slot, recurrent state and residual row
 * with seeded values and resume sequence z at position lengths[z]. */
RTA_API rta_status rta_model_seed_history(rta_model* model, const uint32_t* lengths, uint64_t seed);
/* `count` greedy tokens for every sequence with a history: ids[z * count + i],
 * n_out[z] tokens each (a sequence stops alone at a stop id). */
RTA_API rta_status rta_model_generate_batch(rta_model* model, uint32_t count, uint32_t* ids, uint32_t* n_out,
                                            double* gpu_ms);

/* Prefill a fresh sequence with n prompt ids (positions 0..n-1); stops[2] are
 * the stop ids of the following generate calls.  Worker op 1
 * (Resident::prefill, optical_resident.cpp:609-712). */
RTA_API rta_status rta_model_prefill(rta_model* model, const uint32_t* ids, uint32_t n, const uint32_t stops[2],
                                     double* gpu_ms);
/* Debug prefill, worker op 1 with debug = 1 (Resident::prefill capture,
 * optical_resident.cpp:609-712, per-layer copy :481): prefill as above, and
 * return the final-normed residual row of every position (states, [n][hidden],
 * what the decode readout reads) and, when layers is not NULL, every layer's
 * output row ([depth][n][hidden]). */
RTA_API rta_status rta_model_prefill_capture(rta_model* model, const uint32_t* ids, uint32_t n,
                                             const uint32_t stops[2], float* states, float* layers, double* gpu_ms);
/* Greedy decode of up to `count` tokens (readout -> argmax -> embedding ->
 * layers per token), stopping after a stop id.  Worker op 2
 * (Resident::generatePacket, optical_resident.cpp:760-871). */
RTA_API rta_status rta_model_generate(rta_model* model, uint32_t count, uint32_t* ids, uint32_t* n_out,
                                      double* gpu_ms);
/* Step profile (no reference counterpart; the reference's debug = 2 prefill
 * timestamps play this role for its own dispatches): one decode step of every
 * running sequence, like rta_model_generate_batch(1) (the sequences advance),
 * through a graph with an event after every launch group, so each group is
 * timed on its own.  Per group, in launch order: its kind (RTA_PROF_*), its
 * device time in ms and its algorithmic HBM bytes (packed weights once,
 * activations, the visible history, the recurrent state read and written).
 * Up to `capacity` groups are written; *n_groups receives the total. */
enum {
  RTA_PROF_START = 0, RTA_PROF_READOUT = 1, RTA_PROF_EMBED = 2, RTA_PROF_QKV = 3, RTA_PROF_PREP = 4,
  RTA_PROF_ATTENTION = 5, RTA_PROF_O_PROJ = 6, RTA_PROF_IN_PROJ = 7, RTA_PROF_GATED_DELTA = 8,
  RTA_PROF_OUT_PROJ = 9, RTA_PROF_GATE_UP = 10, RTA_PROF_DOWN = 11, RTA_PROF_EXCHANGE = 12
};
RTA_API rta_status rta_model_profile_step(rta_model* model, uint32_t* kinds, double* ms, double* bytes,
                                          size_t capacity, size_t* n_groups);
/* Full-attention diagnostic, worker op 14 (attentionCheck,
 * resident_attention_runtime.inl:646-753): layer must be a full-attention
 * layer; q, gate [rows][heads][head_dim] (rotated), k, v [count][kv_heads][head_dim]
 * compact history of ages history_start .. history_start+count-1; query row r
 * sits at time query_start + r.  Outputs: out [rows][heads][head_dim] (gated
 * when the model is), phys [rows][heads][2] = (m + 20, Z), the history packets
 * [count][packet bytes], and dense receipts [n_records][head_dim + 8 + block/32]
 * (m, Z, count, work counters, flags, coverage bits, U) in the order row, group
 * of `block` positions newest first, head.  block: 128, 256 or 512. */
RTA_API rta_status rta_model_attention(rta_model* model, uint32_t layer, const float* q, const float* k,
                                       const float* v, const float* gate, uint32_t rows, uint32_t count,
                                       uint32_t query_start, uint32_t history_start, uint32_t block, float* out,
                                       float* phys, uint8_t* packets, uint32_t* receipts, uint32_t* n_records,
                                       double* gpu_ms);
/* Test hook of a packet-history handle: the last step's last full-attention
 * layer for sequence `seq` -- q [heads][head_dim] after QK-norm and RoPE, its
 * gate row, the detector output in o-projection axis order -- and that layer's
 * visible history packets, oldest first ([*n_positions][packet bytes]; size the
 * buffer for capacity rows).  No reference counterpart. */
RTA_API rta_status rta_model_debug_attention(rta_model* model, uint32_t seq, float* q, float* gate, float* att,
                                             uint8_t* packets, uint32_t* n_positions);
/* MLP diagnostic, worker op 6 (mlpCheck, optical_resident.cpp:922-949):
 * y = W_down swiglu(W_gate x, W_up x), rows 1..32, host buffers. */
RTA_API rta_status rta_model_mlp(rta_model* model, uint32_t layer, const float* x, uint32_t rows, float* y,
                                 float* act);
/* Vocabulary diagnostic, worker op 4 (wordCheck, optical_resident.cpp:889-906):
 * argmax (ties -> lowest id) of the readout of `hidden`; logits may be NULL. */
RTA_API rta_status rta_model_vocabulary(rta_model* model, const float* hidden, float* logits, uint32_t* argmax,
                                        float* best);
/* Prefill with the checkpoint of worker ops 11 / 12 (optical_resident.cpp:616-622):
 * `boundary` (1..n) is the stable prefix the request names (n for op 1); with
 * RTA_MODEL_CACHE it is reported back as the stable prefix and decides the
 * snapshot kind.  Without the cache this is rta_model_prefill. */
RTA_API rta_status rta_model_prefill_checkpoint(rta_model* model, const uint32_t* ids, uint32_t n,
                                                const uint32_t stops[2], uint32_t boundary, double* gpu_ms);
/* Counters of the cache's last prefill / generate / finish_history, RTA_CACHE_*
 * indices (the history-cache fields of the prefill reply, resident_runtime.py:
 * 134-147; the reply-cache fields of the generation reply, :200-218), and
 * ms[3] = (prefix lookup wall ms, reply-tree gpu ms of the last generate, state
 * catch-up gpu ms of the last generate).  n words are written (at most
 * RTA_CACHE_INFO_WORDS); ms may be NULL. */
enum {
  RTA_CACHE_PREFILL_HIT = 0,        /* a saved boundary matched a prefix of the prompt */
  RTA_CACHE_REUSED_TOKENS = 1,      /* prompt positions restored instead of computed */
  RTA_CACHE_STABLE_TOKENS = 2,      /* the request's checkpoint boundary */
  RTA_CACHE_SNAPSHOT_KIND = 3,      /* 0 miss, 1 the whole prompt, 2 the checkpoint, 3 another prefix */
  RTA_CACHE_SHARED_BLOCKS = 4,      /* history blocks of the boundary that was restored */
  RTA_CACHE_SAVED_BOUNDARIES = 5,   /* boundaries saved by the call */
  RTA_CACHE_BOUNDARIES = 6,         /* boundaries held */
  RTA_CACHE_LOOKUPS = 7,            /* boundary lengths probed */
  RTA_CACHE_COMPUTED_TOKENS = 8,    /* prompt positions computed */
  RTA_CACHE_EVICTIONS = 9,          /* boundaries dropped for the byte limit so far */
  RTA_CACHE_ADDRESS_HIT = 10,       /* the boundary held the state address: no digest ran */
  RTA_CACHE_REPLAYED_TOKENS = 11,   /* generate: tokens taken from the reply tree */
  RTA_CACHE_TREE_QUERIES = 12,      /* generate: reply-tree lookups */
  RTA_CACHE_TREE_NODES = 13,        /* nodes held */
  RTA_CACHE_TREE_CAPACITY = 14,     /* 65536 */
  RTA_CACHE_TREE_LEAF = 15,         /* slot of the last replayed node (0xffffffff: none) */
  RTA_CACHE_RESTORED_TOKENS = 16,   /* generate: replayed tokens the device state caught up on */
  RTA_CACHE_CHECKPOINT_RESTORED = 17, /* generate: the catch-up started from a saved boundary */
  RTA_CACHE_FINISH_SAVED = 18,      /* finish_history: a boundary was saved */
  RTA_CACHE_FINISH_TOKENS = 19,     /* finish_history: its length */
  RTA_CACHE_BYTES = 20,             /* device bytes held by boundaries and blocks */
  RTA_CACHE_DIGESTS = 21,           /* state digests run by the call */
  RTA_CACHE_INFO_WORDS = 22
};
RTA_API rta_status rta_model_cache_info(rta_model* model, uint64_t* out, size_t n, double* ms);
/* Worker op 13 (finishHistory, optical_resident.cpp:743-759): save the prompt
 * plus the generated reply (a trailing stop id left out: it has no state) as a
 * boundary, when the device state has computed every one of them and they fit
 * the ring.  saved = 1 when a new boundary was saved, tokens = its length,
 * boundaries = boundaries held (any may be NULL). */
RTA_API rta_status rta_model_finish_history(rta_model* model, uint64_t* saved, uint64_t* tokens,
                                            uint64_t* boundaries);
/* Device bytes the boundaries and history blocks may hold (default: a quarter
 * of the device memory free at open, at most 8 GiB). */
RTA_API rta_status rta_model_cache_limit(rta_model* model, uint64_t bytes);
/* The 256-bit address of the current decode state (the digest the reply tree
 * keys on), after the state has caught up with every emitted token. */
RTA_API rta_status rta_model_state_address(rta_model* model, uint32_t address[8], uint32_t* position);
/* Current residual state (hidden_size floats) and absolute position (sequence 0). */
RTA_API rta_status rta_model_state(rta_model* model, float* state, uint32_t* position);
/* Resource counters, worker op 8: payload bytes, derived layer bytes, KV bytes,
 * recurrent state bytes, capacity, attention splits, kernels per decode step,
 * kernels per prefill step, position, sequences, matrices on the tensor cores. */
RTA_API rta_status rta_model_resources(rta_model* model, uint64_t* out, size_t n);

#ifdef __cplusplus
}
#endif
#endif /* RTA_H */
