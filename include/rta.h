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

/* Text of the last error raised on this thread (never NULL). */
RTA_API const char* rta_last_error(void);
/* Library build identity, e.g. "rta_cuda sm_100a". */
RTA_API const char* rta_version(void);

/* ------------------------------------------------------------------ 1. operators */

/* Quantize nblocks x 256 fp32 values into Q4_K (144 B) / Q6_K (210 B) blocks
 * with the reference's packet quantizer
 * (ray_tracing/native/shaders/resident_history_quant.glsl:9-41). */
RTA_API rta_status rta_quantize(int format, const float* src, size_t nblocks, void* dst_blocks, void* stream);

/* Synthetic weights: nblocks x 256 values drawn N(0, sigma) from a counter-based
 * generator keyed by (seed, global coefficient index), quantized as above. */
RTA_API rta_status rta_synthetic_blocks(int format, uint64_t seed, float sigma, uint64_t first_block, size_t nblocks,
                                void* dst_blocks, void* stream);

/* Synthetic fp32 values mean + sigma * N(0,1), same generator. */
RTA_API rta_status rta_synthetic_normal(uint64_t seed, float sigma, float mean, size_t n, float* dst, void* stream);

/* Decode packed blocks to fp32, bit-exact with ggufValue
 * (ray_tracing/native/shaders/resident_quant.glsl:6-20). */
RTA_API rta_status rta_dequantize(int format, const void* blocks, size_t nblocks, float* dst, void* stream);

/* y[b][r] (+)= sum_c W[r][c] x[b][c]; W Q4_K or Q6_K row-major, rows % 16 == 0,
 * cols % 256 == 0, 1 <= batch <= 32.  Replaces op 2 of
 * ray_tracing/native/shaders/resident_math.comp:39-75 (kinds 0-2, 4-6, 8). */
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
 * row (ties -> lowest id).  1 <= batch <= 8.  logits and best may be NULL.
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
 * head_dim must be 256 and heads == 4 * kv_heads.  Replaces the S_t/R_t detector
 * (ray_tracing/native/shaders/resident_ray.comp:97-117 and
 *  resident_detector_ordered_{scores,normalize,value}.comp). */
RTA_API size_t rta_attention_workspace_bytes(uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t splits);
RTA_API uint32_t rta_attention_default_splits(uint32_t history, uint32_t kv_heads);
RTA_API rta_status rta_attention_decode_f16(const float* q, const void* k, const void* v, uint32_t time, uint32_t capacity,
                                    uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t pos_stride,
                                    uint32_t kv_stride, const float* gate, float* out, float* phys, uint32_t splits,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Device error word of the last operator call that had a workspace
 * (0 = clean); synchronizes `stream`. */
RTA_API rta_status rta_workspace_error(const void* workspace, size_t workspace_bytes, void* stream, uint32_t* error_word);

#ifdef __cplusplus
}
#endif
#endif /* RTA_H */
