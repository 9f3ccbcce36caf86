// capi.cu -- extern "C" boundary of librta_cuda.so (declared in include/rta.h).
//
// Operators validate their arguments, launch the sm_100a kernels and translate
// CUDA failures into rta_status codes with a thread-local message; nothing
// here aborts the process.  There is no host fallback: every operator runs
// its CUDA kernel or returns an error.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/rta.h"
#include "attention.h"
#include "layers.h"
#include "rta_internal.h"

namespace {
thread_local std::string g_last_error = "no error";

rta_status fail(rta_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}
rta_status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RTA_OK;
  return fail(RTA_E_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}
cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
bool quant_format(int f) { return f == RTA_Q4_K || f == RTA_Q6_K; }
bool gemv_format(int f) {
  return quant_format(f) || f == RTA_Q4_K_TILED || f == RTA_Q6_K_TILED || f == RTA_F32 || f == RTA_F16 ||
         f == RTA_BF16;
}

constexpr uint32_t kApiMaxBatch = 32;  // batch rows accepted by the GEMV operators (rta.h)
constexpr size_t kErrBytes = 256;  // device error word + padding at the head of every workspace

__global__ void readout_finish_kernel(const unsigned long long* keys, uint32_t batch, uint32_t vocab,
                                      uint32_t* argmax, float* best, uint32_t* err) {
  const uint32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const unsigned long long k = keys[b];
  const uint32_t id = ~static_cast<uint32_t>(k & 0xffffffffull);
  if (k == 0ull || id >= vocab) {
    if (err) atomicOr(err, RTA_DEVERR_TOKEN);
    argmax[b] = 0xffffffffu;
    if (best) best[b] = -INFINITY;
    return;
  }
  argmax[b] = id;
  if (best) best[b] = rta::float_from_order_key(static_cast<uint32_t>(k >> 32));
}
}  // namespace

namespace rta {
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace rta

extern "C" {

const char* rta_last_error(void) { return g_last_error.c_str(); }
const char* rta_version(void) { return "rta_cuda sm_100a"; }

rta_status rta_quantize(int format, const float* src, size_t nblocks, void* dst, void* stream) {
  if (!quant_format(format) || (nblocks && (!src || !dst))) return fail(RTA_E_ARG, "rta_quantize: bad arguments");
  return cuda_status(rta::launch_quantize(format, src, nblocks, static_cast<uint8_t*>(dst), as_stream(stream)),
                     "rta_quantize");
}

rta_status rta_synthetic_blocks(int format, uint64_t seed, float sigma, uint64_t first_block, size_t nblocks,
                                void* dst, void* stream) {
  if (!quant_format(format) || (nblocks && !dst)) return fail(RTA_E_ARG, "rta_synthetic_blocks: bad arguments");
  return cuda_status(rta::launch_random_quantize(format, seed, sigma, first_block, nblocks,
                                                 static_cast<uint8_t*>(dst), as_stream(stream)),
                     "rta_synthetic_blocks");
}

rta_status rta_synthetic_normal(uint64_t seed, float sigma, float mean, size_t n, float* dst, void* stream) {
  if (n && !dst) return fail(RTA_E_ARG, "rta_synthetic_normal: null destination");
  return cuda_status(rta::launch_random_normal(seed, sigma, mean, n, dst, as_stream(stream)), "rta_synthetic_normal");
}

rta_status rta_dequantize(int format, const void* blocks, size_t nblocks, float* dst, void* stream) {
  if (!quant_format(format) || (nblocks && (!blocks || !dst))) return fail(RTA_E_ARG, "rta_dequantize: bad arguments");
  return cuda_status(rta::launch_dequantize(format, static_cast<const uint8_t*>(blocks), nblocks, dst,
                                            as_stream(stream)),
                     "rta_dequantize");
}

rta_status rta_tile_weights(int format, const void* src, uint32_t rows, uint32_t cols, void* dst, void* stream) {
  if (!quant_format(format) || !src || !dst || rows == 0 || rows % 16 || cols == 0 || cols % 256)
    return fail(RTA_E_ARG, "rta_tile_weights: format must be Q4_K/Q6_K, rows % 16 == 0, cols % 256 == 0");
  const size_t bytes = static_cast<size_t>(rows) * (cols / 256) * rta::block_bytes(format);
  const uintptr_t a = reinterpret_cast<uintptr_t>(src), b = reinterpret_cast<uintptr_t>(dst);
  if (a < b + bytes && b < a + bytes) return fail(RTA_E_ARG, "rta_tile_weights: dst overlaps src");
  return cuda_status(rta::launch_tile_weights(format, static_cast<const uint8_t*>(src), rows, cols,
                                              static_cast<uint8_t*>(dst), as_stream(stream)),
                     "rta_tile_weights");
}

rta_status rta_panel_weights(int format, const void* src, uint32_t rows, uint32_t cols, void* dst, void* stream) {
  if (!quant_format(format) || !src || !dst || rows == 0 || rows % 128 || cols == 0 || cols % 256)
    return fail(RTA_E_ARG, "rta_panel_weights: format must be Q4_K/Q6_K, rows % 128 == 0, cols % 256 == 0");
  const size_t bytes = static_cast<size_t>(rows) * (cols / 256) * rta::block_bytes(format);
  const uintptr_t a = reinterpret_cast<uintptr_t>(src), b = reinterpret_cast<uintptr_t>(dst);
  if (a < b + bytes && b < a + bytes) return fail(RTA_E_ARG, "rta_panel_weights: dst overlaps src");
  return cuda_status(rta::launch_tile_tc(format, static_cast<const uint8_t*>(src), rows, cols,
                                         static_cast<uint8_t*>(dst), as_stream(stream)),
                     "rta_panel_weights");
}

size_t rta_gemm_tc_workspace_bytes(int format, uint32_t batch, uint32_t cols) {
  const size_t keys = (8ull * (batch ? batch : 1) + 255u) / 256u * 256u;
  return kErrBytes + keys + rta::tc_workspace_bytes(format, batch ? batch : 1, cols, true);  // either mode
}

rta_status rta_gemm_tc(int format, const void* w, uint32_t rows, uint32_t cols, const float* x, uint32_t batch,
                       float* y, int accumulate, uint32_t* argmax, float* best, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if ((format != RTA_Q4_K_PANEL && format != RTA_Q6_K_PANEL) || !w || !x || (!y && !argmax) || !workspace ||
      rows == 0 || rows % 128 || cols == 0 || cols % 256 || batch == 0 || batch > rta::kMaxBatch ||
      (accumulate & ~(RTA_GEMM_ACCUMULATE | RTA_GEMM_SPLIT_ACTIVATIONS)))
    return fail(RTA_E_ARG, "rta_gemm_tc: panel format, rows % 128 == 0, cols % 256 == 0, 1 <= batch <= 256");
  if (workspace_bytes < rta_gemm_tc_workspace_bytes(format, batch, cols))
    return fail(RTA_E_ARG, "rta_gemm_tc: workspace too small");
  cudaStream_t s = as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t keys_bytes = (8ull * batch + 255u) / 256u * 256u;
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  auto* keys = reinterpret_cast<unsigned long long*>(ws + kErrBytes);
  rta_status st = cuda_status(cudaMemsetAsync(ws, 0, kErrBytes + keys_bytes, s), "rta_gemm_tc(memset)");
  if (st != RTA_OK) return st;
  rta::TcGemmArgs a;
  a.fmt = format;
  a.w0 = static_cast<const uint8_t*>(w);
  a.rows = rows;
  a.cols = cols;
  a.x = x;
  a.x_stride = cols;
  a.batch = batch;
  a.epilogue = rta::kStore;
  a.y = y;
  a.y_stride = rows;
  a.split = (accumulate & RTA_GEMM_SPLIT_ACTIVATIONS) != 0;
  if (accumulate & RTA_GEMM_ACCUMULATE) a.epilogue = rta::kAccumulate;
  a.argmax = argmax ? keys : nullptr;
  a.err = err;
  a.xb = ws + kErrBytes + keys_bytes;
  a.xb_bytes = workspace_bytes - kErrBytes - keys_bytes;
  st = cuda_status(rta::launch_tc_gemm(a, s), "rta_gemm_tc");
  if (st != RTA_OK || !argmax) return st;
  readout_finish_kernel<<<(batch + 255u) / 256u, 256, 0, s>>>(keys, batch, rows, argmax, best, err);
  return cuda_status(cudaGetLastError(), "rta_gemm_tc(finish)");
}

size_t rta_mlp_tc_workspace_bytes(int format, uint32_t batch, uint32_t hidden, uint32_t middle) {
  const uint32_t b = batch ? batch : 1u;
  const size_t gu = (8ull * b * middle + 255u) / 256u * 256u;
  const size_t xb = std::max(rta::tc_workspace_bytes(format, b, hidden), rta::tc_workspace_bytes(format, b, middle));
  return kErrBytes + gu + xb;
}

rta_status rta_mlp_tc(int format, const void* wg, const void* wu, const void* wd, uint32_t hidden, uint32_t middle,
                      const float* x, uint32_t batch, float* act, float* y, int accumulate, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if ((format != RTA_Q4_K_PANEL && format != RTA_Q6_K_PANEL) || !wg || !wu || !wd || !x || !y || !workspace ||
      hidden == 0 || hidden % 256 || middle == 0 || middle % 256 || batch == 0 || batch > rta::kMaxBatch)
    return fail(RTA_E_ARG, "rta_mlp_tc: panel format, hidden and middle multiples of 256, 1 <= batch <= 256");
  if (workspace_bytes < rta_mlp_tc_workspace_bytes(format, batch, hidden, middle))
    return fail(RTA_E_ARG, "rta_mlp_tc: workspace too small");
  cudaStream_t s = as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  float* gu = reinterpret_cast<float*>(ws + kErrBytes);
  const size_t gu_bytes = (8ull * batch * middle + 255u) / 256u * 256u;
  rta_status st = cuda_status(cudaMemsetAsync(ws, 0, kErrBytes, s), "rta_mlp_tc(memset)");
  if (st != RTA_OK) return st;
  rta::TcGemmArgs g;  // gate rows then up rows of each batch row: gu[b][0:middle], gu[b][middle:2 middle]
  g.fmt = format;
  g.w0 = static_cast<const uint8_t*>(wg);
  g.w1 = static_cast<const uint8_t*>(wu);
  g.rows = middle;
  g.cols = hidden;
  g.x = x;
  g.x_stride = hidden;
  g.batch = batch;
  g.y = gu;
  g.y_stride = 2u * middle;
  g.err = err;
  g.xb = ws + kErrBytes + gu_bytes;
  g.xb_bytes = workspace_bytes - kErrBytes - gu_bytes;
  st = cuda_status(rta::launch_tc_gemm(g, s), "rta_mlp_tc(gate/up)");
  if (st != RTA_OK) return st;
  rta::TcGemmArgs d = g;
  d.w0 = static_cast<const uint8_t*>(wd);
  d.w1 = nullptr;
  d.rows = hidden;
  d.cols = middle;
  d.epilogue = accumulate ? rta::kAccumulate : rta::kStore;
  d.y = y;
  d.y_stride = hidden;
  d.pdl = true;
  if (act) {
    st = cuda_status(rta::launch_swiglu_rows(gu, batch, middle, 2u * middle, act, middle, s), "rta_mlp_tc(swiglu)");
    if (st != RTA_OK) return st;
    d.x = act;
    d.x_stride = middle;
  } else {
    d.prologue = rta::kSwiGLUIn;
    d.x = gu;
    d.z = gu + middle;
    d.x_stride = 2u * middle;
    d.z_stride = 2u * middle;
  }
  return cuda_status(rta::launch_tc_gemm(d, s), "rta_mlp_tc(down)");
}

rta_status rta_gemv(int format, const void* w, uint32_t rows, uint32_t cols, const float* x, uint32_t batch,
                    float* y, int accumulate, void* stream) {
  if (!gemv_format(format) || !w || !x || !y || rows == 0 || rows % 16 || cols == 0 || cols % 256 || batch == 0 ||
      batch > kApiMaxBatch)
    return fail(RTA_E_ARG, "rta_gemv: format Q4_K/Q6_K (tiled too), F32, F16 or BF16, rows % 16 == 0, "
                           "cols % 256 == 0, 1 <= batch <= 32");
  rta::GemvArgs a;
  a.fmt = format;
  a.w0 = static_cast<const uint8_t*>(w);
  a.rows = rows;
  a.cols = cols;
  a.x = x;
  a.x_stride = cols;
  a.batch = batch;
  a.epilogue = accumulate ? rta::kAccumulate : rta::kStore;
  a.y = y;
  a.y_stride = rows;
  return cuda_status(rta::launch_gemv(a, as_stream(stream)), "rta_gemv");
}

rta_status rta_gemv_swiglu(int format, const void* wg, const void* wu, uint32_t rows, uint32_t cols, const float* x,
                           uint32_t batch, float* act, void* stream) {
  if (!gemv_format(format) || !wg || !wu || !x || !act || rows == 0 || rows % 16 || cols == 0 || cols % 256 ||
      batch == 0 || batch > kApiMaxBatch)
    return fail(RTA_E_ARG, "rta_gemv_swiglu: rows % 16 == 0, cols % 256 == 0, 1 <= batch <= 32");
  rta::GemvArgs g;
  g.fmt = format;
  g.w0 = static_cast<const uint8_t*>(wg);
  g.w1 = static_cast<const uint8_t*>(wu);
  g.rows = rows;
  g.cols = cols;
  g.x = x;
  g.x_stride = cols;
  g.batch = batch;
  g.epilogue = rta::kSwiGLU;
  g.y = act;
  g.y_stride = rows;
  return cuda_status(rta::launch_gemv(g, as_stream(stream)), "rta_gemv_swiglu");
}

rta_status rta_mlp_swiglu(int format, const void* wg, const void* wu, const void* wd, uint32_t hidden,
                          uint32_t middle, const float* x, uint32_t batch, float* act, float* y, int accumulate,
                          void* stream) {
  if (!gemv_format(format) || !wg || !wu || !wd || !x || !act || !y || hidden % 256 || middle % 256 || !hidden ||
      !middle || batch == 0 || batch > kApiMaxBatch)
    return fail(RTA_E_ARG, "rta_mlp_swiglu: bad arguments (hidden, middle multiples of 256; 1 <= batch <= 32)");
  rta::GemvArgs g;
  g.fmt = format;
  g.w0 = static_cast<const uint8_t*>(wg);
  g.w1 = static_cast<const uint8_t*>(wu);
  g.rows = middle;
  g.cols = hidden;
  g.x = x;
  g.x_stride = hidden;
  g.batch = batch;
  g.epilogue = rta::kSwiGLU;
  g.y = act;
  g.y_stride = middle;
  rta_status st = cuda_status(rta::launch_gemv(g, as_stream(stream)), "rta_mlp_swiglu(gate/up)");
  if (st != RTA_OK) return st;
  rta::GemvArgs d;
  d.fmt = format;
  d.w0 = static_cast<const uint8_t*>(wd);
  d.rows = hidden;
  d.cols = middle;
  d.x = act;
  d.x_stride = middle;
  d.batch = batch;
  d.epilogue = accumulate ? rta::kAccumulate : rta::kStore;
  d.y = y;
  d.y_stride = hidden;
  d.pdl = true;
  return cuda_status(rta::launch_gemv(d, as_stream(stream)), "rta_mlp_swiglu(down)");
}

size_t rta_readout_workspace_bytes(uint32_t batch) { return kErrBytes + 8ull * (batch ? batch : 1); }

rta_status rta_readout(int format, const void* w, uint32_t vocab, uint32_t hidden, const float* x, uint32_t batch,
                       float* logits, uint32_t* argmax, float* best, void* workspace, void* stream) {
  if (!gemv_format(format) || !w || !x || !argmax || !workspace || vocab == 0 || vocab % 16 || hidden % 256 ||
      hidden == 0 || batch == 0 || batch > 64)
    return fail(RTA_E_ARG, "rta_readout: bad arguments (vocab % 16 == 0, hidden % 256 == 0, 1 <= batch <= 64)");
  cudaStream_t s = as_stream(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  auto* keys = reinterpret_cast<unsigned long long*>(ws + kErrBytes);
  rta_status st = cuda_status(cudaMemsetAsync(ws, 0, rta_readout_workspace_bytes(batch), s), "rta_readout(memset)");
  if (st != RTA_OK) return st;
  rta::GemvArgs a;
  a.fmt = format;
  a.w0 = static_cast<const uint8_t*>(w);
  a.rows = vocab;
  a.cols = hidden;
  a.x = x;
  a.x_stride = hidden;
  a.batch = batch;
  a.epilogue = rta::kStore;
  a.y = logits;
  a.y_stride = vocab;
  a.argmax = keys;
  a.err = err;
  st = cuda_status(rta::launch_gemv(a, s), "rta_readout");
  if (st != RTA_OK) return st;
  readout_finish_kernel<<<1, (batch + 31u) / 32u * 32u, 0, s>>>(keys, batch, vocab, argmax, best, err);
  return cuda_status(cudaGetLastError(), "rta_readout(finish)");
}

size_t rta_attention_workspace_bytes(uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t splits) {
  (void)kv_heads;
  const size_t recs = static_cast<size_t>(heads) * (splits ? splits : 1);
  return kErrBytes + recs * 4 * 2 + recs * head_dim * 4 + 64;
}

uint32_t rta_attention_default_splits(uint32_t history, uint32_t kv_heads) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return rta::attention_default_splits(history, kv_heads, sms);
}

rta_status rta_attention_decode_f16(const float* q, const void* k, const void* v, uint32_t time, uint32_t capacity,
                                    uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t pos_stride,
                                    uint32_t kv_stride, const float* gate, float* out, float* phys, uint32_t splits,
                                    void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !out || !workspace || head_dim != 256 || kv_heads == 0 || heads != 4 * kv_heads ||
      capacity == 0 || splits == 0 || splits > 1024)
    return fail(RTA_E_ARG, "rta_attention_decode_f16: head_dim 256, heads == 4*kv_heads, capacity > 0, 1 <= splits <= 1024");
  if (workspace_bytes < rta_attention_workspace_bytes(heads, kv_heads, head_dim, splits))
    return fail(RTA_E_ARG, "rta_attention_decode_f16: workspace too small");
  if (reinterpret_cast<uintptr_t>(k) % 16 || reinterpret_cast<uintptr_t>(v) % 16)
    return fail(RTA_E_ARG, "rta_attention_decode_f16: k and v must be 16-byte aligned (rows are copied in 16-byte "
                           "units)");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t recs = static_cast<size_t>(heads) * splits;
  rta::AttnParams p;
  p.q = q;
  p.q_seq_stride = static_cast<size_t>(heads) * head_dim;
  p.k = static_cast<const __half*>(k);
  p.v = static_cast<const __half*>(v);
  p.seq_stride = 0;
  p.kv_stride = static_cast<size_t>(kv_stride) * head_dim;
  p.pos_stride = static_cast<size_t>(pos_stride) * head_dim;
  p.heads = heads;
  p.kvh = kv_heads;
  p.hd = head_dim;
  p.capacity = capacity;
  p.history_start = 0;
  p.t = time;
  p.gate = gate;
  p.out = out;
  p.out_seq_stride = static_cast<size_t>(heads) * head_dim;
  p.phys = phys;
  p.err = reinterpret_cast<uint32_t*>(ws);
  // split records from the first 16-byte boundary past the error word (the
  // workspace size carries 64 bytes of slack): the merge reads float4 rows
  p.part_m = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(ws + kErrBytes) + 15u) & ~uintptr_t{15});
  p.part_z = p.part_m + recs;
  p.part_o = p.part_z + recs;
  cudaStream_t s = as_stream(stream);
  rta_status st = cuda_status(cudaMemsetAsync(ws, 0, 4, s), "rta_attention_decode_f16(memset)");
  if (st != RTA_OK) return st;
  return cuda_status(rta::launch_attention(p, splits, 1, false, s), "rta_attention_decode_f16");
}

rta_status rta_gated_delta_step(const float* x, const float* attn_norm, const float* w_alpha, const float* w_beta,
                                const float* a_log, const float* dt_bias, const float* proj, uint32_t proj_stride,
                                const float* conv_w, float* conv_state, float* state, float* out,
                                const uint32_t* positions, uint32_t hidden, uint32_t heads, uint32_t key_heads,
                                uint32_t batch, float eps, uint32_t* device_error, void* stream) {
  if (!x || !attn_norm || !w_alpha || !w_beta || !a_log || !dt_bias || !proj || !conv_w || !conv_state || !state ||
      !out || !positions)
    return fail(RTA_E_ARG, "rta_gated_delta_step: null argument");
  if (hidden == 0 || hidden > 4096 || hidden % 4 || heads == 0 || key_heads == 0 || heads % key_heads || batch == 0 ||
      batch > 1024 || proj_stride < 2u * key_heads * 128u + heads * 128u)
    return fail(RTA_E_ARG, "rta_gated_delta_step: hidden 4..4096 (multiple of 4), heads a multiple of key_heads, "
                           "batch 1..1024, proj_stride >= 2 * key_heads * 128 + heads * 128");
  const auto misaligned = [](const void* q, uintptr_t a) { return reinterpret_cast<uintptr_t>(q) % a != 0; };
  if (misaligned(x, 16) || misaligned(attn_norm, 16) || misaligned(w_alpha, 16) || misaligned(w_beta, 16) ||
      misaligned(conv_w, 16) || misaligned(state, 8) || (static_cast<size_t>(hidden) * 4) % 16)
    return fail(RTA_E_ARG, "rta_gated_delta_step: x, attn_norm, w_alpha, w_beta and conv_w must be 16-byte "
                           "aligned, state 8-byte aligned");
  const uint32_t S = heads * 128u;
  rta::GdnParams p;
  p.x = x;
  p.attn_norm = attn_norm;
  p.eps = eps;
  p.wa = w_alpha;
  p.wb = w_beta;
  p.a_log = a_log;
  p.dt_bias = dt_bias;
  p.proj = proj;
  p.conv_w = conv_w;
  p.conv_state = conv_state;
  p.rec = state;
  p.out = out;
  p.D = hidden;
  p.H = heads;
  p.KH = key_heads;
  p.pos = positions;
  p.running = nullptr;
  p.err = device_error;
  p.err_step = 0;
  p.nseq = batch;
  p.ctrl_step = 1;
  p.proj_seq = proj_stride;
  p.conv_seq = static_cast<size_t>(2) * 3 * S * 3;
  p.rec_seq = static_cast<size_t>(heads) * 128 * 128;
  cudaStream_t s = as_stream(stream);
  if (device_error) {
    rta_status st = cuda_status(cudaMemsetAsync(device_error, 0, 4, s), "rta_gated_delta_step(memset)");
    if (st != RTA_OK) return st;
  }
  return cuda_status(rta::launch_gdn(p, s, false), "rta_gated_delta_step");
}

rta_status rta_workspace_error(const void* workspace, size_t workspace_bytes, void* stream, uint32_t* error_word) {
  if (!workspace || workspace_bytes < 4 || !error_word) return fail(RTA_E_ARG, "rta_workspace_error: bad arguments");
  uint32_t w = 0;
  cudaStream_t s = as_stream(stream);
  rta_status st = cuda_status(cudaMemcpyAsync(&w, workspace, 4, cudaMemcpyDeviceToHost, s), "rta_workspace_error");
  if (st != RTA_OK) return st;
  st = cuda_status(cudaStreamSynchronize(s), "rta_workspace_error(sync)");
  if (st != RTA_OK) return st;
  *error_word = w;
  if (w & RTA_DEVERR_TIMEOUT) return fail(RTA_E_TIMEOUT, "device-side wait exceeded its bound");
  if (w) return fail(RTA_E_DEVICE_CHECK, "device error word " + std::to_string(w));
  return RTA_OK;
}

}  // extern "C"
