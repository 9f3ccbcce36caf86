// layers.cu -- per-token kernels of the resident decode step that sit between
// the GEMVs: token readout->embedding control, QK-norm + RoPE + history append
// for full-attention layers, and the fused recurrent (gated delta rule) layer.
#include "layers.h"
#include "rta_internal.h"

namespace rta {
namespace {

__device__ __forceinline__ float block_sum256(float v, float* red) {
  // 256 threads: 8 warps
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) red[8] = s;
  }
  __syncthreads();
  return red[8];
}

__device__ __forceinline__ float q6k_row_value(const uint8_t* b, uint32_t index) {
  const uint32_t half = index / 128u, local = index % 128u;
  const uint32_t ql = (b[half * 64u + local % 64u] >> ((local / 64u) * 4u)) & 15u;
  const uint32_t qh = (b[128u + half * 32u + local % 32u] >> ((local / 32u) * 2u)) & 3u;
  const int scale = static_cast<int>(static_cast<int8_t>(b[192u + index / 16u]));
  const float d = half_bits_to_float(b[208] | (b[209] << 8));
  return (d * static_cast<float>(scale)) * static_cast<float>(static_cast<int>(ql | (qh << 4)) - 32);
}
__device__ __forceinline__ float q4k_row_value(const uint8_t* b, uint32_t index) {
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
  const uint32_t q = (b[16 + (index / 64u) * 32u + index % 32u] >> ((index % 64u) / 32u * 4u)) & 15u;
  const float d = half_bits_to_float(b[0] | (b[1] << 8)), dmin = half_bits_to_float(b[2] | (b[3] << 8));
  return (d * static_cast<float>(sc)) * static_cast<float>(q) - dmin * static_cast<float>(mn);
}

// ------------------------------------------------------------------ embed
// Decode mode: consume the readout's argmax (ops 17/23 of resident_math.comp:
// token, output append, stop check), then op 0 (embedding row -> state).
// Prefill mode: the token is the prompt id at the next position.
__global__ void __launch_bounds__(256) embed_kernel(EmbedParams p) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ uint32_t token_s, go_s;
  Control* c = p.ctrl;
  if (threadIdx.x == 0) {
    uint32_t token = 0xffffffffu, go = 0u;
    if (p.mode == kEmbedDecode) {
      if (c->running) {
        const unsigned long long key = c->argkey;
        c->argkey = 0ull;
        token = ~static_cast<uint32_t>(key & 0xffffffffull);
        if (key == 0ull || token >= p.vocab) {
          atomicOr(&c->err, RTA_DEVERR_TOKEN);
          c->running = 0u;
        } else {
          if (c->n_out < kMaxOut) c->ids[c->n_out] = token;
          c->n_out += 1u;
          c->best_key = key;
          if (token == c->stops[0] || token == c->stops[1]) c->running = 0u;
          else go = 1u;
        }
      }
    } else {
      token = p.prompt[c->pos_next];
      go = token < p.vocab ? 1u : 0u;
      if (!go) atomicOr(&c->err, RTA_DEVERR_TOKEN);
    }
    if (go) {
      c->pos_cur = c->pos_next;
      c->pos_next += 1u;
    }
    token_s = token;
    go_s = go;
  }
  __syncthreads();
  if (!go_s) return;
  const uint8_t* row = p.table + static_cast<size_t>(token_s) * p.row_bytes;
  const uint32_t bb = p.fmt == kQ4K ? 144u : 210u;
  for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) {
    const uint8_t* blk = row + (i / 256u) * bb;
    p.state[i] = p.fmt == kQ4K ? q4k_row_value(blk, i % 256u) : q6k_row_value(blk, i % 256u);
  }
}

// ------------------------------------------------------------ attn prep
// Op 14 (per-head RMS QK-norm, resident_math.comp:113-114), op 3 (RoPE on
// adjacent pairs with coordinatePhase, :76-77, resident_common.glsl:117) and
// the history write (op 34's role) for one token: K and V go to the fp16 ring
// slot pos % capacity.  One CTA per query head, then one per KV head.
__global__ void __launch_bounds__(256) attn_prep_kernel(PrepParams p) {
  pdl_wait();
  pdl_launch_dependents();
  if (p.running && *p.running == 0u) return;
  __shared__ float red[16];
  __shared__ float xs[256];
  const uint32_t d = threadIdx.x, hd = p.hd;
  const uint32_t pos = *p.pos;
  const bool is_q = blockIdx.x < p.heads;
  const uint32_t head = is_q ? blockIdx.x : blockIdx.x - p.heads;
  const float* src = is_q ? p.qkvg + head * hd : p.qkvg + p.q_width + head * hd;
  float x = d < hd ? src[d] : 0.f;
  if (p.qk_norm) {
    const float ss = block_sum256(x * x, red);
    const float inv = rsqrtf(ss / static_cast<float>(hd) + p.eps);
    // key heads use the weights of their first GQA copy (the table is tiled per query head)
    const float* w = is_q ? p.qnorm + head * hd : p.knorm + head * p.group * hd;
    if (d < hd) x = x * (inv * w[d]);
  }
  if (d < hd) xs[d] = x;
  __syncthreads();
  const uint32_t pair = d / 2u;
  if (d < hd && pair < p.rotary / 2u) {
    const float phase = static_cast<float>(pos) * p.inv_freq[pair];
    float sn, cs;
    sincosf(phase, &sn, &cs);
    const float a = xs[d & ~1u], b = xs[d | 1u];
    x = (d & 1u) ? a * sn + b * cs : a * cs - b * sn;
  }
  if (d >= hd) return;
  if (is_q) {
    p.qout[head * hd + d] = x;
  } else {
    const size_t slot = static_cast<size_t>(pos % p.capacity);
    const size_t at = (static_cast<size_t>(head) * p.capacity + slot) * hd + d;
    p.kcache[at] = __float2half_rn(x);
    const float v = p.qkvg[p.q_width + p.kv_width + head * hd + d];
    p.vcache[at] = __float2half_rn(v);
  }
}

// ------------------------------------------------------------------ GDN
// One recurrent layer (ops 18-21 of resident_math.comp:131-148): gates
// decay = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b) from the
// RMS-normed layer input; 4-tap causal conv + SiLU; L2-normalised q, k; and the
// gated delta rule s <- s*decay; r = k.s; s += k*(v - r)*beta; o = (q/sqrt(128)).s
// on a [128 value x 128 key] fp32 state per head.  Grid (head, value slice).
constexpr uint32_t kGdnRows = 32;  // value rows per CTA (8 warps x 4)

__device__ __forceinline__ float signed_product_sum(float a0, float a1, float a2, float a3, float b0, float b1,
                                                    float b2, float b3) {
  // E+ - E- of resident_common.glsl:137 (signedEnergy): positive and negative
  // product energies are reduced separately, then subtracted.
  float P = 0.f, M = 0.f;
  const float pr[4] = {a0 * b0, a1 * b1, a2 * b2, a3 * b3};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float e = fabsf(pr[i]);
    if (pr[i] > 0.f) P += e;
    else if (pr[i] < 0.f) M += e;
  }
  return warp_sum(P) - warp_sum(M);
}

__global__ void __launch_bounds__(256) gdn_kernel(GdnParams p) {
  pdl_wait();
  pdl_launch_dependents();
  if (p.running && *p.running == 0u) return;
  __shared__ float red[16];
  __shared__ float qn[128], kn[128], vv[kGdnRows];
  __shared__ float gates[2];
  const uint32_t h = blockIdx.x, slice = blockIdx.y, tid = threadIdx.x;
  const uint32_t HD = 128u, S = p.H * HD, K = p.KH * HD, kh = h % p.KH;
  const uint32_t par = (*p.pos) & 1u;
  const float* past = p.conv_state + static_cast<size_t>(par) * 3u * S * 3u;
  float* next = p.conv_state + static_cast<size_t>(par ^ 1u) * 3u * S * 3u;

  // gates: a, b = (rmsnorm(x) * attn_norm) . W_alpha[h], W_beta[h]
  float ss = 0.f;
  for (uint32_t c = tid; c < p.D; c += blockDim.x) ss += p.x[c] * p.x[c];
  const float inv = rsqrtf(block_sum256(ss, red) / static_cast<float>(p.D) + p.eps);
  float a = 0.f, b = 0.f;
  for (uint32_t c = tid; c < p.D; c += blockDim.x) {
    const float xn = p.x[c] * inv * p.attn_norm[c];
    a += xn * p.wa[static_cast<size_t>(h) * p.D + c];
    b += xn * p.wb[static_cast<size_t>(h) * p.D + c];
  }
  a = block_sum256(a, red);
  b = block_sum256(b, red);
  if (tid == 0) {
    gates[0] = expf(-expf(p.a_log[h]) * softplus(a + p.dt_bias[h]));
    gates[1] = detector_sigmoid(b);
  }

  // causal conv + SiLU for q, k (128 each) and this slice's v channels
  auto conv = [&](uint32_t coord, float raw, bool write) {
    const float* w = p.conv_w + static_cast<size_t>(coord) * 4u;
    const float* pc = past + static_cast<size_t>(coord) * 3u;
    float signal = 0.f;
    signal = signal + pc[0] * w[0];
    signal = signal + pc[1] * w[1];
    signal = signal + pc[2] * w[2];
    signal = signal + raw * w[3];
    if (write) {
      float* nc = next + static_cast<size_t>(coord) * 3u;
      nc[0] = pc[1];
      nc[1] = pc[2];
      nc[2] = raw;
    }
    return signal * detector_sigmoid(signal);
  };
  if (tid < 128u) {
    qn[tid] = conv(h * HD + tid, p.proj[kh * HD + tid], slice == 0);
  } else {
    const uint32_t c = tid - 128u;
    kn[c] = conv(S + h * HD + c, p.proj[K + kh * HD + c], slice == 0);
  }
  if (tid < kGdnRows) {
    const uint32_t c = slice * kGdnRows + tid;
    vv[tid] = conv(2u * S + h * HD + c, p.proj[2u * K + h * HD + c], true);
  }
  __syncthreads();
  // L2 norms (op 20): q * inversesqrt(sum q^2 + eps), same for k
  const float qv = tid < 128u ? qn[tid] : 0.f, kv = tid < 128u ? kn[tid] : 0.f;
  const float qs = rsqrtf(block_sum256(qv * qv, red) + p.eps);
  const float ks = rsqrtf(block_sum256(kv * kv, red) + p.eps);
  if (tid < 128u) {
    qn[tid] = (qv * qs) / sqrtf(128.0f);
    kn[tid] = kv * ks;
  }
  __syncthreads();
  const float decay = gates[0], beta = gates[1];
  const uint32_t warp = tid >> 5, lane = tid & 31u;
  // lane owns keys (2l, 2l+1) and (2l+64, 2l+65), as fieldPair of op 21
  const float k0 = kn[2 * lane], k1 = kn[2 * lane + 1], k2 = kn[2 * lane + 64], k3 = kn[2 * lane + 65];
  const float q0 = qn[2 * lane], q1 = qn[2 * lane + 1], q2 = qn[2 * lane + 64], q3 = qn[2 * lane + 65];
  float* st = p.rec + static_cast<size_t>(h) * HD * HD;
  for (uint32_t i = 0; i < kGdnRows / 8u; ++i) {
    const uint32_t r = warp * (kGdnRows / 8u) + i, v = slice * kGdnRows + r;
    float* row = st + static_cast<size_t>(v) * HD;
    float2 s0 = *reinterpret_cast<float2*>(row + 2 * lane);
    float2 s1 = *reinterpret_cast<float2*>(row + 2 * lane + 64);
    s0.x *= decay;
    s0.y *= decay;
    s1.x *= decay;
    s1.y *= decay;
    const float received = signed_product_sum(k0, k1, k2, k3, s0.x, s0.y, s1.x, s1.y);
    const float delta = (vv[r] - received) * beta;
    s0.x += k0 * delta;
    s0.y += k1 * delta;
    s1.x += k2 * delta;
    s1.y += k3 * delta;
    const float o = signed_product_sum(q0, q1, q2, q3, s0.x, s0.y, s1.x, s1.y);
    *reinterpret_cast<float2*>(row + 2 * lane) = s0;
    *reinterpret_cast<float2*>(row + 2 * lane + 64) = s1;
    if (lane == 0) p.out[h * HD + v] = o;
  }
}

// Row gather used at load time (rotary row permutations, concatenations).
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, const uint32_t* __restrict__ map, uint32_t rows,
                                   uint32_t row_bytes, uint8_t* __restrict__ dst) {
  const uint32_t r = blockIdx.x;
  if (r >= rows) return;
  const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<size_t>(map[r]) * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + static_cast<size_t>(r) * row_bytes);
  for (uint32_t i = threadIdx.x; i < row_bytes / 16u; i += blockDim.x) d[i] = s[i];
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t s, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_embed(const EmbedParams& p, cudaStream_t s, bool pdl) {
  void* args[] = {const_cast<EmbedParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(embed_kernel), dim3(1), dim3(256), args, s, pdl);
}
cudaError_t launch_attn_prep(const PrepParams& p, cudaStream_t s, bool pdl) {
  if (p.hd > 256) return cudaErrorInvalidValue;
  void* args[] = {const_cast<PrepParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(attn_prep_kernel), dim3(p.heads + p.kvh), dim3(256), args, s, pdl);
}
cudaError_t launch_gdn(const GdnParams& p, cudaStream_t s, bool pdl) {
  void* args[] = {const_cast<GdnParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(gdn_kernel), dim3(p.H, 128u / kGdnRows), dim3(256), args, s,
                    pdl);
}
cudaError_t launch_gather_rows(const uint8_t* src, const uint32_t* map, uint32_t rows, uint32_t row_bytes,
                               uint8_t* dst, cudaStream_t s) {
  if (row_bytes % 16 || reinterpret_cast<uintptr_t>(src) % 16 || reinterpret_cast<uintptr_t>(dst) % 16)
    return cudaErrorMisalignedAddress;
  if (rows == 0) return cudaSuccess;
  gather_rows_kernel<<<rows, 128, 0, s>>>(src, map, rows, row_bytes, dst);
  return cudaGetLastError();
}

}  // namespace rta
