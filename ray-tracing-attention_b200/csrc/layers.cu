// layers.cu -- per-token kernels of the resident decode step that sit between
// the GEMVs: token readout->embedding control, QK-norm + RoPE + history append
// for full-attention layers, and the fused recurrent (gated delta rule) layer.
#include <atomic>

#include "layers.h"
#include "packets.cuh"
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
  const uint32_t z = blockIdx.x;  // sequence
  Control* c = p.ctrl + z;
  if (threadIdx.x == 0) {
    // every control word this step needs, read at once (one round trip)
    const unsigned long long key = c->argkey;
    const uint32_t running = c->running, n_out = c->n_out, pos_next = c->pos_next;
    const uint32_t stop0 = c->stops[0], stop1 = c->stops[1];
    uint32_t token = 0xffffffffu, go = 0u;
    if (p.mode == kEmbedDecode) {
      if (running) {
        c->argkey = 0ull;
        token = ~static_cast<uint32_t>(key & 0xffffffffull);
        if (key == 0ull || token >= p.vocab) {
          atomicOr(&c->err, RTA_DEVERR_TOKEN);
          c->running = 0u;
        } else {
          if (n_out < kMaxOut) c->ids[n_out] = token;
          c->n_out = n_out + 1u;
          c->best_key = key;
          if (token == stop0 || token == stop1) c->running = 0u;
          else go = 1u;
        }
      }
    } else {
      // a sequence whose prompt is consumed sits out the remaining prefill steps
      if (running && pos_next < c->prompt_len) {
        token = p.prompt[static_cast<size_t>(z) * p.prompt_stride + pos_next];
        go = token < p.vocab ? 1u : 0u;
        if (!go) {
          atomicOr(&c->err, RTA_DEVERR_TOKEN);
          c->running = 0u;
        }
      } else if (running) {
        c->running = 0u;
      }
    }
    if (go) {
      c->pos_cur = pos_next;
      c->pos_next = pos_next + 1u;
    }
    token_s = token;
    go_s = go;
  }
  __syncthreads();
  if (!go_s) return;
  const uint8_t* row = p.table + static_cast<size_t>(token_s) * p.row_bytes;
  if (p.fmt == kF32 || p.fmt == kF16 || p.fmt == kBF16) {  // dense rows (ggufValue's first branches)
    float* st = p.state + static_cast<size_t>(z) * p.D;
    for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) {
      float v;
      if (p.fmt == kF32) {
        v = reinterpret_cast<const float*>(row)[i];
      } else {
        const uint32_t h = reinterpret_cast<const uint16_t*>(row)[i];
        v = p.fmt == kF16 ? half_bits_to_float(h) : __uint_as_float(h << 16);
      }
      st[i] = v;
    }
    return;
  }
  const uint32_t bb = p.fmt == kQ4K ? 144u : 210u;
  float* state = p.state + static_cast<size_t>(z) * p.D;
  for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) {
    const uint8_t* blk = row + (i / 256u) * bb;
    state[i] = p.fmt == kQ4K ? q4k_row_value(blk, i % 256u) : q6k_row_value(blk, i % 256u);
  }
}

// ----------------------------------------------------------- prefill chunk
__device__ __forceinline__ float embed_value(const ChunkParams& p, const uint8_t* row, uint32_t i) {
  if (p.fmt == kF32) return reinterpret_cast<const float*>(row)[i];
  if (p.fmt == kF16 || p.fmt == kBF16) {
    const uint32_t h = reinterpret_cast<const uint16_t*>(row)[i];
    return p.fmt == kF16 ? half_bits_to_float(h) : __uint_as_float(h << 16);
  }
  const uint8_t* blk = row + (i / 256u) * (p.fmt == kQ4K ? 144u : 210u);
  return p.fmt == kQ4K ? q4k_row_value(blk, i % 256u) : q6k_row_value(blk, i % 256u);
}
// CTA r: row r of the chunk.
__global__ void __launch_bounds__(256) chunk_begin_kernel(ChunkParams p) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ uint32_t token_s, live_s;
  const uint32_t r = blockIdx.x;
  if (threadIdx.x == 0) {
    const uint32_t pos = p.ctrl->pos_next + r;
    uint32_t live = p.ctrl->running && pos < p.ctrl->prompt_len ? 1u : 0u;
    const uint32_t token = live ? p.prompt[pos] : 0u;
    if (live && token >= p.vocab) {
      atomicOr(&p.ctrl->err, RTA_DEVERR_TOKEN);
      live = 0u;
    }
    p.rowctl[2u * r] = pos;
    p.rowctl[2u * r + 1u] = live;
    token_s = token;
    live_s = live;
  }
  __syncthreads();
  float* dst = p.rows + static_cast<size_t>(r) * p.D;
  const uint8_t* row = p.table + static_cast<size_t>(token_s) * p.row_bytes;
  for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) dst[i] = live_s ? embed_value(p, row, i) : 0.f;
}
__global__ void __launch_bounds__(256) chunk_end_kernel(ChunkParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t next = p.ctrl->pos_next, plen = p.ctrl->prompt_len;
  const uint32_t live = p.ctrl->running && next < plen ? min(p.C, plen - next) : 0u;
  if (live == 0u) return;
  const float* src = p.rows + static_cast<size_t>(live - 1u) * p.D;
  for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) p.state[i] = src[i];
  __syncthreads();  // every thread has read the control words above
  if (threadIdx.x == 0) {
    p.ctrl->pos_cur = next + live - 1u;
    p.ctrl->pos_next = next + live;
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
  const uint32_t z = blockIdx.y;  // sequence
  __shared__ float red[16];
  __shared__ float xs[256];
  const uint32_t d = threadIdx.x, hd = p.hd;
  // the running flag, the position and this head's row travel in one round trip
  const uint32_t run = p.running ? p.running[z * p.ctrl_step] : 1u;
  const uint32_t pos = p.pos[z * p.ctrl_step];
  const bool is_q = blockIdx.x < p.heads;
  const uint32_t head = is_q ? blockIdx.x : blockIdx.x - p.heads;
  const float* qkvg = p.qkvg + z * p.qkvg_seq;
  const float* src = is_q ? qkvg + head * hd : qkvg + p.q_width + head * hd;
  float x = d < hd ? src[d] : 0.f;
  if (run == 0u) return;
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
  if (p.packets && !is_q) {  // op 34: pack this KV head's K (Q4_K) and V (Q6_K) into the position's packet
    __shared__ PackScratch sh;
    const size_t row = static_cast<size_t>(z * p.ring_seq) * p.capacity + pos % p.capacity;
    uint8_t* pkt = p.packets + row * packet_bytes(p.kvh);
    pack_q4k_block(x, pkt + head * kPacketKeyBytes, sh);
    pack_q6k_block(qkvg[p.q_width + p.kv_width + head * hd + d],
                   pkt + p.kvh * kPacketKeyBytes + head * kPacketValueBytes, sh);
    return;
  }
  if (d >= hd) return;
  if (is_q) {
    p.qout[(static_cast<size_t>(z) * p.heads + head) * hd + d] = x;
  } else {
    const size_t slot = static_cast<size_t>(pos % p.capacity);
    const size_t at = ((static_cast<size_t>(z * p.ring_seq) * p.kvh + head) * p.capacity + slot) * hd + d;
    p.kcache[at] = __float2half_rn(x);
    const float v = qkvg[p.q_width + p.kv_width + head * hd + d];
    p.vcache[at] = __float2half_rn(v);
  }
}

// ------------------------------------------------------------------ GDN
// One recurrent layer (ops 18-21 of resident_math.comp:131-148): gates
// decay = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b) from the
// RMS-normed layer input; 4-tap causal conv + SiLU; L2-normalised q, k; and the
// gated delta rule s <- s*decay; r = k.s; s += k*(v - r)*beta; o = (q/sqrt(128)).s
// on a [128 value x 128 key] fp32 state per head.  Grid (head, value slice,
// sequence), 16 value rows per CTA: a few sequences split each head's rows over
// 8 CTAs for parallelism at one token (many sequences go to the persistent
// gdn_batch_kernel below).
//
// Latency layout: the kernel is a short chain of dependent steps, so everything
// that does not depend on the preceding kernels (this CTA's state rows, the
// gate / norm / conv weights, the conv history) is requested before
// griddepcontrol.wait, into registers, and the block reductions carry several
// values per barrier.
constexpr uint32_t kGdnRowsSmall = 16;
constexpr uint32_t kGdnPersistentUnits = 64;  // (head, sequence) units from which gdn_batch_kernel runs

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

// Sum of N values over the 256 threads; `red` holds 8*N floats and is used by
// this call only (one barrier).
template <int N>
__device__ __forceinline__ void block_sums(float (&v)[N], float* red) {
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
  const uint32_t w = threadIdx.x >> 5;
  if ((threadIdx.x & 31u) == 0u)
#pragma unroll
    for (int i = 0; i < N; ++i) red[w * N + i] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += red[j * N + i];
    v[i] = s;
  }
}


constexpr uint32_t kGdnDPer = 16;  // hidden values per thread: hidden size <= 4096

__global__ void __launch_bounds__(256) gdn_kernel(GdnParams p) {
  constexpr uint32_t kGdnRows = kGdnRowsSmall, kGdnRowsPerWarp = kGdnRows / 8u;
  __shared__ float red1[8], red2[16], red3[16];
  __shared__ float qn[128], kn[128], vv[kGdnRows];
  const uint32_t h = blockIdx.x, slice = blockIdx.y, z = blockIdx.z, tid = threadIdx.x;
  const uint32_t HD = 128u, S = p.H * HD, K = p.KH * HD, kh = h % p.KH;
  const uint32_t warp = tid >> 5, lane = tid & 31u;
  const float* x_seq = p.x + static_cast<size_t>(z) * p.D;
  const float* proj = p.proj + z * p.proj_seq;
  float* conv_state = p.conv_state + z * p.conv_seq;

  // ---- independent of the preceding kernels: state rows, weights, conv history
  float* st = p.rec + z * p.rec_seq + static_cast<size_t>(h) * HD * HD;
  float2 s0[kGdnRowsPerWarp], s1[kGdnRowsPerWarp];
#pragma unroll
  for (uint32_t i = 0; i < kGdnRowsPerWarp; ++i) {
    const float* row = st + static_cast<size_t>(slice * kGdnRows + warp * kGdnRowsPerWarp + i) * HD;
    s0[i] = *reinterpret_cast<const float2*>(row + 2 * lane);   // lane owns keys (2l, 2l+1) and
    s1[i] = *reinterpret_cast<const float2*>(row + 2 * lane + 64);  // (2l+64, 2l+65), as op 21
  }
  // The gate weights and the norm weight of this thread's hidden values
  // (c = tid + 256 i) are held in registers, read before the wait.
  constexpr uint32_t kPer = kGdnDPer;
  float nw[kPer], wa[kPer], wb[kPer], xr[kPer];
#pragma unroll
  for (uint32_t i = 0; i < kPer; ++i) {
    const uint32_t c = tid + 256u * i;
    const bool in = c < p.D;
    nw[i] = in ? p.attn_norm[c] : 0.f;
    wa[i] = in ? p.wa[static_cast<size_t>(h) * p.D + c] : 0.f;
    wb[i] = in ? p.wb[static_cast<size_t>(h) * p.D + c] : 0.f;
  }
  // The conv history is double-buffered by position parity; the position is
  // written by this step's embed kernel, so both buffers are read here and the
  // choice is made after the wait.
  const size_t buf = static_cast<size_t>(3u) * S * 3u;
  // this thread's conv channel: q (tid < 128) or k (tid >= 128), plus v rows for tid < kGdnRows
  const uint32_t qk_coord = tid < 128u ? h * HD + tid : S + h * HD + (tid - 128u);
  const uint32_t v_coord = 2u * S + h * HD + slice * kGdnRows + (tid % kGdnRows);
  const float4 wq = *reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(qk_coord) * 4u);
  float pq[2][3], pv[2][3] = {{0.f, 0.f, 0.f}, {0.f, 0.f, 0.f}};
#pragma unroll
  for (int b = 0; b < 2; ++b)
#pragma unroll
    for (int j = 0; j < 3; ++j) pq[b][j] = conv_state[b * buf + qk_coord * 3u + j];
  float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid < kGdnRows) {
    wv = *reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(v_coord) * 4u);
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int j = 0; j < 3; ++j) pv[b][j] = conv_state[b * buf + v_coord * 3u + j];
  }
  const float a_log = p.a_log[h], dt_bias = p.dt_bias[h];

  pdl_wait();
  pdl_launch_dependents();
  // every load that depends on the preceding kernels is issued before the first
  // use, so they share one round trip
  const uint32_t run = p.running ? p.running[z * p.ctrl_step] : 1u;
  const uint32_t posv = p.pos[z * p.ctrl_step];
#pragma unroll
  for (uint32_t i = 0; i < kPer; ++i) {
    const uint32_t c = tid + 256u * i;
    xr[i] = c < p.D ? x_seq[c] : 0.f;
  }
  const float raw_q = proj[tid < 128u ? kh * HD + tid : K + kh * HD + (tid - 128u)];
  const float raw_v = tid < kGdnRows ? proj[2u * K + h * HD + slice * kGdnRows + tid] : 0.f;
  if (run == 0u) return;
  const uint32_t par = posv & 1u;
  float* next = conv_state + (par ^ 1u) * buf;
  const float pq0 = par ? pq[1][0] : pq[0][0], pq1 = par ? pq[1][1] : pq[0][1], pq2 = par ? pq[1][2] : pq[0][2];
  const float pv0 = par ? pv[1][0] : pv[0][0], pv1 = par ? pv[1][1] : pv[0][1], pv2 = par ? pv[1][2] : pv[0][2];

  // ---- op 18 gates: a, b = (rmsnorm(x) * attn_norm) . W_alpha[h], W_beta[h]
  float ss[1] = {0.f};
#pragma unroll
  for (uint32_t i = 0; i < kPer; ++i)
    if (tid + 256u * i < p.D) ss[0] += xr[i] * xr[i];
  block_sums<1>(ss, red1);
  const float inv = rsqrtf(ss[0] / static_cast<float>(p.D) + p.eps);
  float ab[2] = {0.f, 0.f};
#pragma unroll
  for (uint32_t i = 0; i < kPer; ++i) {
    if (tid + 256u * i >= p.D) continue;
    const float xn = xr[i] * inv * nw[i];
    ab[0] += xn * wa[i];
    ab[1] += xn * wb[i];
  }

  // ---- op 19: causal conv + SiLU (independent of the gates)
  auto conv = [](float4 w, float c0, float c1, float c2, float raw) {
    float signal = 0.f;
    signal = signal + c0 * w.x;
    signal = signal + c1 * w.y;
    signal = signal + c2 * w.z;
    signal = signal + raw * w.w;
    return signal * detector_sigmoid(signal);
  };
  const float f = conv(wq, pq0, pq1, pq2, raw_q);
  if (slice == 0u) {
    float* nc = next + static_cast<size_t>(qk_coord) * 3u;
    nc[0] = pq1;
    nc[1] = pq2;
    nc[2] = raw_q;
  }
  if (tid < kGdnRows) {
    vv[tid] = conv(wv, pv0, pv1, pv2, raw_v);
    float* nc = next + static_cast<size_t>(v_coord) * 3u;
    nc[0] = pv1;
    nc[1] = pv2;
    nc[2] = raw_v;
  }
  block_sums<2>(ab, red2);
  const float decay = expf(-expf(a_log) * softplus(ab[0] + dt_bias));
  const float beta = detector_sigmoid(ab[1]);

  // ---- op 20: L2 norms, q * inversesqrt(sum q^2 + eps), same for k
  float qk2[2] = {tid < 128u ? f * f : 0.f, tid >= 128u ? f * f : 0.f};
  block_sums<2>(qk2, red3);
  if (tid < 128u) qn[tid] = (f * rsqrtf(qk2[0] + p.eps)) / sqrtf(128.0f);
  else kn[tid - 128u] = f * rsqrtf(qk2[1] + p.eps);
  __syncthreads();

  // ---- op 21: gated delta rule on this warp's value rows
  const float k0 = kn[2 * lane], k1 = kn[2 * lane + 1], k2 = kn[2 * lane + 64], k3 = kn[2 * lane + 65];
  const float q0 = qn[2 * lane], q1 = qn[2 * lane + 1], q2 = qn[2 * lane + 64], q3 = qn[2 * lane + 65];
#pragma unroll
  for (uint32_t i = 0; i < kGdnRowsPerWarp; ++i) {
    const uint32_t r = warp * kGdnRowsPerWarp + i, v = slice * kGdnRows + r;
    float2 a = s0[i], b = s1[i];
    a.x *= decay;
    a.y *= decay;
    b.x *= decay;
    b.y *= decay;
    const float received = signed_product_sum(k0, k1, k2, k3, a.x, a.y, b.x, b.y);
    const float delta = (vv[r] - received) * beta;
    a.x += k0 * delta;
    a.y += k1 * delta;
    b.x += k2 * delta;
    b.y += k3 * delta;
    const float o = signed_product_sum(q0, q1, q2, q3, a.x, a.y, b.x, b.y);
    float* row = st + static_cast<size_t>(v) * HD;
    *reinterpret_cast<float2*>(row + 2 * lane) = a;
    *reinterpret_cast<float2*>(row + 2 * lane + 64) = b;
    if (lane == 0) p.out[static_cast<size_t>(z) * S + h * HD + v] = o;
  }
}

// Batched recurrent layer (many sequences): one persistent CTA per SM walks
// an equal contiguous range of (head, sequence) units in head-major order.
// Per unit: the [128 value x 128 key] state arrives by one bulk copy into a
// shared stage of a kGdnStages-deep ring, issued units ahead (the first ones
// before griddepcontrol.wait: the state is written only by this layer's
// previous step); the sequence's layer-input row arrives the same way into a
// two-slot ring; the raw projections, conv taps and conv history of the next
// unit are loaded into registers while the current one runs; the gate
// weights of the current head and the norm weight sit in registers.  The RMS
// sum, both gate dot products and both L2 norms share one block reduction
// (a = inv * sum x nw w_a instead of sum (x inv nw) w_a: one multiplication
// moved out of the sum).  The delta rule runs four value rows per warp pass,
// eight lanes per row with sixteen keys each, so each of the row's signed
// reductions (E+ and E- kept apart, as op 21) is a three-level butterfly.
constexpr uint32_t kGdnStages = 3;
constexpr uint32_t kGdnStateFloats = 128u * 128u;
constexpr uint32_t kGdnXSlots = 2;

__global__ void __launch_bounds__(256, 1) gdn_batch_kernel(GdnParams p) {
  extern __shared__ __align__(1024) float gst[];  // [kGdnStages][128][128] state, then [kGdnXSlots][D] input rows
  __shared__ __align__(8) uint64_t full[kGdnStages], xfull[kGdnXSlots];
  __shared__ float red[8 * 5];
  __shared__ float qn[128], kn[128], vv[128];
  __shared__ uint32_t gdn_abort;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
  const uint32_t HD = 128u, S = p.H * HD, K = p.KH * HD;
  const uint32_t U = p.H * p.nseq;
  const uint32_t u0 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x) * U / gridDim.x);
  const uint32_t u1 = static_cast<uint32_t>(static_cast<uint64_t>(blockIdx.x + 1u) * U / gridDim.x);
  float* xring = gst + kGdnStages * kGdnStateFloats;
  auto state_of = [&](uint32_t u) {
    const uint32_t h = u / p.nseq, z = u % p.nseq;
    return p.rec + z * p.rec_seq + static_cast<size_t>(h) * HD * HD;
  };
  uint32_t issued = 0, xissued = 0;  // copies issued (thread 0): states of units u0.., input rows of units u0..
  if (tid == 0) {
    for (uint32_t s = 0; s < kGdnStages; ++s) mbar_init(&full[s], 1);
    for (uint32_t s = 0; s < kGdnXSlots; ++s) mbar_init(&xfull[s], 1);
    fence_mbar_init();
    for (uint32_t i = 0; i < kGdnStages && u0 + i < u1; ++i, ++issued) {
      mbar_expect_tx(&full[i], kGdnStateFloats * 4u);
      bulk_g2s(gst + i * kGdnStateFloats, state_of(u0 + i), kGdnStateFloats * 4u, &full[i]);
    }
    gdn_abort = 0u;
  }
  __syncthreads();
  // constant per CTA: the norm weight of this thread's hidden values c = tid + 256 i
  float nw[kGdnDPer];
#pragma unroll
  for (uint32_t i = 0; i < kGdnDPer; ++i) {
    const uint32_t c = tid + 256u * i;
    nw[i] = c < p.D ? p.attn_norm[c] : 0.f;
  }
  const size_t buf = static_cast<size_t>(3u) * S * 3u;  // floats of one conv-history parity buffer
  // Register inputs of one unit (loaded one unit ahead).
  struct In {
    float raw_q, raw_v, pq[2][3], pv[2][3], a_log, dt_bias;
    float4 wq, wv;
    uint32_t pos, run;
  };
  auto load_in = [&](uint32_t u, In& in) {
    const uint32_t h = u / p.nseq, z = u % p.nseq, kh = h % p.KH;
    const float* proj = p.proj + z * p.proj_seq;
    in.raw_q = proj[tid < 128u ? kh * HD + tid : K + kh * HD + (tid - 128u)];
    in.raw_v = tid < 128u ? proj[2u * K + h * HD + tid] : 0.f;
    const float* cs = p.conv_state + z * p.conv_seq;
    const uint32_t qk = tid < 128u ? h * HD + tid : S + h * HD + (tid - 128u), vc = 2u * S + h * HD + (tid & 127u);
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        in.pq[b][j] = cs[b * buf + qk * 3u + j];
        in.pv[b][j] = tid < 128u ? cs[b * buf + vc * 3u + j] : 0.f;
      }
    in.wq = *reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(qk) * 4u);
    in.wv = *reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(vc) * 4u);
    in.a_log = p.a_log[h];
    in.dt_bias = p.dt_bias[h];
    in.pos = p.pos[z * p.ctrl_step];
    in.run = p.running ? p.running[z * p.ctrl_step] : 1u;
  };
  auto issue_x = [&](uint32_t u) {  // thread 0: the input row of unit u into slot (u - u0) % kGdnXSlots
    const uint32_t slot = (u - u0) % kGdnXSlots, z = u % p.nseq;
    mbar_expect_tx(&xfull[slot], p.D * 4u);
    bulk_g2s(xring + slot * p.D, p.x + static_cast<size_t>(z) * p.D, p.D * 4u, &xfull[slot]);
  };
  auto conv = [](float4 w, float c0, float c1, float c2, float raw) {
    float signal = 0.f;
    signal = signal + c0 * w.x;
    signal = signal + c1 * w.y;
    signal = signal + c2 * w.z;
    signal = signal + raw * w.w;
    return signal * detector_sigmoid(signal);
  };
  // Eight lanes of a warp per value row: lane l takes row (l / 8) of the pass
  // and keys 4 c + 32 j + e (c = l % 8, j, e < 4): four float4 of the row.
  const uint32_t grp = lane >> 3, c8 = lane & 7u;

  pdl_wait();
  pdl_launch_dependents();
  if (tid == 0)
    for (uint32_t i = 0; i < kGdnXSlots && u0 + i < u1; ++i, ++xissued) issue_x(u0 + i);
  In cur, nxt;
  if (u0 < u1) load_in(u0, cur);
  float wa[kGdnDPer], wb[kGdnDPer];
  uint32_t wh = 0xFFFFFFFFu;  // head whose gate rows are in wa / wb
  for (uint32_t u = u0; u < u1; ++u) {
    const uint32_t i = u - u0, stage = i % kGdnStages, xs = i % kGdnXSlots;
    const uint32_t h = u / p.nseq, z = u % p.nseq;
    if (u + 1u < u1) load_in(u + 1u, nxt);
    if (h != wh) {  // the head's gate rows (a head spans nseq consecutive units)
#pragma unroll
      for (uint32_t k = 0; k < kGdnDPer; ++k) {
        const uint32_t c = tid + 256u * k;
        wa[k] = c < p.D ? p.wa[static_cast<size_t>(h) * p.D + c] : 0.f;
        wb[k] = c < p.D ? p.wb[static_cast<size_t>(h) * p.D + c] : 0.f;
      }
      wh = h;
    }
    uint32_t* err = p.err ? p.err + static_cast<size_t>(z) * p.err_step : nullptr;
    const uint32_t qk = tid < 128u ? h * HD + tid : S + h * HD + (tid - 128u), vc = 2u * S + h * HD + (tid & 127u);
    const bool run = cur.run != 0u;
    float v5[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
    float f = 0.f;
    const bool x_ok = mbar_wait(&xfull[xs], (i / kGdnXSlots) & 1u, err);
    if (run && x_ok) {
      // ---- op 18 sums: x^2, x nw w_a, x nw w_b
      const float* xr = xring + xs * p.D;
#pragma unroll
      for (uint32_t k = 0; k < kGdnDPer; ++k) {
        const uint32_t c = tid + 256u * k;
        const float xv = c < p.D ? xr[c] : 0.f, xw = xv * nw[k];
        v5[0] += xv * xv;
        v5[1] += xw * wa[k];
        v5[2] += xw * wb[k];
      }
      // ---- op 19: causal conv + SiLU of this thread's q / k channel (and v channel, tid < 128)
      const uint32_t par = cur.pos & 1u;
      const float c0 = par ? cur.pq[1][0] : cur.pq[0][0], c1 = par ? cur.pq[1][1] : cur.pq[0][1],
                  c2 = par ? cur.pq[1][2] : cur.pq[0][2];
      f = conv(cur.wq, c0, c1, c2, cur.raw_q);
      float* cs = p.conv_state + z * p.conv_seq + (par ^ 1u) * buf;
      float* nc = cs + static_cast<size_t>(qk) * 3u;
      nc[0] = c1;
      nc[1] = c2;
      nc[2] = cur.raw_q;
      if (tid < 128u) {
        const float e0 = par ? cur.pv[1][0] : cur.pv[0][0], e1 = par ? cur.pv[1][1] : cur.pv[0][1],
                    e2 = par ? cur.pv[1][2] : cur.pv[0][2];
        vv[tid] = conv(cur.wv, e0, e1, e2, cur.raw_v);
        float* nv = cs + static_cast<size_t>(vc) * 3u;
        nv[0] = e1;
        nv[1] = e2;
        nv[2] = cur.raw_v;
      }
      v5[3] = tid < 128u ? f * f : 0.f;
      v5[4] = tid >= 128u ? f * f : 0.f;
    }
    block_sums<5>(v5, red);  // uniform: every thread takes part, running or not
    if (!x_ok) gdn_abort = 1u;
    const bool ok = mbar_wait(&full[stage], (i / kGdnStages) & 1u, err);  // the stage has landed
    if (!ok) gdn_abort = 1u;
    if (run && x_ok) {
      const float inv = rsqrtf(v5[0] / static_cast<float>(p.D) + p.eps);
      const float decay = expf(-expf(cur.a_log) * softplus(inv * v5[1] + cur.dt_bias));
      const float beta = detector_sigmoid(inv * v5[2]);
      // ---- op 20: L2 norms
      if (tid < 128u) qn[tid] = (f * rsqrtf(v5[3] + p.eps)) / sqrtf(128.0f);
      else kn[tid - 128u] = f * rsqrtf(v5[4] + p.eps);
      __syncthreads();
      if (ok) {
        // ---- op 21 on this warp's 16 value rows, four per pass, from the stage
        float kk[16], qq[16];
#pragma unroll
        for (uint32_t j = 0; j < 4u; ++j)
#pragma unroll
          for (uint32_t e = 0; e < 4u; ++e) {
            kk[4u * j + e] = kn[4u * c8 + 32u * j + e];
            qq[4u * j + e] = qn[4u * c8 + 32u * j + e];
          }
        const float* sst = gst + stage * kGdnStateFloats;
        float* st = p.rec + z * p.rec_seq + static_cast<size_t>(h) * HD * HD;
#pragma unroll  // the four passes' chains interleave (255 registers, no spills; 82.2 -> 79.8 us per 9B layer)
        for (uint32_t pass = 0; pass < 4u; ++pass) {
          const uint32_t r = warp * 16u + 4u * pass + grp;
          float s[16];
#pragma unroll
          for (uint32_t j = 0; j < 4u; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(sst + r * HD + 4u * c8 + 32u * j);
            s[4u * j] = v.x * decay;
            s[4u * j + 1u] = v.y * decay;
            s[4u * j + 2u] = v.z * decay;
            s[4u * j + 3u] = v.w * decay;
          }
          // received = E+ - E- of k . s over the row's 128 keys (resident_common.glsl:137)
          float P = 0.f, M = 0.f;
#pragma unroll
          for (uint32_t e = 0; e < 16u; ++e) {
            const float pr = kk[e] * s[e];
            if (pr > 0.f) P += pr;
            else if (pr < 0.f) M -= pr;
          }
#pragma unroll
          for (int o = 4; o >= 1; o >>= 1) {
            P += __shfl_xor_sync(0xffffffffu, P, o);
            M += __shfl_xor_sync(0xffffffffu, M, o);
          }
          const float delta = (vv[r] - (P - M)) * beta;
          float P2 = 0.f, M2 = 0.f;
#pragma unroll
          for (uint32_t e = 0; e < 16u; ++e) {
            s[e] += kk[e] * delta;
            const float pr = qq[e] * s[e];
            if (pr > 0.f) P2 += pr;
            else if (pr < 0.f) M2 -= pr;
          }
#pragma unroll
          for (int o = 4; o >= 1; o >>= 1) {
            P2 += __shfl_xor_sync(0xffffffffu, P2, o);
            M2 += __shfl_xor_sync(0xffffffffu, M2, o);
          }
#pragma unroll
          for (uint32_t j = 0; j < 4u; ++j)
            *reinterpret_cast<float4*>(st + r * HD + 4u * c8 + 32u * j) =
                make_float4(s[4u * j], s[4u * j + 1u], s[4u * j + 2u], s[4u * j + 3u]);
          if (c8 == 0u) p.out[static_cast<size_t>(z) * S + h * HD + r] = P2 - M2;
        }
      }
    } else {
      __syncthreads();  // pairs with the running units' barrier above (uniform per unit)
    }
    __syncthreads();  // every read of the stage, of the input row, of qn / kn / vv and of red is done
    if (gdn_abort) break;
    if (tid == 0) {
      if (u + kGdnStages < u1) {
        mbar_expect_tx(&full[stage], kGdnStateFloats * 4u);
        bulk_g2s(gst + stage * kGdnStateFloats, state_of(u + kGdnStages), kGdnStateFloats * 4u, &full[stage]);
        ++issued;
      }
      if (u + kGdnXSlots < u1) {
        issue_x(u + kGdnXSlots);
        ++xissued;
      }
    }
    if (u + 1u < u1) cur = nxt;
  }
  // an aborted walk leaves no copy in flight: wait (bounded) for the last copy into each stage and slot
  if (gdn_abort && tid == 0) {
    for (uint32_t s = 0; s < kGdnStages; ++s) {
      const uint32_t cnt = issued > s ? (issued - s + kGdnStages - 1u) / kGdnStages : 0u;
      if (cnt) (void)mbar_wait(&full[s], (cnt - 1u) & 1u, nullptr);
    }
    for (uint32_t s = 0; s < kGdnXSlots; ++s) {
      const uint32_t cnt = xissued > s ? (xissued - s + kGdnXSlots - 1u) / kGdnXSlots : 0u;
      if (cnt) (void)mbar_wait(&xfull[s], (cnt - 1u) & 1u, nullptr);
    }
  }
}

// Prefill capture of one position's row (see CaptureParams).  The position is
// the one this step's embed kernel advanced to; a sequence that sat the step
// out (prompt consumed) writes nothing.
__global__ void __launch_bounds__(256) capture_row_kernel(CaptureParams p) {
  __shared__ float red[9];
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t pos = p.ctrl->pos_cur, run = p.ctrl->running;
  if (!run || pos >= p.capacity) return;
  float* dst = p.dst + static_cast<size_t>(pos) * p.D;
  if (!p.norm_w) {
    for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) dst[i] = p.state[i];
    return;
  }
  float ss = 0.f;
  for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) ss += p.state[i] * p.state[i];
  const float inv = rsqrtf(block_sum256(ss, red) / static_cast<float>(p.D) + p.eps);
  for (uint32_t i = threadIdx.x; i < p.D; i += blockDim.x) dst[i] = p.state[i] * inv * p.norm_w[i];
}

// -------------------------------------------------- chunked recurrent layer
// Pre-pass, CTA (head h, row r): ops 18 (gates from the RMS-normed row), 19
// (4-tap causal convolution + SiLU of the head's q, k and v channels; the taps
// before row r are rows r-3..r-1 of the chunk or, for the first rows, the conv
// history of the chunk's first position) and 20 (L2 norms).
__global__ void __launch_bounds__(256) gdn_chunk_pre_kernel(GdnChunkParams cp) {
  const GdnParams& p = cp.g;
  __shared__ float red1[8], red2[16], red3[16];
  const uint32_t h = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const uint32_t HD = 128u, S = p.H * HD, K = p.KH * HD, kh = h % p.KH;
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t pos0 = cp.rowctl[0];
  if (!cp.rowctl[2u * r + 1u]) return;  // past the prompt
  const float* x = p.x + static_cast<size_t>(r) * p.D;
  const size_t buf = static_cast<size_t>(3u) * S * 3u;
  const float* hist = p.conv_state + (pos0 & 1u) * buf;  // taps before the chunk's first position
  // ---- op 18
  float ss[1] = {0.f};
  for (uint32_t c = tid; c < p.D; c += 256u) ss[0] += x[c] * x[c];
  block_sums<1>(ss, red1);
  const float inv = rsqrtf(ss[0] / static_cast<float>(p.D) + p.eps);
  float ab[2] = {0.f, 0.f};
  for (uint32_t c = tid; c < p.D; c += 256u) {
    const float xn = x[c] * inv * p.attn_norm[c];
    ab[0] += xn * p.wa[static_cast<size_t>(h) * p.D + c];
    ab[1] += xn * p.wb[static_cast<size_t>(h) * p.D + c];
  }
  block_sums<2>(ab, red2);
  if (tid == 0) {
    cp.gates[(static_cast<size_t>(r) * p.H + h) * 2u] = expf(-expf(p.a_log[h]) * softplus(ab[0] + p.dt_bias[h]));
    cp.gates[(static_cast<size_t>(r) * p.H + h) * 2u + 1u] = detector_sigmoid(ab[1]);
  }
  // ---- op 19: this thread's q (tid < 128) or k channel, and (tid < 128) a v channel
  auto raw_of = [&](uint32_t row, uint32_t coord) {  // raw projection of a conv channel at chunk row `row`
    const float* pr = p.proj + static_cast<size_t>(row) * p.proj_seq;
    return coord < S ? pr[kh * HD + (coord - h * HD)]
         : coord < 2u * S ? pr[K + kh * HD + (coord - S - h * HD)]
                          : pr[2u * K + (coord - 2u * S)];
  };
  auto conv_at = [&](uint32_t coord) {
    const float4 w = *reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(coord) * 4u);
    float t[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {  // taps t[j] = position (first row of this row) - 3 + j
      const int at = static_cast<int>(r) - 3 + j;
      t[j] = at >= 0 ? raw_of(static_cast<uint32_t>(at), coord) : hist[coord * 3u + static_cast<uint32_t>(3 + at)];
    }
    float signal = 0.f;
    signal = signal + t[0] * w.x;
    signal = signal + t[1] * w.y;
    signal = signal + t[2] * w.z;
    signal = signal + raw_of(r, coord) * w.w;
    return signal * detector_sigmoid(signal);
  };
  const uint32_t qk_coord = tid < 128u ? h * HD + tid : S + h * HD + (tid - 128u);
  const float f = conv_at(qk_coord);
  float vcv = 0.f;
  if (tid < 128u) vcv = conv_at(2u * S + h * HD + tid);
  // ---- op 20
  float qk2[2] = {tid < 128u ? f * f : 0.f, tid >= 128u ? f * f : 0.f};
  block_sums<2>(qk2, red3);
  float* qk = cp.qk + (static_cast<size_t>(r) * p.H + h) * 2u * HD;
  if (tid < 128u) {
    qk[tid] = (f * rsqrtf(qk2[0] + p.eps)) / sqrtf(128.0f);
    cp.vc[(static_cast<size_t>(r) * p.H + h) * HD + tid] = vcv;
  } else {
    qk[HD + (tid - 128u)] = f * rsqrtf(qk2[1] + p.eps);
  }
}

// Scan, CTA (head h, 16 value rows): op 21 row after row, the state rows in
// registers (lane owns keys 2l, 2l+1, 2l+64, 2l+65 as in the decode kernel);
// no block-wide barrier inside the walk, the next row's q / k are loaded while
// the current one is applied.
__global__ void __launch_bounds__(256) gdn_chunk_scan_kernel(GdnChunkParams cp) {
  const GdnParams& p = cp.g;
  constexpr uint32_t kRows = kGdnRowsSmall, kPerWarp = kRows / 8u;
  const uint32_t h = blockIdx.x, slice = blockIdx.y, tid = threadIdx.x;
  const uint32_t HD = 128u, S = p.H * HD, warp = tid >> 5, lane = tid & 31u;
  float* st = p.rec + static_cast<size_t>(h) * HD * HD;
  float2 s0[kPerWarp], s1[kPerWarp];
#pragma unroll
  for (uint32_t i = 0; i < kPerWarp; ++i) {
    const float* row = st + static_cast<size_t>(slice * kRows + warp * kPerWarp + i) * HD;
    s0[i] = *reinterpret_cast<const float2*>(row + 2 * lane);
    s1[i] = *reinterpret_cast<const float2*>(row + 2 * lane + 64);
  }
  pdl_wait();
  pdl_launch_dependents();
  uint32_t nlive = 0;
  for (uint32_t i = 0; i < cp.C; ++i) nlive += cp.rowctl[2u * i + 1u];
  auto load_row = [&](uint32_t r, float4& q, float4& k, float2& g, float (&v)[kPerWarp]) {
    const float* qk = cp.qk + (static_cast<size_t>(r) * p.H + h) * 2u * HD;
    const float2 qa = *reinterpret_cast<const float2*>(qk + 2 * lane), qb = *reinterpret_cast<const float2*>(qk + 2 * lane + 64);
    const float2 ka = *reinterpret_cast<const float2*>(qk + HD + 2 * lane),
                 kb = *reinterpret_cast<const float2*>(qk + HD + 2 * lane + 64);
    q = make_float4(qa.x, qa.y, qb.x, qb.y);
    k = make_float4(ka.x, ka.y, kb.x, kb.y);
    g = *reinterpret_cast<const float2*>(cp.gates + (static_cast<size_t>(r) * p.H + h) * 2u);
#pragma unroll
    for (uint32_t i = 0; i < kPerWarp; ++i)
      v[i] = cp.vc[(static_cast<size_t>(r) * p.H + h) * HD + slice * kRows + warp * kPerWarp + i];
  };
  float4 q, k, qn, kn;
  float2 g, gn;
  float v[kPerWarp], vn[kPerWarp];
  if (nlive) load_row(0, q, k, g, v);
  for (uint32_t r = 0; r < nlive; ++r) {
    if (r + 1u < nlive) load_row(r + 1u, qn, kn, gn, vn);  // in flight while row r is applied
    const float decay = g.x, beta = g.y;
#pragma unroll
    for (uint32_t i = 0; i < kPerWarp; ++i) {
      float2 a = s0[i], b = s1[i];
      a.x *= decay;
      a.y *= decay;
      b.x *= decay;
      b.y *= decay;
      const float received = signed_product_sum(k.x, k.y, k.z, k.w, a.x, a.y, b.x, b.y);
      const float delta = (v[i] - received) * beta;
      a.x += k.x * delta;
      a.y += k.y * delta;
      b.x += k.z * delta;
      b.y += k.w * delta;
      const float o = signed_product_sum(q.x, q.y, q.z, q.w, a.x, a.y, b.x, b.y);
      s0[i] = a;
      s1[i] = b;
      if (lane == 0)
        p.out[static_cast<size_t>(r) * S + h * HD + slice * kRows + warp * kPerWarp + i] = o;
    }
    q = qn, k = kn, g = gn;
#pragma unroll
    for (uint32_t i = 0; i < kPerWarp; ++i) v[i] = vn[i];
  }
#pragma unroll
  for (uint32_t i = 0; i < kPerWarp; ++i) {
    float* row = st + static_cast<size_t>(slice * kRows + warp * kPerWarp + i) * HD;
    *reinterpret_cast<float2*>(row + 2 * lane) = s0[i];
    *reinterpret_cast<float2*>(row + 2 * lane + 64) = s1[i];
  }
  // The conv history of the position after the chunk: the three newest raw
  // rows of head h's q, k and v channels (slice 0 of the head; each channel is
  // read and then written by one thread, so the parity buffer may be the one
  // the chunk started from).
  if (slice == 0u && nlive) {
    const uint32_t K = p.KH * HD, kh = h % p.KH, pos0 = cp.rowctl[0];
    const size_t buf = static_cast<size_t>(3u) * S * 3u;
    const float* hist = p.conv_state + (pos0 & 1u) * buf;
    float* next = p.conv_state + ((pos0 + nlive) & 1u) * buf;
    for (uint32_t c = tid; c < 3u * HD; c += 256u) {
      const uint32_t part = c / HD, i = c % HD, coord = part * S + h * HD + i;
      const uint32_t raw_at = part == 0u ? kh * HD + i : part == 1u ? K + kh * HD + i : 2u * K + h * HD + i;
      float t[3];
#pragma unroll
      for (int j = 0; j < 3; ++j) {  // taps = positions (last live) - 2 + j
        const int at = static_cast<int>(nlive) - 3 + j;
        t[j] = at >= 0 ? p.proj[static_cast<size_t>(at) * p.proj_seq + raw_at]
                       : hist[coord * 3u + static_cast<uint32_t>(3 + at)];
      }
#pragma unroll
      for (int j = 0; j < 3; ++j) next[coord * 3u + j] = t[j];
    }
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
  return launch_pdl(reinterpret_cast<const void*>(embed_kernel), dim3(p.nseq), dim3(256), args, s, pdl);
}
cudaError_t launch_capture_row(const CaptureParams& p, cudaStream_t s, bool pdl) {
  if (!p.state || !p.dst || !p.ctrl || p.D == 0) return cudaErrorInvalidValue;
  void* args[] = {const_cast<CaptureParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(capture_row_kernel), dim3(1), dim3(256), args, s, pdl);
}
cudaError_t launch_chunk_begin(const ChunkParams& p, cudaStream_t s, bool pdl) {
  if (!p.table || !p.ctrl || !p.prompt || !p.rowctl || !p.rows || p.C == 0) return cudaErrorInvalidValue;
  void* args[] = {const_cast<ChunkParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(chunk_begin_kernel), dim3(p.C), dim3(256), args, s, pdl);
}
cudaError_t launch_chunk_end(const ChunkParams& p, cudaStream_t s, bool pdl) {
  if (!p.ctrl || !p.rows || !p.state || p.C == 0) return cudaErrorInvalidValue;
  void* args[] = {const_cast<ChunkParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(chunk_end_kernel), dim3(1), dim3(256), args, s, pdl);
}
cudaError_t launch_attn_prep(const PrepParams& p, cudaStream_t s, bool pdl) {
  if (p.hd > 256 || (p.packets && p.hd != 256)) return cudaErrorInvalidValue;  // a packet block is 256 values
  void* args[] = {const_cast<PrepParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(attn_prep_kernel), dim3(p.heads + p.kvh, p.nseq), dim3(256), args, s,
                    pdl);
}
cudaError_t launch_gdn(const GdnParams& p, cudaStream_t s, bool pdl) {
  if (p.D == 0 || p.D > 256u * kGdnDPer) return cudaErrorInvalidValue;
  void* args[] = {const_cast<GdnParams*>(&p)};
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // From 64 (head, sequence) units on, one persistent CTA per SM walks them: the
  // 16-row CTAs re-read the gate rows, the norm weight and the hidden row in all
  // eight slices of a head (64 KB each at the 9B shape: 134 MB of L2 reads per
  // layer at 8 sequences), and below one unit per SM the empty CTAs just leave.
  if (p.H * p.nseq >= kGdnPersistentUnits) {
    // bulk copies of whole states: 16-byte aligned, and each state row block contiguous
    if ((reinterpret_cast<uintptr_t>(p.rec) % 16u) || (p.rec_seq * 4u) % 16u || (reinterpret_cast<uintptr_t>(p.conv_w) % 16u))
      return cudaErrorMisalignedAddress;
    if (p.D % 4u || reinterpret_cast<uintptr_t>(p.x) % 16u) return cudaErrorMisalignedAddress;  // input rows by bulk copy
    const uint32_t smem = (kGdnStages * kGdnStateFloats + kGdnXSlots * p.D) * 4u;
    static std::atomic<int> attr_dev[64];
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_dev[dev].load()) {
      // the largest stage set (hidden size 256 * kGdnDPer), whatever model opens first
      const cudaError_t e = cudaFuncSetAttribute(
          gdn_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
          static_cast<int>((kGdnStages * kGdnStateFloats + kGdnXSlots * 256u * kGdnDPer) * 4u));
      if (e != cudaSuccess) return e;
      attr_dev[dev].store(1);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<uint32_t>(sms));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(gdn_batch_kernel), args);
  }
  return launch_pdl(reinterpret_cast<const void*>(gdn_kernel),
                    dim3(p.H, 128u / kGdnRowsSmall, p.nseq), dim3(256), args, s, pdl);
}
cudaError_t launch_gdn_chunk(const GdnChunkParams& p, cudaStream_t s, bool pdl) {
  if (p.g.D == 0 || p.g.D > 256u * kGdnDPer || p.C == 0 || !p.rowctl || !p.gates || !p.qk || !p.vc)
    return cudaErrorInvalidValue;
  void* args[] = {const_cast<GdnChunkParams*>(&p)};
  cudaError_t e = launch_pdl(reinterpret_cast<const void*>(gdn_chunk_pre_kernel), dim3(p.g.H, p.C), dim3(256), args,
                             s, pdl);
  if (e != cudaSuccess) return e;
  return launch_pdl(reinterpret_cast<const void*>(gdn_chunk_scan_kernel), dim3(p.g.H, 128u / kGdnRowsSmall),
                    dim3(256), args, s, true);
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
