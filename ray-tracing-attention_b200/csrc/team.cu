// team.cu -- peer exchange between the GPUs of one box for the tensor-parallel
// MLP and vocabulary readout (one process per GPU).
//
// The reference runs one worker on one GPU and has no collective at all; the
// split it would need is the textbook one: the MLP's gate / up rows and the
// down projection's columns are divided between the ranks, each rank forms a
// partial [batch x hidden] product, and the partials are summed on every rank;
// the vocabulary rows are divided, each rank finds its best row, and the ranks
// agree on the best of the bests.  Both exchanges are small (8 KB per layer at
// batch 1, 1 MiB at batch 64 x 4096), so they are latency-bound: this file does
// them in ONE kernel launch each, over NVLink peer memory, instead of a library
// collective.
//
// Exchange allocation of one rank (cudaMalloc, shared with the other ranks
// through CUDA IPC handles that the caller passes around on the host):
//   flags  [kMaxRanks source][kMaxBlocks] u32     call counters, written by the source
//   slots  [2 parity][world source][cap words]     partial contributions
// A call made by block b of every rank with counter value e:
//   1. copies this rank's chunk b into slot [e & 1][rank] of every rank
//      (plain stores into peer memory over NVLink, 16 B each);
//   2. publishes e in flag [rank][b] of every rank (release at system scope);
//   3. waits, bounded by RTA_WAIT_NS, until flag [s][b] >= e for every source s;
//   4. reduces the world slots of chunk b in rank order 0, 1, ... (so every
//      rank computes the same bits) and writes the result.
// Slots alternate by parity: a rank can be at most one call ahead of another
// (it needs the other's flag of the current call to finish it), and the other
// has finished reading the previous call's parity before it publishes the
// current call's flag, so a slot is never overwritten while it is read.
// A rank whose peer never arrives records RTA_DEVERR_TIMEOUT in the team's
// error word and returns; rta_team_error() reports it.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "../../include/rta.h"
#include "rta_device.cuh"
#include "rta_internal.h"

namespace {
constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kMaxBlocks = 256;   // exchange blocks of one call
constexpr uint32_t kChunkWords = 2048; // 8 KB of one rank's contribution per block
constexpr uint32_t kThreads = 512;
constexpr size_t kFlagBytes = size_t(kMaxRanks) * kMaxBlocks * 4u;
constexpr size_t kMetaBytes = kMaxRanks * sizeof(void*) + (kMaxBlocks + 1u) * 4u;

struct View {
  uint8_t* const* base;      // [world] every rank's exchange allocation as this GPU addresses it
  uint32_t* ctr;             // this rank's per-block call counters [kMaxBlocks]
  uint32_t* err;             // this rank's error word
  uint32_t rank, world;
  uint32_t cap_words;        // 32-bit words per (parity, source) slot
};

__device__ __forceinline__ uint32_t* flag_at(const View& v, uint32_t owner, uint32_t src, uint32_t b) {
  return reinterpret_cast<uint32_t*>(v.base[owner]) + src * kMaxBlocks + b;
}
__device__ __forceinline__ uint32_t* slot_at(const View& v, uint32_t owner, uint32_t parity, uint32_t src) {
  return reinterpret_cast<uint32_t*>(v.base[owner] + kFlagBytes) +
         (size_t(parity) * v.world + src) * v.cap_words;
}

// Counter value of this call for block b (every rank makes the same calls).
__device__ __forceinline__ uint32_t begin_call(const View& v, uint32_t b) {
  __shared__ uint32_t e;
  if (threadIdx.x == 0) e = v.ctr[b] + 1u;
  __syncthreads();
  return e;
}

// After this block's stores to every rank's slot: publish counter e.
__device__ __forceinline__ void publish(const View& v, uint32_t b, uint32_t e) {
  __syncthreads();
  if (threadIdx.x < v.world) {
    uint32_t* f = flag_at(v, threadIdx.x, v.rank, b);
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
  }
}

// Bounded wait for counter e from every source; false after a timeout.
__device__ __forceinline__ bool await_all(const View& v, uint32_t b, uint32_t e) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if (threadIdx.x < v.world) {
    const uint32_t* f = flag_at(v, v.rank, threadIdx.x, b);
    const uint64_t start = rta::globaltimer();
    for (uint32_t spin = 0;; ++spin) {
      uint32_t x;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(x) : "l"(f) : "memory");
      if (static_cast<int32_t>(x - e) >= 0) break;
      if ((spin & 15u) == 15u && rta::globaltimer() - start > RTA_WAIT_NS) {
        atomicOr(v.err, RTA_DEVERR_TIMEOUT);
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ void end_call(const View& v, uint32_t b, uint32_t e) {
  if (threadIdx.x == 0) v.ctr[b] = e;
}

// Rows of sequences that sat a step out (a ragged prefill's consumed prompts,
// stopped generations): their products wrote nothing this step, so whatever
// their rows of the exchanged buffer hold is not added.  running == null: every
// row takes part.  Every rank holds the same flags, so every rank skips alike.
struct RowMask {
  const uint32_t* running;
  uint32_t step, width;  // u32 between the sequences' flags; floats per row
  __device__ __forceinline__ bool live(uint32_t float4_index) const {
    return !running || running[static_cast<size_t>(4u * float4_index / width) * step] != 0u;
  }
};

// out[i] = addend[i] + sum over ranks s (in order) of partial_s[i]; n % 4 == 0.
__global__ void __launch_bounds__(kThreads) allreduce_kernel(View v, const float* __restrict__ partial,
                                                             const float* addend, float* out, uint32_t n, RowMask rows) {
  const uint32_t b = blockIdx.x;
  const uint32_t e = begin_call(v, b);
  const uint32_t par = e & 1u;
  const uint32_t q0 = b * (kChunkWords / 4u), q1 = min(n / 4u, q0 + kChunkWords / 4u);
  for (uint32_t i = q0 + threadIdx.x; i < q1; i += blockDim.x) {
    const float4 val = reinterpret_cast<const float4*>(partial)[i];
    for (uint32_t p = 0; p < v.world; ++p) reinterpret_cast<float4*>(slot_at(v, p, par, v.rank))[i] = val;
  }
  publish(v, b, e);
  if (await_all(v, b, e)) {
    for (uint32_t i = q0 + threadIdx.x; i < q1; i += blockDim.x) {
      float4 acc = addend ? reinterpret_cast<const float4*>(addend)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (rows.live(i))
        for (uint32_t s = 0; s < v.world; ++s) {
          const float4 c = __ldcg(reinterpret_cast<const float4*>(slot_at(v, v.rank, par, s)) + i);
          acc.x += c.x;
          acc.y += c.y;
          acc.z += c.z;
          acc.w += c.w;
        }
      reinterpret_cast<float4*>(out)[i] = acc;
    }
  }
  end_call(v, b, e);
}

// Best (value, lowest id) over the ranks' local argmax results; ids of rank r
// are offset by id_base, the first vocabulary row this rank holds.
__global__ void __launch_bounds__(kThreads) argmax_kernel(View v, const uint32_t* ids, const float* best,
                                                          uint32_t id_base, uint32_t batch, uint32_t* out_ids,
                                                          float* out_best) {
  const uint32_t e = begin_call(v, 0);
  const uint32_t par = e & 1u;
  for (uint32_t i = threadIdx.x; i < batch; i += blockDim.x) {
    const uint32_t id = ids[i];
    const unsigned long long key = id == 0xffffffffu ? 0ull : rta::pack_argmax(best[i], id + id_base);
    for (uint32_t p = 0; p < v.world; ++p) reinterpret_cast<unsigned long long*>(slot_at(v, p, par, v.rank))[i] = key;
  }
  publish(v, 0, e);
  if (await_all(v, 0, e)) {
    for (uint32_t i = threadIdx.x; i < batch; i += blockDim.x) {
      unsigned long long k = 0ull;
      for (uint32_t s = 0; s < v.world; ++s)
        k = max(k, __ldcg(reinterpret_cast<const unsigned long long*>(slot_at(v, v.rank, par, s)) + i));
      if (k == 0ull) {
        atomicOr(v.err, RTA_DEVERR_TOKEN);
        out_ids[i] = 0xffffffffu;
        if (out_best) out_best[i] = -INFINITY;
      } else {
        out_ids[i] = ~static_cast<uint32_t>(k & 0xffffffffull);
        if (out_best) out_best[i] = rta::float_from_order_key(static_cast<uint32_t>(k >> 32));
      }
    }
  }
  end_call(v, 0, e);
}

// state[i] += delta_s[i] for the rows of every source s: each rank owns the
// rows [row_start[rank], row_start[rank + 1]) of a [rows][width] float matrix
// and contributes only those (its attention / recurrent block outputs); the
// rows of different ranks are disjoint, so every element of state receives
// exactly one addend and every rank ends with the same bits.  Block b handles
// chunk b of every source's rows.  Pushes 1/world of the one-shot allreduce's
// bytes.
__global__ void __launch_bounds__(kThreads) gather_add_kernel(View v, const float* __restrict__ delta, float* state,
                                                              uint32_t width, uint32_t start0, uint32_t start1,
                                                              uint32_t start2, uint32_t start3, uint32_t start4,
                                                              uint32_t start5, uint32_t start6, uint32_t start7,
                                                              uint32_t start8, RowMask rows) {
  const uint32_t starts[kMaxRanks + 1] = {start0, start1, start2, start3, start4, start5, start6, start7, start8};
  const uint32_t b = blockIdx.x, nb = gridDim.x;
  const uint32_t e = begin_call(v, b);
  const uint32_t par = e & 1u;
  auto chunk = [&](uint32_t s, uint32_t& q0, uint32_t& q1) {  // float4 range of source s handled by block b
    const uint32_t lo = starts[s] * width / 4u, hi = starts[s + 1] * width / 4u, n = hi - lo;
    q0 = lo + static_cast<uint32_t>(static_cast<uint64_t>(n) * b / nb);
    q1 = lo + static_cast<uint32_t>(static_cast<uint64_t>(n) * (b + 1) / nb);
  };
  uint32_t q0, q1;
  chunk(v.rank, q0, q1);
  for (uint32_t i = q0 + threadIdx.x; i < q1; i += blockDim.x) {
    const float4 val = reinterpret_cast<const float4*>(delta)[i];
    for (uint32_t p = 0; p < v.world; ++p) reinterpret_cast<float4*>(slot_at(v, p, par, v.rank))[i] = val;
  }
  publish(v, b, e);
  if (await_all(v, b, e)) {
    for (uint32_t s = 0; s < v.world; ++s) {
      chunk(s, q0, q1);
      for (uint32_t i = q0 + threadIdx.x; i < q1; i += blockDim.x) {
        if (!rows.live(i)) continue;
        float4 acc = reinterpret_cast<const float4*>(state)[i];
        const float4 c = __ldcg(reinterpret_cast<const float4*>(slot_at(v, v.rank, par, s)) + i);
        acc.x += c.x;
        acc.y += c.y;
        acc.z += c.z;
        acc.w += c.w;
        reinterpret_cast<float4*>(state)[i] = acc;
      }
    }
  }
  end_call(v, b, e);
}

// out = addend + sum over ranks of partial, in two phases of one launch (a
// reduce-scatter, then an all-gather): rank o owns chunk o of the n floats;
// phase 1 pushes every other rank's chunk of this rank's partial to that rank
// only, the owner sums its chunk in rank order (plus the addend) and phase 2
// pushes the sum to every rank.  Each rank sends 2 (world - 1) / world of its
// contribution instead of world - 1 copies of all of it (the one-shot
// allreduce_kernel), for one more flag round trip.  Block b handles part b of
// every chunk.  Counters: phase 1 publishes e, phase 2 e + 1 (the other slot
// parity); the call leaves the counter at e + 1.
__global__ void __launch_bounds__(kThreads) allreduce2_kernel(View v, const float* __restrict__ partial,
                                                              const float* addend, float* out, uint32_t n,
                                                              RowMask rows) {
  const uint32_t b = blockIdx.x, nb = gridDim.x;
  __shared__ uint32_t e_s;
  if (threadIdx.x == 0) e_s = v.ctr[b] + 1u;
  __syncthreads();
  const uint32_t e1 = e_s, e2 = e1 + 1u;
  const uint32_t q4 = n / 4u;  // float4 elements
  auto part = [&](uint32_t o, uint32_t& lo, uint32_t& hi) {  // float4 range of chunk o handled by block b
    const uint32_t c0 = static_cast<uint32_t>(static_cast<uint64_t>(q4) * o / v.world);
    const uint32_t c1 = static_cast<uint32_t>(static_cast<uint64_t>(q4) * (o + 1u) / v.world);
    lo = c0 + static_cast<uint32_t>(static_cast<uint64_t>(c1 - c0) * b / nb);
    hi = c0 + static_cast<uint32_t>(static_cast<uint64_t>(c1 - c0) * (b + 1u) / nb);
  };
  uint32_t lo, hi;
  // phase 1: chunk o of this rank's partial -> slot [e1 & 1][rank] of rank o
  for (uint32_t o = 0; o < v.world; ++o) {
    part(o, lo, hi);
    float4* dst = reinterpret_cast<float4*>(slot_at(v, o, e1 & 1u, v.rank));
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = reinterpret_cast<const float4*>(partial)[i];
  }
  publish(v, b, e1);
  bool ok = await_all(v, b, e1);
  // the owner's sum of its chunk, in rank order, to every rank (slot [e2 & 1][rank])
  part(v.rank, lo, hi);
  if (ok)
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      float4 acc = addend ? reinterpret_cast<const float4*>(addend)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (rows.live(i))
        for (uint32_t s = 0; s < v.world; ++s) {
          const float4 c = __ldcg(reinterpret_cast<const float4*>(slot_at(v, v.rank, e1 & 1u, s)) + i);
          acc.x += c.x;
          acc.y += c.y;
          acc.z += c.z;
          acc.w += c.w;
        }
      reinterpret_cast<float4*>(out)[i] = acc;
      for (uint32_t pr = 0; pr < v.world; ++pr)
        if (pr != v.rank) reinterpret_cast<float4*>(slot_at(v, pr, e2 & 1u, v.rank))[i] = acc;
    }
  publish(v, b, e2);
  ok = await_all(v, b, e2) && ok;
  if (ok)
    for (uint32_t o = 0; o < v.world; ++o) {
      if (o == v.rank) continue;
      part(o, lo, hi);
      for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x)
        reinterpret_cast<float4*>(out)[i] = __ldcg(reinterpret_cast<const float4*>(slot_at(v, v.rank, e2 & 1u, o)) + i);
    }
  end_call(v, b, e2);
}

// In place over n packed argmax keys (order key << 32 | ~id, 0 = none) spaced
// `stride` u64 apart: this rank's keys carry ids local to its vocabulary rows
// starting at id_base; afterwards every rank holds the largest key over the
// ranks with global ids (ties -> lowest id, as ops 16/17 of resident_math.comp).
__global__ void __launch_bounds__(kThreads) allmax_keys_kernel(View v, unsigned long long* keys, uint32_t n,
                                                               uint32_t stride, uint32_t id_base) {
  const uint32_t b = blockIdx.x;
  const uint32_t e = begin_call(v, b);
  const uint32_t par = e & 1u;
  if (b != 0u) n = 0u;  // the other blocks only keep the per-block call counters in step
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    unsigned long long k = keys[static_cast<size_t>(i) * stride];
    if (k != 0ull) {
      const uint32_t low = static_cast<uint32_t>(k & 0xffffffffull) - id_base;  // ~(id + base) = ~id - base
      k = (k & 0xffffffff00000000ull) | low;
    }
    for (uint32_t p = 0; p < v.world; ++p) reinterpret_cast<unsigned long long*>(slot_at(v, p, par, v.rank))[i] = k;
  }
  publish(v, b, e);
  if (await_all(v, b, e)) {
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
      unsigned long long k = 0ull;
      for (uint32_t s = 0; s < v.world; ++s)
        k = max(k, __ldcg(reinterpret_cast<const unsigned long long*>(slot_at(v, v.rank, par, s)) + i));
      keys[static_cast<size_t>(i) * stride] = k;
    }
  }
  end_call(v, b, e);
}

rta_status team_fail(rta_status code, const std::string& msg) {
  rta::set_last_error(msg);
  return code;
}
rta_status team_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return RTA_OK;
  return team_fail(RTA_E_CUDA, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}
}  // namespace

struct rta_team {
  int device = 0;
  uint32_t rank = 0, world = 1;
  size_t cap_words = 0;
  uint8_t* local = nullptr;                  // this rank's exchange allocation
  uint8_t* peer[kMaxRanks] = {};             // every rank's allocation as mapped here
  uint8_t** meta = nullptr;                  // device: [kMaxRanks] peer bases, [kMaxBlocks] counters, error word
  uint32_t* ctr = nullptr;                   // counters inside meta
  bool connected = false;

  View view() const {
    View v{};
    v.base = meta;
    v.ctr = ctr;
    v.err = ctr + kMaxBlocks;
    v.rank = rank;
    v.world = world;
    v.cap_words = static_cast<uint32_t>(cap_words);
    return v;
  }
};

// Internal entry points of the decode engine's tensor-parallel mode.
namespace rta {
uint32_t team_rank(const rta_team* t) { return t->rank; }
uint32_t team_world(const rta_team* t) { return t->world; }
bool team_ready(const rta_team* t) { return t->connected; }
size_t team_capacity_words(const rta_team* t) { return t->cap_words; }
// The engine launches every exchange of a handle with the same block count
// (team_blocks), so the per-block call counters -- and with them the slot
// parity of a call -- advance in step across exchange kinds whose chunks of
// the slots differ.
uint32_t team_blocks(size_t words) {
  const size_t b = (words + kChunkWords - 1u) / kChunkWords;
  return b < 1u ? 1u : b > kMaxBlocks ? kMaxBlocks : static_cast<uint32_t>(b);
}
cudaError_t team_allreduce(rta_team* t, const float* partial, const float* addend, float* out, size_t n,
                           uint32_t blocks, cudaStream_t s, const uint32_t* running, uint32_t run_step,
                           uint32_t width) {
  if (!t->connected || n == 0 || n % 4u || n > t->cap_words || blocks > kMaxBlocks ||
      static_cast<size_t>(blocks) * kChunkWords < n)
    return cudaErrorInvalidValue;
  if (running && (width == 0 || width % 4u)) return cudaErrorInvalidValue;
  allreduce_kernel<<<blocks, kThreads, 0, s>>>(t->view(), partial, addend, out, static_cast<uint32_t>(n),
                                               RowMask{running, run_step, width});
  return cudaGetLastError();
}
cudaError_t team_allreduce2(rta_team* t, const float* partial, const float* addend, float* out, size_t n,
                            uint32_t blocks, cudaStream_t s, const uint32_t* running, uint32_t run_step,
                            uint32_t width) {
  if (!t->connected || n == 0 || n % 4u || n > t->cap_words || blocks == 0 || blocks > kMaxBlocks)
    return cudaErrorInvalidValue;
  if (running && (width == 0 || width % 4u)) return cudaErrorInvalidValue;
  allreduce2_kernel<<<blocks, kThreads, 0, s>>>(t->view(), partial, addend, out, static_cast<uint32_t>(n),
                                                RowMask{running, run_step, width});
  return cudaGetLastError();
}
cudaError_t team_gather_add(rta_team* t, const float* delta, float* state, uint32_t width,
                            const uint32_t* row_start, uint32_t blocks, cudaStream_t s, const uint32_t* running,
                            uint32_t run_step) {
  if (!t->connected || width % 4u || static_cast<size_t>(row_start[t->world]) * width > t->cap_words ||
      blocks == 0 || blocks > kMaxBlocks)
    return cudaErrorInvalidValue;
  uint32_t st[kMaxRanks + 1];
  for (uint32_t i = 0; i <= kMaxRanks; ++i) st[i] = row_start[i < t->world ? i : t->world];
  gather_add_kernel<<<blocks, kThreads, 0, s>>>(t->view(), delta, state, width, st[0], st[1], st[2], st[3], st[4],
                                                st[5], st[6], st[7], st[8], RowMask{running, run_step, width});
  return cudaGetLastError();
}
cudaError_t team_allmax_keys(rta_team* t, unsigned long long* keys, uint32_t n, uint32_t stride, uint32_t id_base,
                             uint32_t blocks, cudaStream_t s) {
  if (!t->connected || n == 0 || n > kChunkWords / 2u || 2ull * n > t->cap_words || blocks == 0 ||
      blocks > kMaxBlocks)
    return cudaErrorInvalidValue;
  allmax_keys_kernel<<<blocks, kThreads, 0, s>>>(t->view(), keys, n, stride, id_base);
  return cudaGetLastError();
}
uint32_t* team_error_word(rta_team* t) { return t->ctr + kMaxBlocks; }
}  // namespace rta

extern "C" {

size_t rta_team_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

rta_status rta_team_create(uint32_t rank, uint32_t world, size_t capacity_bytes, rta_team** team, void* handle) {
  if (!team || world == 0 || world > kMaxRanks || rank >= world || capacity_bytes == 0 ||
      capacity_bytes > size_t(kMaxBlocks) * kChunkWords * 4u || (world > 1 && !handle))
    return team_fail(RTA_E_ARG, "rta_team_create: 1 <= world <= 8, rank < world, 0 < capacity <= 2 MiB, handle");
  *team = nullptr;
  auto* t = new rta_team();
  t->rank = rank;
  t->world = world;
  t->cap_words = (capacity_bytes + 15u) / 16u * 4u;
  rta_status st = team_cuda(cudaGetDevice(&t->device), "rta_team_create(device)");
  const size_t bytes = kFlagBytes + 2u * world * t->cap_words * 4u;
  if (st == RTA_OK) st = team_cuda(cudaMalloc(&t->local, bytes), "rta_team_create(exchange)");
  if (st == RTA_OK) st = team_cuda(cudaMalloc(&t->meta, kMetaBytes), "rta_team_create(counters)");
  if (st == RTA_OK) st = team_cuda(cudaMemset(t->local, 0, bytes), "rta_team_create(memset)");
  if (st == RTA_OK) st = team_cuda(cudaMemset(t->meta, 0, kMetaBytes), "rta_team_create(memset)");
  if (st == RTA_OK) {
    t->ctr = reinterpret_cast<uint32_t*>(t->meta + kMaxRanks);
    st = team_cuda(cudaMemcpy(t->meta + rank, &t->local, sizeof(void*), cudaMemcpyHostToDevice), "rta_team_create");
  }
  if (st == RTA_OK) st = team_cuda(cudaDeviceSynchronize(), "rta_team_create(sync)");
  if (st == RTA_OK && world > 1)
    st = team_cuda(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), t->local), "rta_team_create(ipc)");
  if (st != RTA_OK) {
    rta_team_destroy(t);
    return st;
  }
  t->peer[rank] = t->local;
  t->connected = world == 1;
  *team = t;
  return RTA_OK;
}

rta_status rta_team_connect(rta_team* t, const void* handles) {
  if (!t || (t->world > 1 && !handles)) return team_fail(RTA_E_ARG, "rta_team_connect: bad arguments");
  if (t->connected) return RTA_OK;
  int dev = 0;
  rta_status st = team_cuda(cudaGetDevice(&dev), "rta_team_connect(device)");
  if (st == RTA_OK && dev != t->device) return team_fail(RTA_E_STATE, "rta_team_connect: wrong current device");
  const auto* h = static_cast<const cudaIpcMemHandle_t*>(handles);
  for (uint32_t p = 0; p < t->world && st == RTA_OK; ++p) {
    if (p == t->rank) continue;
    void* ptr = nullptr;
    st = team_cuda(cudaIpcOpenMemHandle(&ptr, h[p], cudaIpcMemLazyEnablePeerAccess), "rta_team_connect(open)");
    if (st == RTA_OK) t->peer[p] = static_cast<uint8_t*>(ptr);
  }
  if (st == RTA_OK)
    st = team_cuda(cudaMemcpy(t->meta, t->peer, t->world * sizeof(void*), cudaMemcpyHostToDevice), "rta_team_connect");
  if (st != RTA_OK) {
    rta_team_disconnect(t);
    return st;
  }
  t->connected = true;
  return RTA_OK;
}

rta_status rta_team_allreduce_f32(rta_team* t, const float* partial, const float* addend, float* out, size_t n,
                                  void* stream) {
  if (!t || !partial || !out || n == 0 || n % 4u || n > t->cap_words ||
      (reinterpret_cast<uintptr_t>(partial) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(addend)) % 16u)
    return team_fail(RTA_E_ARG, "rta_team_allreduce_f32: n % 4 == 0, n <= capacity / 4, 16-byte aligned buffers");
  if (!t->connected) return team_fail(RTA_E_STATE, "rta_team_allreduce_f32: team not connected");
  const uint32_t blocks = static_cast<uint32_t>((n + kChunkWords - 1u) / kChunkWords);
  allreduce_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(t->view(), partial, addend, out,
                                                                               static_cast<uint32_t>(n),
                                                                               RowMask{nullptr, 0u, 0u});
  return team_cuda(cudaGetLastError(), "rta_team_allreduce_f32");
}

rta_status rta_team_argmax(rta_team* t, const uint32_t* ids, const float* best, uint32_t id_base, uint32_t batch,
                           uint32_t* argmax, float* best_out, void* stream) {
  if (!t || !ids || !best || !argmax || batch == 0 || 2u * size_t(batch) > t->cap_words || batch > kChunkWords / 2u)
    return team_fail(RTA_E_ARG, "rta_team_argmax: 1 <= batch <= min(1024, capacity / 8)");
  if (!t->connected) return team_fail(RTA_E_STATE, "rta_team_argmax: team not connected");
  argmax_kernel<<<1, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(t->view(), ids, best, id_base, batch, argmax,
                                                                       best_out);
  return team_cuda(cudaGetLastError(), "rta_team_argmax");
}

rta_status rta_team_error(rta_team* t, void* stream, uint32_t* word) {
  if (!t || !word) return team_fail(RTA_E_ARG, "rta_team_error: bad arguments");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rta_status st = team_cuda(cudaStreamSynchronize(s), "rta_team_error(sync)");
  if (st == RTA_OK) st = team_cuda(cudaMemcpy(word, t->ctr + kMaxBlocks, 4, cudaMemcpyDeviceToHost), "rta_team_error");
  if (st == RTA_OK && *word) st = team_cuda(cudaMemset(t->ctr + kMaxBlocks, 0, 4), "rta_team_error(clear)");
  return st;
}

rta_status rta_team_disconnect(rta_team* t) {
  if (!t) return RTA_OK;
  rta_status st = RTA_OK;
  for (uint32_t p = 0; p < t->world; ++p) {
    if (p == t->rank || !t->peer[p]) continue;
    const rta_status s = team_cuda(cudaIpcCloseMemHandle(t->peer[p]), "rta_team_disconnect");
    if (st == RTA_OK) st = s;
    t->peer[p] = nullptr;
  }
  t->connected = t->world == 1;
  return st;
}

void rta_team_destroy(rta_team* t) {
  if (!t) return;
  rta_team_disconnect(t);
  if (t->local) cudaFree(t->local);
  if (t->meta) cudaFree(t->meta);
  delete t;
}

}  // extern "C"
