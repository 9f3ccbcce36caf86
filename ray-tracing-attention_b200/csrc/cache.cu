// cache.cu -- device digests of the decode state, batched row-segment copies,
// and the host indexes of the prefix boundaries and the reply tree (cache.h).
//
// The state address follows the reference's verification key
// (ray_tracing/native/shaders/optical_path_key.comp:27-96): every live word of
// the next decode step's inputs enters an order-free 256-bit fold (lanes 0-3
// XOR, lanes 4-7 sum) under an identity of its position, history rows with the
// identity of their layer and absolute position, and the fold is finished with
// the position, the epoch and the stop ids.  The mixing function here is
// MurmurHash3's 32-bit finalizer (public domain), with four lane hashes per
// word; the reference's own mixer and lane seeds are not reproduced, since the
// key never leaves the process that computed it.
#include <algorithm>
#include <cstring>

#include "cache.h"
#include "rta_device.cuh"

namespace rta {

namespace {

__host__ __device__ __forceinline__ uint32_t fmix32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x85ebca6bu;
  x ^= x >> 13;
  x *= 0xc2b2ae35u;
  x ^= x >> 16;
  return x;
}

// odd multipliers of the word index, one per lane
__constant__ uint32_t kLaneMul[4] = {0x9E3779B1u, 0x85EBCA77u, 0xC2B2AE3Du, 0x27D4EB2Fu};
constexpr uint32_t kStateSeed = 0x6A09E667u;

struct Fold {
  uint32_t x[4], a[4];
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = a[k] = 0u;
  }
  // word v at index i of a row (or of the state) whose identity is r
  __device__ __forceinline__ void absorb(uint32_t v, uint32_t i, uint32_t r) {
    const uint32_t t = v ^ r;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t h = fmix32(t + i * kLaneMul[k]);
      x[k] ^= h;
      a[k] += h;
    }
  }
  __device__ __forceinline__ void merge(const uint32_t* w) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[k] ^= w[k];
      a[k] += w[4 + k];
    }
  }
  __device__ __forceinline__ void warp_fold() {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        x[k] ^= __shfl_xor_sync(0xffffffffu, x[k], off);
        a[k] += __shfl_xor_sync(0xffffffffu, a[k], off);
      }
  }
  // the whole CTA's fold into thread 0 (blockDim.x = 256)
  __device__ __forceinline__ void block_fold(uint32_t (*sh)[8]) {
    warp_fold();
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (lane == 0)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        sh[warp][k] = x[k];
        sh[warp][4 + k] = a[k];
      }
    __syncthreads();
    if (threadIdx.x == 0) {
      clear();
      for (uint32_t w = 0; w < blockDim.x / 32u; ++w) merge(sh[w]);
    }
  }
};

__device__ __forceinline__ uint32_t row_identity(uint32_t layer, uint32_t position) {
  return fmix32(layer * 0x9E3779B9u + 0x7F4A7C15u) ^ fmix32(position * 0x85EBCA77u + 0x165667B1u);
}

// The history positions still to digest: [lo, hi), inside the live window.
__device__ __forceinline__ void history_range(const DigestArgs& a, uint32_t& lo, uint32_t& hi) {
  hi = *a.pos_next;
  const uint32_t window = hi > a.capacity ? hi - a.capacity : 0u;
  lo = *a.cursor;
  if (lo > hi || lo < window) lo = window;
}

// 32-bit words of one history row of one layer
__host__ __device__ __forceinline__ uint32_t row_words(const DigestArgs& a) {
  return a.packets ? a.pbytes / 4u : a.kvh * a.hd;  // fp16: K then V, kvh x hd halves each
}

// (1) one warp per (position, layer, 128-word chunk of the row): the chunk's
// digest into its slot entry.  Four independent loads per lane, so a step's
// few new rows spread over many warps instead of one dependent chain each.
__global__ void __launch_bounds__(256) digest_rows_kernel(const DigestArgs a) {
  uint32_t lo, hi;
  history_range(a, lo, hi);
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t words = row_words(a), chunks = (words + kRowChunk - 1u) / kRowChunk;
  const uint32_t per_row = a.n_full * chunks, items = (hi - lo) * per_row, warps = gridDim.x * 8u;
  const uint32_t hw = a.hd / 2u, per = a.kvh * hw;  // fp16: 32-bit words of one K (or V) row
  for (uint32_t it = blockIdx.x * 8u + (threadIdx.x >> 5); it < items; it += warps) {
    const uint32_t p = lo + it / per_row, rem = it % per_row, layer = rem / chunks, c = rem % chunks;
    const uint32_t slot = p % a.capacity, r = row_identity(layer, p);
    uint32_t v[kRowChunk / 32u];
    bool in[kRowChunk / 32u];
#pragma unroll
    for (uint32_t u = 0; u < kRowChunk / 32u; ++u) {
      const uint32_t j = c * kRowChunk + u * 32u + lane;
      in[u] = j < words;
      v[u] = 0u;
      if (!in[u]) continue;
      if (a.packets) {
        v[u] = reinterpret_cast<const uint32_t*>(a.packets + (static_cast<size_t>(layer) * a.capacity + slot) *
                                                             a.pbytes)[j];
      } else {
        const uint32_t kv = j / per, jj = j % per, h = jj / hw, w = jj % hw;
        const __half* base =
            (kv ? a.vcache : a.kcache) + layer * a.layer_kv + (static_cast<size_t>(h) * a.capacity + slot) * a.hd;
        v[u] = reinterpret_cast<const uint32_t*>(base)[w];
      }
    }
    Fold f;
    f.clear();
#pragma unroll
    for (uint32_t u = 0; u < kRowChunk / 32u; ++u)
      if (in[u]) f.absorb(v[u], c * kRowChunk + u * 32u + lane, r);
    f.warp_fold();
    if (lane == 0) {
      uint32_t* out = a.slot_hash + ((static_cast<size_t>(layer) * a.capacity + slot) * chunks + c) * 8u;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        out[k] = f.x[k];
        out[4 + k] = f.a[k];
      }
    }
  }
}

// (2) the state words and the live slots' chunk digests -> one partial per
// CTA.  Each thread keeps four 16-byte loads in flight before it hashes them
// (the fold is memory-latency bound otherwise).
__global__ void __launch_bounds__(256) digest_fold_kernel(const DigestArgs a) {
  __shared__ uint32_t sh[8][8];
  Fold f;
  f.clear();
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t nth = static_cast<size_t>(gridDim.x) * blockDim.x;
  uint32_t base = 0;  // index of the array's first word in the state's word order
  for (int s = 0; s < 3; ++s) {
    const uint32_t* w = a.words[s];
    const size_t n = a.count[s];
    const size_t n4 = (reinterpret_cast<uintptr_t>(w) & 15u) == 0 ? n / 4u : 0u;
    const uint4* w4 = reinterpret_cast<const uint4*>(w);
    size_t i = tid;
    for (; i + 3u * nth < n4; i += 4u * nth) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = w4[i + u * nth];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t at = base + static_cast<uint32_t>(4u * (i + u * nth));
        f.absorb(v[u].x, at, kStateSeed);
        f.absorb(v[u].y, at + 1u, kStateSeed);
        f.absorb(v[u].z, at + 2u, kStateSeed);
        f.absorb(v[u].w, at + 3u, kStateSeed);
      }
    }
    for (; i < n4; i += nth) {
      const uint4 v = w4[i];
      const uint32_t at = base + static_cast<uint32_t>(4u * i);
      f.absorb(v.x, at, kStateSeed);
      f.absorb(v.y, at + 1u, kStateSeed);
      f.absorb(v.z, at + 2u, kStateSeed);
      f.absorb(v.w, at + 3u, kStateSeed);
    }
    for (size_t j = 4u * n4 + tid; j < n; j += nth) f.absorb(w[j], base + static_cast<uint32_t>(j), kStateSeed);
    base += static_cast<uint32_t>(n);
  }
  const uint32_t chunks = (row_words(a) + kRowChunk - 1u) / kRowChunk;
  const uint32_t live = min(*a.pos_next, a.capacity), per_layer = live * chunks, entries = a.n_full * per_layer;
  for (size_t e = tid; e < entries; e += nth) {
    const size_t layer = e / per_layer, at = e % per_layer;  // (slot, chunk) entries are contiguous per layer
    f.merge(a.slot_hash + (layer * a.capacity * chunks + at) * 8u);
  }
  f.block_fold(sh);
  if (threadIdx.x == 0)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      a.partial[blockIdx.x * 8u + k] = f.x[k];
      a.partial[blockIdx.x * 8u + 4u + k] = f.a[k];
    }
}

// (3) the partials, the position and the seeds -> the address; the history
// rows up to the position are digested from now on
__global__ void __launch_bounds__(256) digest_final_kernel(const DigestArgs a) {
  __shared__ uint32_t sh[8][8];
  Fold f;
  f.clear();
  for (uint32_t b = threadIdx.x; b < kDigestBlocks; b += blockDim.x) f.merge(a.partial + b * 8u);
  f.block_fold(sh);
  if (threadIdx.x == 0) {
    uint32_t* out = a.out;
    if (a.slot) {
      const uint32_t at = *a.slot;
      *a.slot = at + 1u;
      if (at >= a.slots) return;  // past the caller's buffer: nothing written, the cursor kept
      out += at * 8u;
    }
    const uint32_t pos = *a.pos_next;
    const uint32_t s = fmix32(pos ^ 0xA54FF53Au) ^ fmix32(a.seed[0] + 0x510E527Fu) ^
                       fmix32(a.seed[1] * 3u + 0x9B05688Cu) ^ fmix32(a.seed[2] ^ 0x1F83D9ABu) ^
                       fmix32(a.seed[3] + 0x5BE0CD19u);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[k] = fmix32(f.x[k] ^ fmix32(s + static_cast<uint32_t>(k) * 0x9E3779B9u));
      out[4 + k] = fmix32(f.a[k] ^ fmix32(s ^ static_cast<uint32_t>(k + 1) * 0x85EBCA77u));
    }
    *a.cursor = pos;
  }
}

constexpr uint64_t kCopyChunk = 16384;  // bytes per CTA
__global__ void __launch_bounds__(256) copy_segments_kernel(const CopySeg* segs) {
  const CopySeg sg = segs[blockIdx.y];
  const uint64_t b0 = static_cast<uint64_t>(blockIdx.x) * kCopyChunk;
  if (b0 >= sg.bytes) return;
  const uint64_t b1 = min(sg.bytes, b0 + kCopyChunk);
  const bool v16 = ((reinterpret_cast<uintptr_t>(sg.src) | reinterpret_cast<uintptr_t>(sg.dst) | sg.bytes) & 15u) == 0;
  if (v16) {
    const uint4* s = reinterpret_cast<const uint4*>(sg.src);
    uint4* d = reinterpret_cast<uint4*>(sg.dst);
    for (uint64_t i = b0 / 16u + threadIdx.x; i < b1 / 16u; i += blockDim.x) d[i] = s[i];
  } else {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(sg.src);
    uint32_t* d = reinterpret_cast<uint32_t*>(sg.dst);
    for (uint64_t i = b0 / 4u + threadIdx.x; i < b1 / 4u; i += blockDim.x) d[i] = s[i];
  }
}

}  // namespace

cudaError_t launch_copy_segments(const CopySeg* segs_device, uint32_t n, uint64_t max_bytes, cudaStream_t s) {
  if (n == 0 || max_bytes == 0) return cudaSuccess;
  const uint64_t chunks = (max_bytes + kCopyChunk - 1u) / kCopyChunk;
  if (chunks > 0x7fffffffull) return cudaErrorInvalidValue;
  for (uint32_t first = 0; first < n; first += 65535u) {  // grid y holds 65535 segments
    const uint32_t count = std::min(65535u, n - first);
    copy_segments_kernel<<<dim3(static_cast<uint32_t>(chunks), count), 256, 0, s>>>(segs_device + first);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_state_digest(const DigestArgs& a, cudaStream_t s) {
  if (!a.cursor || !a.pos_next || !a.partial || !a.out || a.capacity == 0) return cudaErrorInvalidValue;
  if (a.n_full && (!a.slot_hash || (a.packets ? (a.pbytes % 4u) != 0 : (!a.kcache || !a.vcache || a.hd % 2u))))
    return cudaErrorInvalidValue;
  if (a.n_full) digest_rows_kernel<<<kDigestBlocks, 256, 0, s>>>(a);
  digest_fold_kernel<<<kDigestBlocks, 256, 0, s>>>(a);
  digest_final_kernel<<<1, 256, 0, s>>>(a);
  return cudaGetLastError();
}

// ----------------------------------------------------------------- host side
std::vector<Key256> prefix_identities(const uint32_t* ids, size_t n, uint32_t epoch) {
  std::vector<Key256> keys(n + 1);
  Key256 k;
  for (uint32_t j = 0; j < 8; ++j) k[j] = fmix32(epoch * 0x9E3779B1u + (j + 1u) * 0x85EBCA77u);
  keys[0] = k;
  for (size_t i = 0; i < n; ++i) {
    const uint32_t t = fmix32(ids[i] ^ fmix32(static_cast<uint32_t>(i) * 0xC2B2AE3Du + 0x27D4EB2Fu));
    for (uint32_t j = 0; j < 8; ++j) k[j] = fmix32((k[j] ^ t) + (j + 1u) * 0x165667B1u);
    keys[i + 1] = k;
  }
  return keys;
}

cudaError_t DevMem::alloc(size_t bytes, cudaStream_t stream) {
  if (p) cudaFreeAsync(p, s);
  p = nullptr;
  n = 0;
  s = stream;
  const cudaError_t e = cudaMallocAsync(&p, std::max<size_t>(bytes, 16), stream);
  if (e != cudaSuccess) {
    p = nullptr;
    return e;
  }
  n = bytes;
  return cudaSuccess;
}
DevMem::~DevMem() {
  if (p) cudaFreeAsync(p, s);
}

std::shared_ptr<HistoryEntry> HistoryIndex::find(const uint32_t* ids, size_t n, const std::vector<Key256>& keys,
                                                 size_t minimum, uint32_t* lookups) {
  uint32_t probes = 0;
  std::shared_ptr<HistoryEntry> best;
  for (auto it = lengths_.rbegin(); it != lengths_.rend(); ++it) {  // longest first
    const uint32_t len = it->first;
    if (len > n) continue;
    if (len < minimum) break;
    ++probes;
    const auto f = entries_.find(keys[len]);
    if (f == entries_.end()) continue;
    const HistoryEntry& e = *f->second;
    if (e.saved && e.ids.size() == len && std::equal(e.ids.begin(), e.ids.end(), ids)) {
      best = f->second;
      break;
    }
  }
  if (best) touch(*best);
  if (lookups) *lookups = probes;
  return best;
}

std::shared_ptr<HistoryEntry> HistoryIndex::reserve(const uint32_t* ids, uint32_t count, uint32_t kind,
                                                    const Key256& key) {
  const auto f = entries_.find(key);
  if (f != entries_.end()) {
    HistoryEntry& e = *f->second;
    if (e.ids.size() == count && std::equal(e.ids.begin(), e.ids.end(), ids)) {
      e.kind |= kind;
      touch(e);
    }
    return nullptr;  // held already (or an identity collision, which is not admitted)
  }
  auto e = std::make_shared<HistoryEntry>();
  e->ids.assign(ids, ids + count);
  e->key = key;
  e->kind = kind;
  touch(*e);
  entries_[key] = e;
  ++lengths_[count];
  return e;
}

std::shared_ptr<HistoryBlock> HistoryIndex::block(const Key256& identity, uint32_t first, uint32_t count,
                                                  bool* fresh) {
  std::weak_ptr<HistoryBlock>& w = blocks_[identity];
  std::shared_ptr<HistoryBlock> b = w.lock();
  if (b && b->ready && b->first == first && b->count == count) {
    *fresh = false;
    return b;
  }
  b = std::make_shared<HistoryBlock>();
  b->first = first;
  b->count = count;
  w = b;
  *fresh = true;
  return b;
}

void HistoryIndex::erase(const std::shared_ptr<HistoryEntry>& e) {
  if (!e) return;
  const auto f = entries_.find(e->key);
  if (f == entries_.end() || f->second != e) return;
  entries_.erase(f);
  const auto l = lengths_.find(static_cast<uint32_t>(e->ids.size()));
  if (l != lengths_.end() && --l->second == 0) lengths_.erase(l);
}

uint64_t HistoryIndex::bytes() {
  uint64_t total = 0;
  for (const auto& kv : entries_) total += kv.second->snapshot.n;
  for (auto it = blocks_.begin(); it != blocks_.end();) {
    if (auto b = it->second.lock()) {
      total += b->rows.n;
      ++it;
    } else {
      it = blocks_.erase(it);
    }
  }
  return total;
}

uint64_t HistoryIndex::evict(uint64_t budget, const HistoryEntry* keep0, const HistoryEntry* keep1) {
  uint64_t held = bytes();
  while (held > budget) {
    std::shared_ptr<HistoryEntry> victim;
    for (const auto& kv : entries_) {
      const HistoryEntry* e = kv.second.get();
      if (e == keep0 || e == keep1) continue;
      if (!victim || e->touched < victim->touched) victim = kv.second;
    }
    if (!victim) break;
    erase(victim);
    ++evictions;
    victim.reset();
    held = bytes();
  }
  return held;
}

const ReplyTree::Node* ReplyTree::find(const Key256& key, uint32_t position, uint32_t* slot) const {
  const auto f = index_.find(At{key, position});
  if (f == index_.end()) return nullptr;
  if (slot) *slot = f->second;
  return &nodes_[f->second];
}

void ReplyTree::record(const Key256& key, uint32_t position, uint32_t token, const Key256& next) {
  if (nodes_.empty()) nodes_.resize(kCapacity);
  const At at{key, position};
  uint32_t slot;
  const auto f = index_.find(at);
  if (f != index_.end()) {
    slot = f->second;
  } else {
    slot = cursor_;
    Node& old = nodes_[slot];
    if (old.valid) index_.erase(At{old.key, old.position});
    cursor_ = (cursor_ + 1u) % kCapacity;
    size_ = std::min(kCapacity, size_ + 1u);
    index_[at] = slot;
  }
  Node& nd = nodes_[slot];
  nd.key = key;
  nd.next = next;
  nd.position = position;
  nd.token = token;
  nd.valid = true;
}

}  // namespace rta
