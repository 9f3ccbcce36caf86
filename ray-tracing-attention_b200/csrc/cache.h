// cache.h -- the decode caches of single-sequence handles (RTA_MODEL_CACHE):
//   * prefix boundaries: the decode state (residual row, recurrent and
//     convolution states) saved where a prompt or a generated reply ended,
//     plus the attention history of the prefix in immutable 16-position blocks
//     shared by every boundary whose ids agree up to the block's end
//     (SharedHistoryCache, ray_tracing/native/src/shared_history_cache.hpp:5-142);
//   * the reply tree: (state address, position) -> emitted token and the
//     successor address, so a reply already decoded from an identical state is
//     replayed without computing it (ReplyTreeCache, reply_cache.hpp:6-68);
//   * the state address: a 256-bit digest of every live input of the next
//     decode step -- residual row, recurrent and convolution states, the
//     visible history rows with their absolute positions, the position, the
//     stop ids -- computed on the device (OpticalPathKey,
//     optical_path_key.hpp:7-91, shaders/optical_path_key.comp).
// The reference finds candidates by ray queries against an angular chart of
// the address and then compares the full key; here the host looks the full
// key up in hash maps (the chart only ever served the ray query).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <array>
#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <unordered_map>
#include <vector>

namespace rta {

using Key256 = std::array<uint32_t, 8>;
struct Key256Hash {
  size_t operator()(const Key256& k) const noexcept {
    return (static_cast<size_t>(k[0]) << 32) ^ k[1] ^ (static_cast<size_t>(k[6]) << 13);
  }
};

// --------------------------------------------------------------- device side
// One launch copies every segment: src and dst 4-byte aligned, bytes % 4 == 0
// (16-byte vectors where a segment is 16-byte aligned throughout).
struct CopySeg {
  const void* src;
  void* dst;
  uint64_t bytes;
};
cudaError_t launch_copy_segments(const CopySeg* segs_device, uint32_t n, uint64_t max_bytes, cudaStream_t s);

// The state address.  Three launches: (1) the history rows written since the
// last digest (positions [*cursor, *pos_next), the live window at most) are
// hashed into per-slot digests of their 128-word chunks; (2) every state word
// and the chunk digests of the live slots are folded into per-CTA partial
// digests; (3) one CTA
// combines them with the position and the seeds into out[8] and advances
// *cursor.  Lanes 0-3 fold by XOR and lanes 4-7 by addition: both are
// order-free, so the CTA split and the slot order do not matter.
constexpr uint32_t kDigestBlocks = 592;  // 4 CTAs of 256 threads per SM
constexpr uint32_t kRowChunk = 128;      // history row words per chunk digest
struct DigestArgs {
  const uint32_t* words[3] = {nullptr, nullptr, nullptr};  // state row, recurrent states, convolution states
  size_t count[3] = {0, 0, 0};                             // 32-bit words of each
  const __half* kcache = nullptr;  // fp16 rings [layer][kvh][capacity][hd] (null with packets)
  const __half* vcache = nullptr;
  const uint8_t* packets = nullptr;  // packet rings [layer][capacity][pbytes]
  size_t layer_kv = 0;               // halves between two layers' K planes
  uint32_t n_full = 0, kvh = 0, hd = 0, capacity = 0, pbytes = 0;
  uint32_t* slot_hash = nullptr;       // [n_full][capacity][row chunks][8]
  uint32_t* cursor = nullptr;          // history positions digested so far (device word)
  const uint32_t* pos_next = nullptr;  // the control block's next position
  uint32_t* partial = nullptr;         // [kDigestBlocks][8]
  uint32_t* out = nullptr;             // [8], or [slots][8] with a slot counter
  // Optional device counter: the address goes to out[*slot] and the counter
  // advances (a graph that digests after every replay); `slots` bounds it.
  uint32_t* slot = nullptr;
  uint32_t slots = 0;
  uint32_t seed[4] = {0, 0, 0, 0};     // epoch, capacity, stop ids
};
cudaError_t launch_state_digest(const DigestArgs& a, cudaStream_t s);

// ----------------------------------------------------------------- host side
// Chained identities of every prefix of ids: keys[i] names ids[0..i) (keys[0]
// the empty prefix of this epoch).  Equal keys mean equal prefixes up to a
// 2^-256 accident; the index still compares the ids before it reuses anything.
std::vector<Key256> prefix_identities(const uint32_t* ids, size_t n, uint32_t epoch);

// Stream-ordered device allocation owned by a host object.
struct DevMem {
  void* p = nullptr;
  size_t n = 0;
  cudaStream_t s = nullptr;
  DevMem() = default;
  DevMem(const DevMem&) = delete;
  DevMem& operator=(const DevMem&) = delete;
  cudaError_t alloc(size_t bytes, cudaStream_t stream);
  ~DevMem();
};

// The attention history of positions [first, first + count) of every full
// layer, in the handle's row format; immutable once saved.
struct HistoryBlock {
  uint32_t first = 0, count = 0;
  bool ready = false;
  DevMem rows;
};

// One saved boundary: ids[0..n) and the decode state after them.
struct HistoryEntry {
  std::vector<uint32_t> ids;
  Key256 key{};
  uint32_t kind = 0;  // 1: a prompt end, 2: a generated reply's end
  uint64_t touched = 0;
  DevMem snapshot;  // [state row | recurrent states | convolution states]
  bool saved = false;
  std::vector<std::shared_ptr<HistoryBlock>> blocks;
  Key256 address{};  // the state address at the boundary, when known
  bool address_ready = false;
  uint32_t stops[2] = {0xffffffffu, 0xffffffffu};
};

class HistoryIndex {
 public:
  // The longest saved boundary whose ids are a prefix of ids[0..n) and at least
  // `minimum` long (null: none); *lookups = the prefix lengths probed.
  std::shared_ptr<HistoryEntry> find(const uint32_t* ids, size_t n, const std::vector<Key256>& keys,
                                     size_t minimum, uint32_t* lookups);
  // A new boundary for ids[0..count) (null when one exists already: it is touched).
  std::shared_ptr<HistoryEntry> reserve(const uint32_t* ids, uint32_t count, uint32_t kind, const Key256& key);
  // The shared block named by identity (the key of the prefix it ends), made
  // if absent (*fresh = true: its rows still have to be saved).
  std::shared_ptr<HistoryBlock> block(const Key256& identity, uint32_t first, uint32_t count, bool* fresh);
  void erase(const std::shared_ptr<HistoryEntry>& e);
  // Drop the least recently used boundaries until the held bytes fit the
  // budget (entries named by keep stay); returns the bytes then held.
  uint64_t evict(uint64_t budget, const HistoryEntry* keep0, const HistoryEntry* keep1);
  uint64_t bytes();
  uint32_t size() const { return static_cast<uint32_t>(entries_.size()); }
  void touch(HistoryEntry& e) { e.touched = ++clock_; }
  uint64_t evictions = 0;

 private:
  std::unordered_map<Key256, std::shared_ptr<HistoryEntry>, Key256Hash> entries_;
  std::map<uint32_t, uint32_t> lengths_;  // boundary length -> boundaries of that length
  std::unordered_map<Key256, std::weak_ptr<HistoryBlock>, Key256Hash> blocks_;
  uint64_t clock_ = 0;
};

class ReplyTree {
 public:
  static constexpr uint32_t kCapacity = 65536;  // nodes; the oldest is overwritten (ReplyTreeCache::nodeCapacity)
  struct Node {
    Key256 key{}, next{};
    uint32_t position = 0, token = 0;
    bool valid = false;
  };
  const Node* find(const Key256& key, uint32_t position, uint32_t* slot) const;
  void record(const Key256& key, uint32_t position, uint32_t token, const Key256& next);
  uint32_t size() const { return size_; }

 private:
  struct At {
    Key256 key;
    uint32_t position;
    bool operator==(const At& o) const { return position == o.position && key == o.key; }
  };
  struct AtHash {
    size_t operator()(const At& a) const noexcept { return Key256Hash{}(a.key) ^ (static_cast<size_t>(a.position) * 0x9E3779B97F4A7C15ull); }
  };
  std::vector<Node> nodes_;
  std::unordered_map<At, uint32_t, AtHash> index_;
  uint32_t cursor_ = 0, size_ = 0;
};

}  // namespace rta
