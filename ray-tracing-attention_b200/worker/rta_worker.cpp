// rta_worker -- drop-in replacement for the reference's native worker process.
//
// It speaks the binary stdin/stdout protocol of ray_tracing/native/src/
// optical_resident.cpp (main loop :964-971) so that the unmodified
// ray_tracing.runtime.ResidentRuntime (resident_runtime.py:10) drives the B200
// backend: same argv, same hello words, same request framing <3I op,count,debug>
// + body, same reply framing <2I status,size> + payload, and the payload
// layouts its parsers read (resident_runtime.py:116-263).  All model work goes
// through librta_cuda.so (include/rta.h); this file only frames bytes.
//
// Served operations: 0 quit, 1 prefill (debug 0, 1 = per-position and per-layer
// rows, 2 = timing layout), 2 generate, 4 vocabulary, 6 mlp, 8 resources,
// 9 stream, 10 grow (capacity), 11 / 12 checkpointed prefill, 13
// finish_history, 14 full-attention diagnostic (dense receipts).  With the
// `cache` argument on (argv[4], on by default as in the reference) the handle
// keeps the prefix boundaries and the reply tree (RTA_MODEL_CACHE) and the
// replies carry their counters.  The attention history is kept
// in the reference's packet format.  Operations tied to the ray-traced geometry
// and its statistics (5 codec, 7 aperture, 15 statistics) answer status 1, which
// the runtime turns into RuntimeError.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "rta.h"

namespace {

using Clock = std::chrono::steady_clock;

// ------------------------------------------------------------ model.json
// Minimal reader for the flat "model_spec" object the compiler writes
// (ray_tracing/compiler/export.py:233, spec.py:66).
struct SpecReader {
  std::string text;
  size_t find_key(const std::string& key) const {
    const size_t spec = text.find("\"model_spec\"");
    if (spec == std::string::npos) throw std::runtime_error("model.json has no model_spec");
    const size_t at = text.find("\"" + key + "\"", spec);
    if (at == std::string::npos) throw std::runtime_error("model_spec field missing: " + key);
    return text.find(':', at) + 1;
  }
  double number(const std::string& key) const {
    size_t i = find_key(key);
    while (i < text.size() && std::isspace(static_cast<unsigned char>(text[i]))) ++i;
    if (text.compare(i, 4, "true") == 0) return 1.0;
    if (text.compare(i, 5, "false") == 0) return 0.0;
    return std::stod(text.substr(i, 40));
  }
  std::vector<std::string> strings(const std::string& key) const {
    size_t i = text.find('[', find_key(key)), end = text.find(']', i);
    std::vector<std::string> out;
    while (true) {
      const size_t a = text.find('"', i);
      if (a == std::string::npos || a > end) break;
      const size_t b = text.find('"', a + 1);
      out.push_back(text.substr(a + 1, b - a - 1));
      i = b + 1;
    }
    return out;
  }
};

rta_model_spec read_spec(const std::string& dir) {
  std::ifstream f(dir + "/model.json");
  if (!f) throw std::runtime_error("cannot read model.json next to the model payload");
  std::stringstream ss;
  ss << f.rdbuf();
  SpecReader r{ss.str()};
  rta_model_spec s{};
  s.hidden_size = static_cast<uint32_t>(r.number("hidden_size"));
  s.middle_size = static_cast<uint32_t>(r.number("middle_size"));
  s.vocabulary_size = static_cast<uint32_t>(r.number("vocabulary_size"));
  s.attention_heads = static_cast<uint32_t>(r.number("attention_heads"));
  s.kv_heads = static_cast<uint32_t>(r.number("kv_heads"));
  s.attention_head_dim = static_cast<uint32_t>(r.number("attention_head_dim"));
  s.rotary_dim = static_cast<uint32_t>(r.number("rotary_dim"));
  s.state_heads = static_cast<uint32_t>(r.number("state_heads"));
  s.state_key_heads = static_cast<uint32_t>(r.number("state_key_heads"));
  s.state_head_dim = static_cast<uint32_t>(r.number("state_head_dim"));
  s.attention_gate = static_cast<uint32_t>(r.number("attention_gate"));
  s.qk_norm = static_cast<uint32_t>(r.number("qk_norm"));
  s.rope_theta = static_cast<float>(r.number("rope_theta"));
  s.norm_epsilon = static_cast<float>(r.number("norm_epsilon"));
  const auto kinds = r.strings("layer_types");
  if (kinds.empty() || kinds.size() > 256) throw std::runtime_error("model_spec.layer_types out of range");
  s.depth = static_cast<uint32_t>(kinds.size());
  for (size_t i = 0; i < kinds.size(); ++i) s.layer_kinds[i] = kinds[i] == "full" ? 1 : 2;
  return s;
}

// ------------------------------------------------------------- framing
template <class T>
void append(std::vector<char>& out, const T* v, size_t n) {
  const char* p = reinterpret_cast<const char*>(v);
  out.insert(out.end(), p, p + n * sizeof(T));
}
template <class T>
void append(std::vector<char>& out, std::initializer_list<T> v) {
  append(out, v.begin(), v.size());
}
void reply(uint32_t status, const std::vector<char>& payload) {
  const uint32_t header[2] = {status, static_cast<uint32_t>(payload.size())};
  std::cout.write(reinterpret_cast<const char*>(header), 8);
  if (!payload.empty()) std::cout.write(payload.data(), static_cast<std::streamsize>(payload.size()));
  std::cout.flush();
}
template <class T>
void input(std::vector<T>& v, size_t n) {
  v.resize(n);
  if (n && !std::cin.read(reinterpret_cast<char*>(v.data()), static_cast<std::streamsize>(n * sizeof(T))))
    throw std::runtime_error("Incomplete resident request body");
}

struct Worker {
  rta_model* model = nullptr;
  rta_model_spec spec{};
  std::string model_bin, geometry_bin, vocab_bin;
  uint32_t capacity = 300, position = 0;
  uint32_t stops[2] = {0xffffffffu, 0xffffffffu};
  uint32_t block = 128;  // RT_ATTENTION_BLOCK: receipt group size (128, 256 or 512)
  bool cache = true;     // argv[4] (optical_resident.cpp:967: argc <= 4 || stoul(argv[4]) != 0)

  void check(rta_status st) {
    if (st != RTA_OK) throw std::runtime_error(rta_model_last_error());
  }
  void open() {
    // the reference's history format: Q4_K key / Q6_K value packets
    check(rta_model_open_files_ex(&spec, model_bin.c_str(), geometry_bin.c_str(), vocab_bin.c_str(), capacity, 1u,
                                  RTA_MODEL_PACKET_HISTORY | (cache ? RTA_MODEL_CACHE : 0u), 0, &model));
  }

  // ops 1 / 11 / 12 (Resident::prefill, optical_resident.cpp:609-712): ids[count] +
  // stops[2] (+ op 11: u32 checkpoint; op 12: u32 n + n x <u32 position, u32 kind>)
  // -> 6 doubles + 8 control words [+ debug 1: final-normed rows [count][D] and
  // every layer's output rows [depth][count][D]] + 4 batch statistics [+ debug 2:
  // 6 phase timings] + the history-cache counters (prefill parser,
  // resident_runtime.py:116-158).  The checkpoint (op 11), or the largest
  // boundary of kind bit 1 (op 12), is the stable prefix the history cache
  // reports; the prefix itself is saved at the prompt's end
  // (optical_resident.cpp:616-622, :646-651).  A layer capture bypasses the
  // caches, as in the reference.
  void prefill(uint32_t op, uint32_t count, uint32_t debug) {
    if (debug > 2u || !count || count > capacity) throw std::runtime_error("Invalid resident prefix");
    std::vector<uint32_t> ids, st;
    input(ids, count);
    input(st, 2);
    uint32_t boundary = count;
    if (op == 11) {
      std::vector<uint32_t> b;
      input(b, 1);
      if (!b[0] || b[0] > count) throw std::runtime_error("Invalid prefix word IDs or boundary");
      boundary = b[0];
    } else if (op == 12) {
      std::vector<uint32_t> n;
      input(n, 1);
      if (n[0] > 4096u) throw std::runtime_error("Too many history boundaries");
      std::vector<uint32_t> marks;
      input(marks, 2ull * n[0]);
      uint32_t stable = 0;
      for (uint32_t i = 0; i < n[0]; ++i) {
        if (!marks[2 * i] || marks[2 * i] > count || !(marks[2 * i + 1] & 15u) || marks[2 * i + 1] > 15u)
          throw std::runtime_error("Invalid history boundary");
        if (marks[2 * i + 1] & 1u) stable = std::max(stable, marks[2 * i]);
      }
      if (stable) boundary = stable;
    }
    for (uint32_t id : ids)
      if (id >= spec.vocabulary_size) throw std::runtime_error("Invalid prefix word IDs or boundary");
    stops[0] = st[0];
    stops[1] = st[1];
    const size_t D = spec.hidden_size;
    std::vector<float> states, layers;
    const auto t0 = Clock::now();
    double gpu = 0.0;
    if (debug == 1u) {
      states.resize(count * D);
      layers.resize(static_cast<size_t>(spec.depth) * count * D);
      check(rta_model_prefill_capture(model, ids.data(), count, stops, states.data(), layers.data(), &gpu));
    } else {
      check(rta_model_prefill_checkpoint(model, ids.data(), count, stops, boundary, &gpu));
    }
    const double wall = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    position = count;
    uint64_t c[RTA_CACHE_INFO_WORDS] = {0};
    double cms[3] = {0.0, 0.0, 0.0};
    const bool cached = cache && debug != 1u;
    if (cached) check(rta_model_cache_info(model, c, RTA_CACHE_INFO_WORDS, cms));
    else c[RTA_CACHE_COMPUTED_TOKENS] = count;
    std::vector<char> out;
    append<double>(out, {0.0, gpu, wall, wall, static_cast<double>(c[RTA_CACHE_PREFILL_HIT]),
                         static_cast<double>(c[RTA_CACHE_REUSED_TOKENS])});
    append<uint32_t>(out, {ids.back(), 0u, 1u, 0u, stops[0], stops[1], 0u, 0u});
    if (debug == 1u) {
      append(out, states.data(), states.size());
      append(out, layers.data(), layers.size());
    }
    append<uint64_t>(out, {1ull, static_cast<uint64_t>(count), 0ull, static_cast<uint64_t>(count)});
    if (debug == 2u) append<double>(out, {0.0, 0.0, 0.0, 0.0, 0.0, 0.0});  // no ray-traced phases here
    append<uint64_t>(out, {0ull, 0ull});                                    // feature rows traced / reused
    append<uint64_t>(out, {c[RTA_CACHE_STABLE_TOKENS], c[RTA_CACHE_SNAPSHOT_KIND]});
    append<uint64_t>(out, {c[RTA_CACHE_SHARED_BLOCKS], c[RTA_CACHE_SAVED_BOUNDARIES], c[RTA_CACHE_BOUNDARIES],
                           c[RTA_CACHE_LOOKUPS], c[RTA_CACHE_COMPUTED_TOKENS], c[RTA_CACHE_EVICTIONS]});
    append<double>(out, {cms[0]});                            // history lookup wall ms
    append<uint64_t>(out, {0ull, c[RTA_CACHE_ADDRESS_HIT]});  // rebuilt tokens, address hit
    if (debug == 2u) append<double>(out, {0.0, 0.0});
    reply(0, out);
  }

  // op 13 (finishHistory, optical_resident.cpp:743-759): the prompt plus the
  // generated reply saved as a boundary -> saved, tokens, boundaries, wall ms
  // (nothing is saved with the cache off).
  void finish_history() {
    const auto t0 = Clock::now();
    uint64_t saved = 0, tokens = 0, boundaries = 0;
    if (cache) check(rta_model_finish_history(model, &saved, &tokens, &boundaries));
    std::vector<char> out;
    append<uint64_t>(out, {saved, tokens, boundaries});
    append<double>(out, {std::chrono::duration<double, std::milli>(Clock::now() - t0).count()});
    reply(0, out);
  }

  // GenerationPacket::bytes (optical_resident.cpp:63-71), parsed by _generation_result
  std::vector<char> packet(const std::vector<uint32_t>& ids, bool running, double gpu, double wall) {
    std::vector<char> out;
    const uint32_t n = static_cast<uint32_t>(std::min<size_t>(ids.size(), 64));
    uint64_t c[RTA_CACHE_INFO_WORDS] = {0};
    double cms[3] = {0.0, 0.0, 0.0};
    if (cache) check(rta_model_cache_info(model, c, RTA_CACHE_INFO_WORDS, cms));
    const uint32_t replayed = static_cast<uint32_t>(c[RTA_CACHE_REPLAYED_TOKENS]);
    const bool all_cached = replayed > 0 && replayed == ids.size();
    append<double>(out, {gpu, wall, 1.0, 1.0, 0.0, all_cached ? 1.0 : 0.0, static_cast<double>(position), 0.0, 0, 0,
                         0, 0, 0, 0, 0, 0, 0, 0});
    append<uint32_t>(out, {n ? ids[n - 1] : 0u, n, running ? 1u : 0u, 0u, stops[0], stops[1], 0u, 0u});
    std::vector<uint32_t> id64(64, 0u);
    std::copy_n(ids.begin(), n, id64.begin());
    append(out, id64.data(), 64);
    // rows through the MLPs: computed tokens but a final stop id (generatePacket's counts, :845-846)
    const uint32_t fresh = static_cast<uint32_t>(ids.size()) - replayed;
    const uint32_t computed = fresh - (!running && fresh > 0 ? 1u : 0u);
    append<uint32_t>(out, {spec.middle_size * spec.depth * computed, spec.middle_size * spec.depth * computed,
                           spec.vocabulary_size * computed, replayed,
                           static_cast<uint32_t>(c[RTA_CACHE_TREE_LEAF])});
    append<double>(out, {0.0, 0.0, 0.0, cms[1]});  // ray-query time by kind: history, vocabulary, mlp, cache
    append<uint32_t>(out, {replayed, static_cast<uint32_t>(c[RTA_CACHE_TREE_QUERIES]),
                           static_cast<uint32_t>(c[RTA_CACHE_TREE_NODES]),
                           static_cast<uint32_t>(c[RTA_CACHE_TREE_CAPACITY])});
    append<double>(out, {cms[1], cms[1], cms[2], static_cast<double>(c[RTA_CACHE_RESTORED_TOKENS]),
                         static_cast<double>(c[RTA_CACHE_CHECKPOINT_RESTORED])});
    append<uint32_t>(out, {replayed, 0u});  // candidates, rejected candidates
    append<uint64_t>(out, {0ull, 0ull});
    return out;
  }

  bool generate_one_packet(uint32_t count) {
    std::vector<uint32_t> ids(count);
    uint32_t n = 0;
    double gpu = 0.0;
    const auto t0 = Clock::now();
    check(rta_model_generate(model, count, ids.data(), &n, &gpu));
    const double wall = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    ids.resize(n);
    position += n;
    const bool running = !(n && (ids.back() == stops[0] || ids.back() == stops[1])) && n == count;
    reply(0, packet(ids, running, gpu, wall));
    return running;
  }

  // op 4: hidden[D] -> timings, winner, hit ids, first decoded rows, packets, charts
  void vocabulary() {
    const uint32_t D = spec.hidden_size, V = spec.vocabulary_size, blocks = D / 256;
    std::vector<float> h;
    input(h, D);
    uint32_t arg = 0;
    float best = 0.f;
    const auto t0 = Clock::now();
    check(rta_model_vocabulary(model, h.data(), nullptr, &arg, &best));
    const double wall = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    std::vector<char> out;
    append<double>(out, {wall, wall, 0.0, 0.0, 0.0});
    float b20 = best + 20.0f, one = 1.0f;
    uint32_t w[4] = {arg, 0, 0, 0};
    std::memcpy(&w[1], &b20, 4);
    std::memcpy(&w[2], &one, 4);
    std::memcpy(&w[3], &one, 4);
    append(out, w, 4);
    append<uint32_t>(out, {V});
    std::vector<uint32_t> ids(V);
    for (uint32_t i = 0; i < V; ++i) ids[i] = i;
    append(out, ids.data(), V);
    std::vector<float> rows(256ull * D, 0.f);  // geometric word rows are a ray-traced artefact: zeros
    append(out, rows.data(), rows.size());
    std::vector<uint32_t> packets(blocks * 256ull);
    std::memcpy(packets.data(), h.data(), D * 4ull);  // encodePathPair is the identity on the bits
    append(out, packets.data(), packets.size());
    std::vector<float> charts(blocks * 4ull, 0.f);
    append(out, charts.data(), charts.size());
    append<uint32_t>(out, {V * blocks});
    reply(0, out);
  }

  // op 6: rows x D -> rows x D output, rows x middle activation, rows feature hits, 3 timings
  void mlp(uint32_t rows, uint32_t layer) {
    const uint32_t D = spec.hidden_size, F = spec.middle_size;
    if (rows == 0 || rows > std::min(capacity, 32u) || layer >= spec.depth)
      throw std::runtime_error("Invalid optical MLP input");
    std::vector<float> x;
    input(x, static_cast<size_t>(rows) * D);
    for (float v : x)
      if (!std::isfinite(v)) throw std::runtime_error("Optical MLP input must be finite");
    std::vector<float> y(static_cast<size_t>(rows) * D), act(static_cast<size_t>(rows) * F);
    const auto t0 = Clock::now();
    check(rta_model_mlp(model, layer, x.data(), rows, y.data(), act.data()));
    const double wall = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    std::vector<char> out;
    append(out, y.data(), y.size());
    append(out, act.data(), act.size());
    std::vector<uint32_t> hits(rows, F);
    append(out, hits.data(), rows);
    append<double>(out, {0.0, wall, 0.0});
    reply(0, out);
  }

  // op 14 (attentionCheck, resident_attention_runtime.inl:646-753): rows of rotated
  // q + compact K/V history + gate -> outputs, physical, history packets, receipts
  void attention(uint32_t rows, uint32_t layer) {
    uint32_t hdr[4];
    if (!std::cin.read(reinterpret_cast<char*>(hdr), sizeof hdr)) throw std::runtime_error("Incomplete attention header");
    const uint32_t count = hdr[0], query_start = hdr[1], history_start = hdr[2];
    const uint32_t H = spec.attention_heads, KVH = spec.kv_heads, hd = spec.attention_head_dim;
    if (!rows || rows > 32 || !count || hdr[3] || layer >= spec.depth || spec.layer_kinds[layer] != 1)
      throw std::runtime_error("Invalid full-attention diagnostic shape or causal domain");
    std::vector<float> q, k, v, gate;
    input(q, static_cast<size_t>(rows) * H * hd);
    input(k, static_cast<size_t>(count) * KVH * hd);
    input(v, static_cast<size_t>(count) * KVH * hd);
    input(gate, static_cast<size_t>(rows) * H * hd);
    uint32_t records = 0;
    for (uint32_t r = 0; r < rows; ++r)
      records += H * ((std::min(query_start - history_start + r + 1u, capacity) + block - 1u) / block);
    const uint32_t stride = hd + 8u + block / 32u, pbytes = KVH * (144u + 210u);
    std::vector<float> out(q.size()), phys(static_cast<size_t>(rows) * H * 2);
    std::vector<uint8_t> packets(static_cast<size_t>(count) * pbytes);
    std::vector<uint32_t> receipts(static_cast<size_t>(records) * stride);
    uint32_t n = 0;
    double gpu = 0.0;
    const auto t0 = Clock::now();
    check(rta_model_attention(model, layer, q.data(), k.data(), v.data(), gate.data(), rows, count, query_start,
                              history_start, block, out.data(), phys.data(), packets.data(), receipts.data(), &n,
                              &gpu));
    const double wall = std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
    if (n != records) throw std::runtime_error("Full-attention diagnostic record count mismatch");
    const uint32_t legacy = history_start == 0u ? 1u : 0u;
    std::vector<char> o;
    append<uint32_t>(o, {0x41545231u, rows, count, H, KVH, hd, pbytes, block, stride, records, legacy, 0u});
    append<double>(o, {gpu, 0.0, 0.0, wall});
    append(o, out.data(), out.size());
    append(o, phys.data(), phys.size());
    append(o, out.data(), out.size());    // legacy output: this backend has one detector
    append(o, phys.data(), phys.size());
    append(o, packets.data(), packets.size());
    append(o, receipts.data(), receipts.size());
    reply(0, o);
  }

  // op 8: the 61 counters resident_runtime.resources() names, in its order
  void resources() {
    uint64_t r[9] = {0};
    check(rta_model_resources(model, r, 9));
    std::vector<uint64_t> v(61, 0ull);
    v[1] = r[0] + r[1] + r[2] + r[3];  // device allocation bytes (payloads, derived, history, state)
    v[9] = r[0];                        // packed coefficient bytes
    v[13] = r[2];                       // history bytes
    v[15] = r[3];                       // recurrent field bytes
    v[26] = 32;                         // workspace rows (MLP check rows)
    v[38] = block;                      // attention block
    std::vector<char> out;
    append(out, v.data(), v.size());
    reply(0, out);
  }

  // op 10: reopen with a larger history ring -> previous, capacity, wall ms
  void grow(uint32_t next) {
    if (next <= capacity) throw std::runtime_error("Invalid tree growth request");
    const auto t0 = Clock::now();
    const uint32_t previous = capacity;
    rta_model_close(model);
    model = nullptr;
    capacity = next;
    open();
    position = 0;  // the reference re-prefills after growth
    std::vector<char> out;
    append<double>(out, {static_cast<double>(previous), static_cast<double>(capacity),
                         std::chrono::duration<double, std::milli>(Clock::now() - t0).count()});
    reply(0, out);
  }
};

}  // namespace

int main(int argc, char** argv) {
  try {
    if (argc < 3) throw std::runtime_error("Usage: rta_worker optical_model.bin vocabulary.bin [capacity] ...");
    Worker w;
    w.model_bin = argv[1];
    w.vocab_bin = argv[2];
    const std::string dir = w.model_bin.substr(0, w.model_bin.find_last_of('/') == std::string::npos
                                                       ? 0
                                                       : w.model_bin.find_last_of('/'));
    w.geometry_bin = (dir.empty() ? std::string(".") : dir) + "/geometry_weights.bin";
    w.capacity = argc > 3 ? static_cast<uint32_t>(std::stoul(argv[3])) : 300u;
    w.cache = argc <= 4 || std::stoul(argv[4]) != 0;
    w.spec = read_spec(dir.empty() ? "." : dir);
    if (const char* b = std::getenv("RT_ATTENTION_BLOCK")) {
      w.block = static_cast<uint32_t>(std::strtoul(b, nullptr, 10));
      if (w.block != 128 && w.block != 256 && w.block != 512)
        throw std::runtime_error("RT_ATTENTION_BLOCK must be 128, 256 or 512");
    }
    w.open();
    // hello: magic, depth, blocks (= depth, header word 2), middle, mode =
    // quantization 4 | standard MLP 4096 | ordered detector 131072
    const uint32_t hello[5] = {0x5254523au, w.spec.depth, w.spec.depth, w.spec.middle_size, 4u | 4096u | 131072u};
    std::cout.write(reinterpret_cast<const char*>(hello), 20);
    std::cout.flush();
    uint32_t op = 0;
    while (std::cin.read(reinterpret_cast<char*>(&op), 4)) {
      if (!op) break;
      uint32_t count = 0, debug = 0;
      if (!std::cin.read(reinterpret_cast<char*>(&count), 4) || !std::cin.read(reinterpret_cast<char*>(&debug), 4))
        throw std::runtime_error("Incomplete resident request");
      try {
        if (op == 1 || op == 11 || op == 12) w.prefill(op, count, debug);
        else if (op == 13) w.finish_history();
        else if (op == 2) {
          if (count == 0 || count > 4096) throw std::runtime_error("Resident generation expects 1..4096 tokens");
          w.generate_one_packet(count);
        } else if (op == 9) {
          if (!count || count > 64) throw std::runtime_error("Resident stream expects 1..64 tokens");
          for (uint32_t i = 0; i < count; ++i)
            if (!w.generate_one_packet(1)) break;
        } else if (op == 4) w.vocabulary();
        else if (op == 6) w.mlp(count, debug);
        else if (op == 8) w.resources();
        else if (op == 10) w.grow(count);
        else if (op == 14) w.attention(count, debug);
        else throw std::runtime_error("Operation " + std::to_string(op) + " is not served by the B200 backend");
      } catch (const std::exception& e) {
        std::cerr << e.what() << std::endl;
        reply(1, {});
      }
    }
    if (w.model) rta_model_close(w.model);
    return 0;
  } catch (const std::exception& e) {
    std::cerr << e.what() << std::endl;
    return 1;
  }
}
