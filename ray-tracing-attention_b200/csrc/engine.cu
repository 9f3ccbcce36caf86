// engine.cu -- the resident decode engine behind the rta_model_* C-ABI.
//
// It owns one model on one GPU: the exporter's three payloads
// (optical_model.bin parameters, geometry_weights.bin matrices and
// vocabulary.bin rows; ray_tracing/compiler/export.py:51-150) copied to HBM,
// load-time row gathers that turn the reference's row modes 1/2/3
// (resident_quant.glsl:21-27) into plain row-major matrices, fp16 K/V rings,
// recurrent states, and two CUDA graphs: one decode step (readout -> argmax ->
// embedding -> layers, the per-token loop of Resident::generatePacket,
// optical_resident.cpp:825-828) and one prefill step (prompt token ->
// embedding -> layers).  Positions, the running flag and emitted ids live in a
// device control block, so the graphs replay unchanged step after step.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "../../include/rta.h"
#include "attention.h"
#include "cache.h"
#include "layers.h"
#include "packets.cuh"
#include "rta_internal.h"

namespace rta {
namespace {

thread_local std::string g_model_error = "no error";

struct Failure {
  rta_status code;
  std::string msg;
};
#define RTA_CUDA(call)                                                                                     \
  do {                                                                                                     \
    cudaError_t e_ = (call);                                                                               \
    if (e_ != cudaSuccess) throw ::rta::Failure{RTA_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)}; \
  } while (0)

inline void require(bool ok, const std::string& msg, rta_status code = RTA_E_ASSET) {
  if (!ok) throw Failure{code, msg};
}

// Packed (Q4_K / Q6_K) or dense (F32 / F16 / BF16) exporter formats the engine serves.
inline bool packed_fmt(int f) { return f == kQ4K || f == kQ6K; }
inline bool served_fmt(int f) { return packed_fmt(f) || dense_format(f); }
// Bytes of one row of `cols` coefficients (tiled / panel codes count as their packed format).
inline size_t row_bytes(int fmt, size_t cols) {
  return dense_format(fmt) ? cols * dense_bytes(fmt) : cols / 256 * block_bytes(fmt % 100);
}

template <class T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  void alloc(size_t count) {
    n = count;
    RTA_CUDA(cudaMalloc(&p, std::max<size_t>(1, count) * sizeof(T)));
  }
  void zero(cudaStream_t s) { RTA_CUDA(cudaMemsetAsync(p, 0, std::max<size_t>(1, n) * sizeof(T), s)); }
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};

struct Layer {
  bool full = true;
  uint32_t fi = 0, ri = 0;
  const float* attn_norm = nullptr;
  const float* post_norm = nullptr;
  // full attention
  DevBuf<uint8_t> qkvg;  // [q | k | v | gate] rows, internal (rotary-paired) order
  int qkvg_fmt = kQ4K;
  uint32_t qkvg_rows = 0;
  bool gated = false;
  const uint8_t* o = nullptr;
  int o_fmt = kQ4K;
  uint32_t rotary_out = 0;  // o_proj mode 4: un-pair the attention output
  const float* qnorm = nullptr;
  const float* knorm = nullptr;
  // recurrent
  DevBuf<uint8_t> inproj;  // [q (K) | k (K) | v (S) | z (S)]
  int inproj_fmt = kQ4K;
  uint32_t inproj_rows = 0;
  const uint8_t* out = nullptr;
  int out_fmt = kQ4K;
  const float *wa = nullptr, *wb = nullptr, *a_log = nullptr, *dt_bias = nullptr, *conv_w = nullptr,
              *ssm_norm = nullptr;
  // 16-byte aligned copies [wa H*D | wb H*D | attn_norm D] that the gated-delta
  // kernel stages with bulk copies (the payload only aligns tensors to words)
  DevBuf<float> gate_w;
  // MLP
  const uint8_t *gate = nullptr, *up = nullptr, *down = nullptr;
  int mlp_fmt = kQ4K, down_fmt = kQ4K;
  DevBuf<uint8_t> gate_s, up_s, down_s;  // tensor-parallel mode: this rank's slices (own copies)
  // dense (F32 / F16 / BF16) matrices that sat off a 16-byte boundary in the payload: aligned copies
  std::vector<std::unique_ptr<DevBuf<uint8_t>>> dense_copies;
  // Prefill chunks of a single-sequence handle: panel-order copies of the packed
  // matrices (a: QKV(+gate) / in-projection, b: o / out projection), so the
  // chunk's rows run on the tensor cores; fmt -1 = none (the tiled / dense
  // matrix serves the chunk on the GEMV).
  DevBuf<uint8_t> pc_a, pc_b, pc_gate, pc_up, pc_down;
  int pc_a_fmt = -1, pc_b_fmt = -1, pc_gate_fmt = -1, pc_down_fmt = -1;
};

struct Engine {
  rta_model_spec spec{};
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t capacity = 0, nsplit = 1;
  uint32_t nseq = 1;   // sequences decoded side by side (one token each per step)
  // Tensor-parallel hybrid (rta_model_open_team): every rank holds the residual
  // rows of all nseq sequences, runs the attention / recurrent blocks of its own
  // sequences [z0, z0 + na) only, and a 1/world slice of every MLP (middle rows
  // [f0, f0 + fcount)) and of the vocabulary readout (rows [v0, v0 + vcount)) for
  // all of them; team exchanges after each block keep the residual rows equal
  // on every rank.  Without a team: z0 = 0, na = nseq, whole matrices.
  rta_team* team = nullptr;
  uint32_t z0 = 0, na = 1;
  uint32_t f0 = 0, fcount = 0, v0 = 0, vcount = 0;
  uint32_t xblocks = 0;             // blocks of every team exchange (team_blocks)
  std::vector<uint32_t> row_start;  // [world + 1] first sequence of every rank
  DevBuf<float> delta, partial;     // block outputs of this rank's rows / MLP partial sums, [nseq][D]
  DevBuf<uint8_t> lm_slice;         // this rank's vocabulary rows (GGUF order)
  uint32_t F() const { return team ? fcount : spec.middle_size; }
  uint32_t VL() const { return team ? vcount : spec.vocabulary_size; }
  uint32_t projw = 0;  // floats of one sequence's projection row
  std::vector<uint32_t> hp;  // host copy of the parameter words
  DevBuf<uint32_t> params;
  DevBuf<uint8_t> matrices, basis;
  std::vector<std::unique_ptr<Layer>> layers;
  uint32_t n_full = 0, n_rec = 0;
  const uint8_t* lm = nullptr;
  int lm_fmt = kQ6K;
  DevBuf<uint8_t> lm_tiled;  // the LM head in tiled / panel order (its GGUF rows may double as the embedding)
  // Batched products run on the tensor cores (qgemm.cu) when the handle decodes
  // at least kTcMinSeq sequences: matrices with rows % 128 == 0 are then kept in
  // panel order, the gate / up outputs go to gu (raw, [row][gate | up]) and the
  // down projection's prep applies SwiGLU; tc_ws holds the fp16 activation stages.
  static constexpr uint32_t kTcMinSeq = 16;
  bool tc = false;
  uint32_t panel_matrices = 0;  // matrices kept in panel order (products on the tensor cores)
  DevBuf<float> gu;
  DevBuf<uint8_t> tc_ws;
  const uint8_t* embed = nullptr;
  int embed_fmt = kQ6K;
  const float* out_norm = nullptr;
  // activations
  DevBuf<float> state, proj, qproc, att, gdn, act, inv_freq, part_m, part_z, part_o, scratch_x, scratch_y;
  DevBuf<__half> kcache, vcache;
  bool packet_history = false;  // the reference's history packets instead of fp16 K/V
  DevBuf<uint8_t> pring;        // [full layer][sequence][capacity][packet_bytes(kvh)]
  uint32_t pbytes = 0;
  DevBuf<float> rec, conv;
  DevBuf<Control> ctrl;
  DevBuf<uint32_t> prompt;
  Control* ctrl_host = nullptr;  // pinned mirror [nseq]
  cudaGraphExec_t g_decode = nullptr, g_prefill = nullptr;
  // Debug prefill (worker op 1 with debug = 1): a third graph, captured on first
  // use, that also copies every layer's output row and the final-normed row of
  // the position it processes into cap = [depth + 1][capacity][D] (final rows first).
  cudaGraphExec_t g_prefill_cap = nullptr;
  DevBuf<float> cap;
  // Chunked prefill (single-sequence handles): kChunk prompt positions per graph
  // replay as kChunk rows -- products as one batch (the decode GEMV's exact
  // integer products, 16 rows per weight pass; with RTA_MODEL_TC_PREFILL the
  // tensor cores on panel copies), attention rows over the one ring (each row
  // sees its own causal window), the recurrent layer as a parallel pre-pass and
  // a scan over the rows (its state is sequential).
  static constexpr uint32_t kChunk = 64, kChunkSplits = 2;
  bool chunked = false, token_prefill = false, tc_prefill = false;
  bool split_decode = false;  // RTA_MODEL_SPLIT_ACTIVATIONS: batched decode products take x as two fp16 operands
  bool tc_split = false;      // the products being recorded take x as two fp16 operands
  cudaGraphExec_t g_chunk = nullptr;
  uint32_t kernels_per_chunk = 0;
  DevBuf<float> c_rows, c_proj, c_q, c_att, c_gdn, c_act, c_gu, c_pm, c_pz, c_po, c_gates, c_qk, c_vc;
  DevBuf<uint32_t> c_rowctl;
  DevBuf<uint8_t> c_tcws;
  // Step profile (rta_model_profile_step): while `profiling` is set, record_step
  // puts an event after every launch group of the step it records, labelled
  // with the group's kind and its algorithmic HBM bytes.
  bool profiling = false;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<uint32_t> prof_kind;
  std::vector<double> prof_bytes;
  void mark(uint32_t kind, double bytes, cudaStream_t s) {
    if (!profiling) return;
    cudaEvent_t e = nullptr;
    RTA_CUDA(cudaEventCreate(&e));
    prof_ev.push_back(e);
    prof_kind.push_back(kind);
    prof_bytes.push_back(bytes);
    // External: recorded as an event node of the graph being captured (a plain
    // record inside a capture only orders the capture's streams)
    RTA_CUDA(cudaEventRecordWithFlags(e, s, cudaEventRecordExternal));
  }
  // Algorithmic bytes of one product: the packed weights once, x read, y written
  // (read too when accumulated).
  static double product_bytes(const GemvArgs& a) {
    const int base = a.fmt % 100;  // tiled / panel codes keep the packed format in the last two digits
    const double w = static_cast<double>(a.rows) * row_bytes(base, a.cols) * (a.w1 ? 2.0 : 1.0);
    const double rows_out = static_cast<double>(a.rows) * (a.w1 ? 2.0 : 1.0);
    return w + 4.0 * a.batch * (a.cols + rows_out * (a.epilogue == kAccumulate ? 2.0 : 1.0));
  }
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  uint32_t stops[2] = {0xffffffffu, 0xffffffffu};
  uint32_t position = 0;          // sequence 0's next position (single-sequence API)
  std::vector<uint32_t> positions;  // next position per sequence
  uint32_t kernels_per_decode = 0, kernels_per_prefill = 0;
  double last_gpu_ms = 0.0;
  uint64_t payload_bytes = 0;

  uint32_t D() const { return spec.hidden_size; }
  uint32_t Q() const { return spec.attention_heads * spec.attention_head_dim; }
  uint32_t KVW() const { return spec.kv_heads * spec.attention_head_dim; }
  uint32_t S() const { return spec.state_heads * spec.state_head_dim; }
  uint32_t K() const { return spec.state_key_heads * 128u; }

  // ---------------------------------------------------------------- caches
  // Prefix boundaries, the reply tree and the state address of a
  // single-sequence handle opened with RTA_MODEL_CACHE (cache.h).
  struct Caches {
    HistoryIndex index;
    ReplyTree tree;
    DevBuf<uint32_t> slot_hash;  // [n_full][capacity][row chunks][8] history chunk digests
    DevBuf<uint32_t> cursor;     // [1] history positions digested so far
    DevBuf<uint32_t> partial;    // [kDigestBlocks][8]
    DevBuf<uint32_t> addresses;  // [kMaxOut + 1][8]: slot 0 the state now, slot i + 1 after step i
    DevBuf<uint32_t> slot;       // [1] the digesting decode graph's next address slot
    cudaGraphExec_t g_step = nullptr;  // one decode step and the digest of its result
    uint32_t g_step_stops[2] = {0, 0};  // the stop ids g_step's digest was captured with
    DevBuf<CopySeg> segs;        // the copy list of one save / restore
    uint64_t budget = 0;
    uint32_t epoch = 0;
    // The live sequence: its prompt, the tokens emitted since (a trailing stop
    // id is emitted but never consumed), how many of them the device state has
    // consumed, and the address of the state after all of them.
    std::vector<uint32_t> prefix, gen;
    uint32_t fwd = 0;
    bool ready = false;      // prefix / gen describe the handle's sequence (a cached prefill ran)
    bool prefix_ok = false;  // boundaries may be saved from / restored into the live state
    Key256 address{};
    bool address_ok = false;
    std::vector<std::shared_ptr<HistoryBlock>> attached;  // blocks of the last restored boundary
    uint64_t info[RTA_CACHE_INFO_WORDS] = {};
    double ms[3] = {0.0, 0.0, 0.0};
  };
  std::unique_ptr<Caches> cache;

  ~Engine() {
    if (cache && cache->g_step) cudaGraphExecDestroy(cache->g_step);
    cache.reset();  // stream-ordered frees need the stream
    if (g_decode) cudaGraphExecDestroy(g_decode);
    if (g_prefill) cudaGraphExecDestroy(g_prefill);
    if (g_prefill_cap) cudaGraphExecDestroy(g_prefill_cap);
    if (g_chunk) cudaGraphExecDestroy(g_chunk);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    if (ctrl_host) cudaFreeHost(ctrl_host);
    if (stream) cudaStreamDestroy(stream);
  }

  uint32_t word(size_t i) const {
    require(i < hp.size(), "parameter index out of range: " + std::to_string(i));
    return hp[i];
  }
  const float* pf(uint32_t off, size_t count) const {
    require(static_cast<size_t>(off) + count <= hp.size(), "parameter tensor out of range");
    return reinterpret_cast<const float*>(params.p + off);
  }
  // descriptor i (0 q, 1 k, 2 o, 3 gate, 4 down, 5 up, 6 attn-gate/z, 8 v) of layer l
  struct Desc {
    const uint8_t* ptr;
    int fmt, mode;
  };
  Desc desc(uint32_t l, uint32_t i, size_t rows, size_t cols) const {
    const uint32_t base = 32u + l * 64u;
    const uint32_t field = i == 8u ? base + 32u : base + 9u + 2u * i;
    const uint32_t at = word(base + 27u) + word(field), meta = word(field + 1u);
    Desc d{matrices.p + static_cast<size_t>(at) * 4u, static_cast<int>(meta & 255u), static_cast<int>(meta >> 8)};
    size_t bytes = 0;
    if (served_fmt(d.fmt)) bytes = rows * row_bytes(d.fmt, cols);
    else throw Failure{RTA_E_ASSET, "layer " + std::to_string(l) + " descriptor " + std::to_string(i) +
                                        ": coefficient format " + std::to_string(d.fmt) + " not supported"};
    require(static_cast<size_t>(at) * 4u + bytes <= matrices.n, "matrix descriptor beyond geometry_weights");
    return d;
  }
  uint32_t orig_axis(uint32_t a) const {
    const uint32_t R = spec.rotary_dim;
    return a < R ? (a % 2u) * (R / 2u) + a / 2u : a;
  }
  uint32_t src_row(int mode, uint32_t r) const {
    const uint32_t hd = spec.attention_head_dim;
    switch (mode) {
      case 1: return (r / hd) * (2u * hd) + orig_axis(r % hd);
      case 2: return (r / hd) * (2u * hd) + hd + orig_axis(r % hd);
      case 3: return (r / hd) * hd + orig_axis(r % hd);
      case 5: return r % (spec.state_key_heads * 128u);
      default: return r;
    }
  }
  void gather(uint8_t* dst, const Desc& d, uint32_t rows, uint32_t row_bytes, int mode) {
    std::vector<uint32_t> map(rows);
    for (uint32_t r = 0; r < rows; ++r) map[r] = src_row(mode, r);
    DevBuf<uint32_t> dmap;
    dmap.alloc(rows);
    RTA_CUDA(cudaMemcpyAsync(dmap.p, map.data(), rows * 4u, cudaMemcpyHostToDevice, stream));
    RTA_CUDA(launch_gather_rows(d.ptr, dmap.p, rows, row_bytes, dst, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
  }

  // Tensor-parallel hybrid: this rank's sequences and slices.  The middle
  // dimension is divided in units of 256 (one block column of the down
  // projection) and the vocabulary in units of 128 rows, the first ranks taking
  // one unit more; every rank derives the same split.
  static void split_units(uint32_t total, uint32_t unit, uint32_t world, uint32_t rank, uint32_t& start,
                          uint32_t& count) {
    const uint32_t units = total / unit, base = units / world, extra = units % world;
    start = (rank * base + std::min(rank, extra)) * unit;
    count = (base + (rank < extra ? 1u : 0u)) * unit;
  }
  void setup_team(rta_team* tm, const uint32_t* seq_starts) {
    require(seq_starts != nullptr, "a team handle needs every rank's first sequence", RTA_E_ARG);
    require(team_ready(tm), "the team is not connected", RTA_E_STATE);
    const uint32_t world = team_world(tm), rank = team_rank(tm);
    row_start.assign(seq_starts, seq_starts + world + 1);
    require(row_start[0] == 0 && row_start[world] == nseq, "sequence starts must run from 0 to the sequence count",
            RTA_E_ARG);
    for (uint32_t r = 0; r < world; ++r)
      require(row_start[r + 1] > row_start[r], "every rank needs at least one sequence", RTA_E_ARG);
    require(spec.middle_size % 256 == 0 && spec.middle_size / 256 >= world && spec.vocabulary_size % 128 == 0 &&
                spec.vocabulary_size / 128 >= world,
            "middle size (units of 256) and vocabulary (units of 128) must cover every rank", RTA_E_ARG);
    require(team_capacity_words(tm) >= static_cast<size_t>(nseq) * spec.hidden_size &&
                team_capacity_words(tm) >= 2ull * nseq,
            "the team's exchange capacity must hold sequences x hidden floats", RTA_E_ARG);
    team = tm;
    z0 = row_start[rank];
    na = row_start[rank + 1] - row_start[rank];
    split_units(spec.middle_size, 256u, world, rank, f0, fcount);
    split_units(spec.vocabulary_size, 128u, world, rank, v0, vcount);
  }
  // Copies of this rank's gate / up rows and down-projection columns.
  void slice_mlp(Layer& L) {
    const uint32_t D = this->D(), Ff = spec.middle_size;
    const size_t rg = row_bytes(L.mlp_fmt, D);
    L.gate_s.alloc(static_cast<size_t>(fcount) * rg);
    L.up_s.alloc(static_cast<size_t>(fcount) * rg);
    RTA_CUDA(cudaMemcpyAsync(L.gate_s.p, L.gate + static_cast<size_t>(f0) * rg, L.gate_s.n, cudaMemcpyDeviceToDevice,
                             stream));
    RTA_CUDA(cudaMemcpyAsync(L.up_s.p, L.up + static_cast<size_t>(f0) * rg, L.up_s.n, cudaMemcpyDeviceToDevice,
                             stream));
    const size_t row = row_bytes(L.down_fmt, Ff), width = row_bytes(L.down_fmt, fcount);
    const size_t skip = row_bytes(L.down_fmt, f0);  // f0 is a multiple of 256
    L.down_s.alloc(static_cast<size_t>(D) * width);
    RTA_CUDA(cudaMemcpy2DAsync(L.down_s.p, width, L.down + skip, row, width, D, cudaMemcpyDeviceToDevice, stream));
    L.gate = L.gate_s.p;
    L.up = L.up_s.p;
    L.down = L.down_s.p;
  }

  // Re-lay every GEMV matrix once into the tiled order (same bytes; see
  // launch_tile_weights): layer matrices in place through a scratch buffer,
  // the LM head into its own buffer.  Fails on projections sharing bytes.
  void tile_matrices() {
    const uint32_t D = this->D(), F = this->F();
    struct Job {
      uint8_t* p;
      int fmt;           // packed format of the payload (Q4_K / Q6_K)
      int* tiled_field;  // format field switched to the tiled code afterwards (null: shared with another job)
      uint32_t rows, cols;
      DevBuf<uint8_t>* pc = nullptr;  // prefill-chunk panel copy (single-sequence handles)
      int* pc_fmt = nullptr;
    };
    std::vector<Job> jobs;
    auto mut = [](const uint8_t* q) { return const_cast<uint8_t*>(q); };
    // Dense matrices keep their row-major layout (the dense GEMV streams rows);
    // the ones off a 16-byte boundary get an aligned copy.
    auto add = [&](Layer& L, const uint8_t*& ptr, int fmt, int* field, uint32_t rows, uint32_t cols,
                   DevBuf<uint8_t>* pc, int* pc_fmt) {
      if (!dense_format(fmt)) {
        jobs.push_back({mut(ptr), fmt, field, rows, cols, pc, pc_fmt});
        return;
      }
      if (reinterpret_cast<uintptr_t>(ptr) % 16 == 0) return;
      auto copy = std::make_unique<DevBuf<uint8_t>>();
      copy->alloc(static_cast<size_t>(rows) * row_bytes(fmt, cols));
      RTA_CUDA(cudaMemcpyAsync(copy->p, ptr, copy->n, cudaMemcpyDeviceToDevice, stream));
      ptr = copy->p;
      L.dense_copies.push_back(std::move(copy));
    };
    for (size_t li = 0; li < layers.size(); ++li) {
      Layer& L = *layers[li];
      if (L.full) {
        const uint8_t* q = L.qkvg.p;
        add(L, q, L.qkvg_fmt, &L.qkvg_fmt, L.qkvg_rows, D, &L.pc_a, &L.pc_a_fmt);
        add(L, L.o, L.o_fmt, &L.o_fmt, D, Q(), &L.pc_b, &L.pc_b_fmt);
      } else {
        const uint8_t* q = L.inproj.p;
        add(L, q, L.inproj_fmt, &L.inproj_fmt, L.inproj_rows, D, &L.pc_a, &L.pc_a_fmt);
        add(L, L.out, L.out_fmt, &L.out_fmt, D, S(), &L.pc_b, &L.pc_b_fmt);
      }
      add(L, L.gate, L.mlp_fmt, &L.mlp_fmt, F, D, &L.pc_gate, &L.pc_gate_fmt);
      add(L, L.up, L.mlp_fmt, nullptr, F, D, &L.pc_up, nullptr);  // up shares the gate's format field
      add(L, L.down, L.down_fmt, &L.down_fmt, D, F, &L.pc_down, &L.pc_down_fmt);
    }
    std::vector<std::pair<uintptr_t, size_t>> spans;
    size_t need = 0;
    for (const Job& j : jobs) {
      const size_t bytes = static_cast<size_t>(j.rows) * row_bytes(j.fmt, j.cols);
      const uintptr_t a = reinterpret_cast<uintptr_t>(j.p);
      for (const auto& d : spans)
        require(!(a < d.first + d.second && d.first < a + bytes),
                "two projections share payload bytes; the tiled re-layout needs distinct matrices");
      require(a % 16 == 0, "projection payload not 16-byte aligned");
      spans.push_back({a, bytes});
      need = std::max(need, bytes);
    }
    DevBuf<uint8_t> tmp;
    tmp.alloc(std::max<size_t>(need, 1));
    // gate and up share one format field: both take the panel order only together
    auto panel_ok = [&](uint32_t rows) { return tc && rows % 128u == 0u; };
    if (chunked && tc_prefill)  // panel copies for the prefill chunks, from the GGUF-order bytes (before tiling)
      for (const Job& j : jobs) {
        if (!j.pc || j.rows % 128u) continue;
        j.pc->alloc(static_cast<size_t>(j.rows) * row_bytes(j.fmt, j.cols));
        RTA_CUDA(launch_tile_tc(j.fmt, j.p, j.rows, j.cols, j.pc->p, stream));
        if (j.pc_fmt) *j.pc_fmt = j.fmt + kPanelOffset;
      }
    for (const Job& j : jobs) {
      const size_t bytes = static_cast<size_t>(j.rows) * row_bytes(j.fmt, j.cols);
      if (panel_ok(j.rows))
        RTA_CUDA(launch_tile_tc(j.fmt, j.p, j.rows, j.cols, tmp.p, stream));
      else
        RTA_CUDA(launch_tile_weights(j.fmt, j.p, j.rows, j.cols, tmp.p, stream));
      RTA_CUDA(cudaMemcpyAsync(j.p, tmp.p, bytes, cudaMemcpyDeviceToDevice, stream));
    }
    for (const Job& j : jobs) {
      if (j.tiled_field) *j.tiled_field = j.fmt + (panel_ok(j.rows) ? kPanelOffset : kTiledOffset);
      panel_matrices += panel_ok(j.rows) ? 1u : 0u;
    }
    const size_t lm_bytes = static_cast<size_t>(VL()) * row_bytes(lm_fmt, D);
    lm_tiled.alloc(lm_bytes);
    if (dense_format(lm_fmt)) {  // row-major as exported, in an aligned buffer of its own
      RTA_CUDA(cudaMemcpyAsync(lm_tiled.p, lm, lm_bytes, cudaMemcpyDeviceToDevice, stream));
    } else if (panel_ok(VL())) {
      RTA_CUDA(launch_tile_tc(lm_fmt, lm, VL(), D, lm_tiled.p, stream));
      lm_fmt += kPanelOffset;
      ++panel_matrices;
    } else {
      RTA_CUDA(launch_tile_weights(lm_fmt, lm, VL(), D, lm_tiled.p, stream));
      lm_fmt += kTiledOffset;
    }
    if (lm_slice.p) {  // the tiled copy replaces this rank's GGUF-order rows
      RTA_CUDA(cudaStreamSynchronize(stream));
      cudaFree(lm_slice.p);
      lm_slice.p = nullptr;
      lm_slice.n = 0;
    }
    lm = lm_tiled.p;
    RTA_CUDA(cudaStreamSynchronize(stream));
  }

  void load(const rta_model_spec& sp, const uint32_t* prm, size_t n_params, const void* mat, size_t matrix_bytes,
            const void* bas, size_t basis_bytes, uint32_t cap, uint32_t sequences, uint32_t flags, int dev,
            rta_team* tm = nullptr, const uint32_t* seq_starts = nullptr) {
    spec = sp;
    device = dev;
    require((flags & ~static_cast<uint32_t>(RTA_MODEL_PACKET_HISTORY | RTA_MODEL_TOKEN_PREFILL |
                                            RTA_MODEL_TC_PREFILL | RTA_MODEL_SPLIT_ACTIVATIONS |
                                            RTA_MODEL_CACHE)) == 0,
            "unknown model flags", RTA_E_ARG);
    split_decode = (flags & RTA_MODEL_SPLIT_ACTIVATIONS) != 0;
    token_prefill = (flags & RTA_MODEL_TOKEN_PREFILL) != 0;
    tc_prefill = (flags & RTA_MODEL_TC_PREFILL) != 0;
    packet_history = (flags & RTA_MODEL_PACKET_HISTORY) != 0;
    require(sequences >= 1 && sequences <= 256, "sequences must be 1..256", RTA_E_ARG);
    nseq = sequences;
    na = nseq;
    if (tm) setup_team(tm, seq_starts);
    require(!(flags & RTA_MODEL_CACHE) || (nseq == 1 && !tm), "the caches serve single-sequence handles",
            RTA_E_ARG);
    require(spec.depth >= 1 && spec.depth <= 256, "depth must be 1..256", RTA_E_ARG);
    require(spec.hidden_size % 256 == 0 && spec.middle_size % 256 == 0, "hidden/middle must be multiples of 256",
            RTA_E_ARG);
    require(spec.attention_head_dim == 256 && spec.attention_heads == 4 * spec.kv_heads,
            "this build serves head_dim 256 with 4 query heads per KV head", RTA_E_ARG);
    require(spec.state_head_dim == 128 && spec.state_heads % std::max(1u, spec.state_key_heads) == 0,
            "recurrent heads must be 128 wide", RTA_E_ARG);
    require(spec.rotary_dim % 2 == 0 && spec.rotary_dim <= spec.attention_head_dim, "bad rotary_dim", RTA_E_ARG);
    require(cap >= 1, "capacity must be positive", RTA_E_ARG);
    capacity = cap;
    RTA_CUDA(cudaSetDevice(device));
    RTA_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    RTA_CUDA(cudaEventCreate(&ev0));
    RTA_CUDA(cudaEventCreate(&ev1));
    hp.assign(prm, prm + n_params);
    require(n_params >= 32 + 64ull * spec.depth, "parameter table too short");
    require(hp[0] == spec.depth && hp[2] == spec.middle_size, "parameter header does not match the model spec");
    params.alloc(n_params);
    RTA_CUDA(cudaMemcpyAsync(params.p, prm, n_params * 4, cudaMemcpyDefault, stream));
    matrices.alloc(matrix_bytes);
    RTA_CUDA(cudaMemcpyAsync(matrices.p, mat, matrix_bytes, cudaMemcpyDefault, stream));
    basis.alloc(basis_bytes);
    RTA_CUDA(cudaMemcpyAsync(basis.p, bas, basis_bytes, cudaMemcpyDefault, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
    payload_bytes = n_params * 4ull + matrix_bytes + basis_bytes;

    const uint32_t D = this->D(), hd = spec.attention_head_dim;
    out_norm = pf(word(4), D);
    embed_fmt = static_cast<int>(word(13));
    lm_fmt = static_cast<int>(word(15));
    require(served_fmt(embed_fmt) && served_fmt(lm_fmt),
            "token embedding and output rows must be Q4_K, Q6_K, F32, F16 or BF16");
    const size_t row_e = row_bytes(embed_fmt, D), row_l = row_bytes(lm_fmt, D);
    require(static_cast<size_t>(word(14)) * 4 + row_e * spec.vocabulary_size <= basis_bytes, "token_embd out of range");
    require(static_cast<size_t>(word(16)) * 4 + row_l * spec.vocabulary_size <= basis_bytes, "output rows out of range");
    require(spec.vocabulary_size % 16 == 0, "vocabulary must be a multiple of 16 rows");
    embed = basis.p + static_cast<size_t>(word(14)) * 4;
    lm = basis.p + static_cast<size_t>(word(16)) * 4;

    for (uint32_t l = 0; l < spec.depth; ++l) {
      auto L = std::make_unique<Layer>();
      const uint32_t base = 32u + l * 64u;
      L->full = word(base + 26u) == 1u;
      require(L->full == (spec.layer_kinds[l] == 1), "layer kind disagrees with the parameter table");
      L->attn_norm = pf(word(base), D);
      L->post_norm = pf(word(base + 1u), D);
      if (L->full) {
        L->fi = n_full++;
        const uint32_t Qw = Q(), KV = KVW();
        L->gated = spec.attention_gate != 0;
        Desc dq = desc(l, 0, static_cast<size_t>(Qw) * (L->gated ? 2 : 1), D);
        Desc dk = desc(l, 1, KV, D), dv = desc(l, 8, KV, D);
        Desc dg = L->gated ? desc(l, 6, static_cast<size_t>(Qw) * 2, D) : dq;
        require(dq.fmt == dk.fmt && dq.fmt == dv.fmt && dq.fmt == dg.fmt && served_fmt(dq.fmt),
                "q/k/v (and gate) projections must share one format");
        L->qkvg_fmt = dq.fmt;
        const uint32_t rb = static_cast<uint32_t>(row_bytes(dq.fmt, D));
        L->qkvg_rows = Qw + 2 * KV + (L->gated ? Qw : 0);
        L->qkvg.alloc(static_cast<size_t>(L->qkvg_rows) * rb);
        gather(L->qkvg.p, dq, Qw, rb, dq.mode);
        gather(L->qkvg.p + static_cast<size_t>(Qw) * rb, dk, KV, rb, dk.mode);
        gather(L->qkvg.p + static_cast<size_t>(Qw + KV) * rb, dv, KV, rb, dv.mode);
        if (L->gated) gather(L->qkvg.p + static_cast<size_t>(Qw + 2 * KV) * rb, dg, Qw, rb, dg.mode);
        Desc dO = desc(l, 2, D, Qw);
        L->o = dO.ptr;
        L->o_fmt = dO.fmt;
        L->rotary_out = dO.mode == 4 ? spec.rotary_dim : 0u;
        L->qnorm = pf(word(base + 24u), Qw);
        L->knorm = pf(word(base + 25u), Qw);
        require(word(base + 29u) == spec.rotary_dim, "per-layer rotary_dim disagrees with the spec");
      } else {
        L->ri = n_rec++;
        const uint32_t Kw = K(), Sw = S(), H = spec.state_heads;
        Desc dqkv = desc(l, 0, 2ull * Kw + Sw, D);
        Desc dz = desc(l, 6, Sw, D);
        require(dqkv.fmt == dz.fmt && served_fmt(dqkv.fmt),
                "recurrent qkv and gate projections must share one format");
        const uint32_t rb = static_cast<uint32_t>(row_bytes(dqkv.fmt, D));
        L->inproj_fmt = dqkv.fmt;
        L->inproj_rows = 2 * Kw + 2 * Sw;
        L->inproj.alloc(static_cast<size_t>(L->inproj_rows) * rb);
        RTA_CUDA(cudaMemcpyAsync(L->inproj.p, dqkv.ptr, static_cast<size_t>(2 * Kw + Sw) * rb,
                                 cudaMemcpyDeviceToDevice, stream));
        RTA_CUDA(cudaMemcpyAsync(L->inproj.p + static_cast<size_t>(2 * Kw + Sw) * rb, dz.ptr,
                                 static_cast<size_t>(Sw) * rb, cudaMemcpyDeviceToDevice, stream));
        Desc dO = desc(l, 2, D, Sw);
        L->out = dO.ptr;
        L->out_fmt = dO.fmt;
        const uint32_t at_b = word(base + 27u) + word(base + 35u), at_a = word(base + 27u) + word(base + 36u);
        require((word(base + 39u) & 255u) == kF32 && (word(base + 40u) & 255u) == kF32,
                "recurrent alpha/beta projections must be F32 in this build");
        require((static_cast<size_t>(std::max(at_a, at_b)) * 4 + static_cast<size_t>(H) * D * 4) <= matrices.n,
                "alpha/beta beyond geometry_weights");
        const size_t hd_floats = static_cast<size_t>(H) * D;
        L->gate_w.alloc(2 * hd_floats + D);
        RTA_CUDA(cudaMemcpyAsync(L->gate_w.p, matrices.p + static_cast<size_t>(at_a) * 4, hd_floats * 4,
                                 cudaMemcpyDeviceToDevice, stream));
        RTA_CUDA(cudaMemcpyAsync(L->gate_w.p + hd_floats, matrices.p + static_cast<size_t>(at_b) * 4, hd_floats * 4,
                                 cudaMemcpyDeviceToDevice, stream));
        RTA_CUDA(cudaMemcpyAsync(L->gate_w.p + 2 * hd_floats, L->attn_norm, static_cast<size_t>(D) * 4,
                                 cudaMemcpyDeviceToDevice, stream));
        L->wa = L->gate_w.p;
        L->wb = L->gate_w.p + hd_floats;
        L->dt_bias = pf(word(base + 37u), H);
        L->a_log = pf(word(base + 38u), H);
        L->conv_w = pf(word(base + 34u), 3ull * Sw * 4);
        L->ssm_norm = pf(word(base + 31u), Sw);
      }
      Desc dg = desc(l, 3, spec.middle_size, D), du = desc(l, 5, spec.middle_size, D),
           dd = desc(l, 4, D, spec.middle_size);
      require(dg.fmt == du.fmt && served_fmt(dg.fmt) && served_fmt(dd.fmt),
              "MLP projections must be Q4_K, Q6_K, F32, F16 or BF16 (gate and up alike)");
      L->gate = dg.ptr;
      L->up = du.ptr;
      L->down = dd.ptr;
      L->mlp_fmt = dg.fmt;
      L->down_fmt = dd.fmt;
      if (team) slice_mlp(*L);
      layers.push_back(std::move(L));
    }
    if (team) {  // this rank's vocabulary rows, a contiguous run of the GGUF rows
      const size_t rb = row_bytes(lm_fmt, D);
      lm_slice.alloc(static_cast<size_t>(vcount) * rb);
      RTA_CUDA(cudaMemcpyAsync(lm_slice.p, lm + static_cast<size_t>(v0) * rb, lm_slice.n, cudaMemcpyDeviceToDevice,
                               stream));
      lm = lm_slice.p;
    }
    RTA_CUDA(cudaStreamSynchronize(stream));
    tc = nseq >= kTcMinSeq;
    chunked = nseq == 1 && !team && !token_prefill;
    tile_matrices();

    // activations and state, one row per sequence
    projw = std::max(Q() + 2 * KVW() + Q(), 2 * K() + 2 * S());
    projw = (projw + 3u) / 4u * 4u;  // 16-byte aligned rows
    state.alloc(static_cast<size_t>(nseq) * D);
    proj.alloc(static_cast<size_t>(na) * projw);
    qproc.alloc(static_cast<size_t>(na) * Q());
    att.alloc(static_cast<size_t>(na) * Q());
    gdn.alloc(static_cast<size_t>(na) * std::max(1u, S()));
    act.alloc(static_cast<size_t>(nseq) * F());
    if (team) {
      delta.alloc(static_cast<size_t>(nseq) * D);
      partial.alloc(static_cast<size_t>(nseq) * D);
      delta.zero(stream);
      partial.zero(stream);
      xblocks = team_blocks(static_cast<size_t>(nseq) * D);
    }
    scratch_x.alloc(32ull * std::max(D, spec.middle_size));
    scratch_y.alloc(32ull * std::max(D, spec.middle_size));
    if (tc) {  // raw gate | up rows and the tensor-core activation stages (largest K, largest batch)
      const uint32_t rows = std::max(nseq, 32u);
      gu.alloc(static_cast<size_t>(rows) * 2 * F());
      size_t ws = 0;
      for (uint32_t cols : {D, Q(), std::max(1u, S()), F()})
        if (cols % 256 == 0)
          ws = std::max({ws, tc_workspace_bytes(kQ4KPanel, rows, cols, split_decode),
                         tc_workspace_bytes(kQ6KPanel, rows, cols, split_decode)});
      tc_ws.alloc(ws);
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    // History splits per (sequence, KV head): one sequence needs sms / kvh of them
    // to fill the GPU; many sequences fill it by themselves, and then a few
    // splits (about eight waves of CTAs in all) keep the longest histories' CTAs
    // short next to the ragged mean without paying every split's fixed cost
    // (query load, combine, record, merge) for the short ones.
    // Many sequences (the tensor-core regime; below it a batch keeps the
    // single-sequence arithmetic): splits in proportion to each sequence's history
    // (AttnParams::split_by_length), up to capacity / 2048 of them, so a split
    // covers up to ~2048 positions whatever the history (config 5: 4 splits for
    // the longest histories, 1 for the shortest; measured against 512 / 1024 /
    // 1536 positions per split and against a uniform split count).
    const uint32_t fill = (8u * static_cast<uint32_t>(sms) + spec.kv_heads * na - 1u) / (spec.kv_heads * na);
    // Below that regime both split kernels round a split up to a multiple of 64
    // positions.  One sequence, and packet history (every K/V value decoded on
    // the CUDA cores), get up to capacity / 64 splits, so a decode-length history
    // gives each CTA about 64 positions; a few fp16 sequences keep capacity / 256.
    const uint32_t per_split = packet_history || na == 1 ? 64u : 256u;
    nsplit = nseq >= kTcMinSeq ? std::max(1u, std::min(static_cast<uint32_t>(sms) / spec.kv_heads, capacity / 2048u))
                       : std::max(1u, std::min({static_cast<uint32_t>(sms) / spec.kv_heads, capacity / per_split, fill}));
    const size_t recs = static_cast<size_t>(na) * spec.kv_heads * nsplit * 4;
    part_m.alloc(recs);
    part_z.alloc(recs);
    part_o.alloc(recs * hd);
    if (chunked) {
      const size_t C = kChunk;  // chunk buffers (the tensor-core workspace only with panel copies)
      c_rows.alloc(C * D);
      c_proj.alloc(C * projw);
      c_q.alloc(C * Q());
      c_att.alloc(C * Q());
      c_gdn.alloc(C * std::max(1u, S()));
      c_act.alloc(C * F());
      c_gu.alloc(C * 2 * F());
      const size_t crecs = C * spec.kv_heads * kChunkSplits * 4;
      c_pm.alloc(crecs);
      c_pz.alloc(crecs);
      c_po.alloc(crecs * hd);
      c_rowctl.alloc(2 * C);
      c_gates.alloc(C * std::max(1u, spec.state_heads) * 2);
      c_qk.alloc(C * std::max(1u, spec.state_heads) * 2 * 128);
      c_vc.alloc(C * std::max(1u, spec.state_heads) * 128);
      size_t ws = 0;
      for (uint32_t cols : {D, Q(), std::max(1u, S()), F()})
        if (cols % 256 == 0)
          ws = std::max({ws, tc_workspace_bytes(kQ4KPanel, kChunk, cols, true),
                         tc_workspace_bytes(kQ6KPanel, kChunk, cols, true)});
      c_tcws.alloc(ws);
    }
    // [layer][sequence] x per-sequence blocks
    pbytes = packet_bytes(spec.kv_heads);
    if (packet_history) {
      pring.alloc(static_cast<size_t>(std::max(1u, n_full)) * na * capacity * pbytes);
      kcache.alloc(1);
      vcache.alloc(1);
    } else {
      kcache.alloc(static_cast<size_t>(std::max(1u, n_full)) * na * spec.kv_heads * capacity * hd);
      vcache.alloc(kcache.n);
    }
    rec.alloc(static_cast<size_t>(std::max(1u, n_rec)) * na * spec.state_heads * 128 * 128);
    conv.alloc(static_cast<size_t>(std::max(1u, n_rec)) * na * 2 * 3 * S() * 3);
    ctrl.alloc(nseq);
    prompt.alloc(static_cast<size_t>(nseq) * capacity);
    positions.assign(nseq, 0u);
    RTA_CUDA(cudaMallocHost(&ctrl_host, sizeof(Control) * nseq));
    std::vector<float> freq(hd / 2, 0.f);
    for (uint32_t p = 0; p < spec.rotary_dim / 2u; ++p)
      freq[p] = std::pow(spec.rope_theta, -static_cast<float>(p) / static_cast<float>(spec.rotary_dim / 2u));
    inv_freq.alloc(hd / 2);
    RTA_CUDA(cudaMemcpyAsync(inv_freq.p, freq.data(), freq.size() * 4, cudaMemcpyHostToDevice, stream));
    if (flags & RTA_MODEL_CACHE) open_caches();
    reset_sequence();
    capture();
  }

  void open_caches() {
    cache = std::make_unique<Caches>();
    Caches& c = *cache;
    const uint32_t row_words = packet_history ? pbytes / 4u : spec.kv_heads * spec.attention_head_dim;
    const uint32_t chunks = (row_words + kRowChunk - 1u) / kRowChunk;
    c.slot_hash.alloc(static_cast<size_t>(std::max(1u, n_full)) * capacity * chunks * 8u);
    c.cursor.alloc(1);
    c.partial.alloc(static_cast<size_t>(kDigestBlocks) * 8u);
    c.addresses.alloc((kMaxOut + 1ull) * 8u);
    c.slot.alloc(1);
    const size_t per_block = std::max(1u, n_full) * (packet_history ? 1ull : 2ull * spec.kv_heads);
    c.segs.alloc((capacity / 16ull + 2ull) * per_block);
    size_t free_b = 0, total_b = 0;
    RTA_CUDA(cudaMemGetInfo(&free_b, &total_b));
    c.budget = std::min<uint64_t>(8ull << 30, free_b / 4u);
  }

  void reset_sequence() {
    if (cache) cache->cursor.zero(stream);  // every history row is digested again
    ctrl.zero(stream);
    rec.zero(stream);
    conv.zero(stream);
    state.zero(stream);
    position = 0;
    std::fill(positions.begin(), positions.end(), 0u);
    RTA_CUDA(cudaStreamSynchronize(stream));
  }

  // One product: panel formats run on the tensor cores, the others on the GEMV.
  cudaError_t matmul(const GemvArgs& a, cudaStream_t s, DevBuf<uint8_t>* ws = nullptr) {
    if (a.fmt != kQ4KPanel && a.fmt != kQ6KPanel) return launch_gemv(a, s);
    if (!ws) ws = &tc_ws;
    TcGemmArgs t;
    t.fmt = a.fmt;
    t.w0 = a.w0;
    t.w1 = a.w1;
    t.rows = a.rows;
    t.cols = a.cols;
    t.x = a.x;
    t.x_stride = a.x_stride ? a.x_stride : a.cols;
    t.batch = a.batch;
    t.prologue = a.prologue;
    t.norm_w = a.norm_w;
    t.eps = a.eps;
    t.z = a.z;
    t.z_stride = a.z_stride;
    t.epilogue = a.epilogue;
    t.y = a.y;
    t.y_stride = a.y_stride ? a.y_stride : a.rows;
    t.argmax = a.argmax;
    t.argmax_step = a.argmax_step;
    t.err = a.err;
    t.running = a.running;
    t.running_step = a.running_step;
    t.xb = ws->p;
    t.xb_bytes = ws->n;
    t.pdl = a.pdl;
    t.split = tc_split;
    return launch_tc_gemm(t, s);
  }

  // SwiGLU MLP: `g` (gate / up with the kSwiGLU epilogue into g.y = the
  // activation rows) then `dn` (down, reading them).  Panel-format gate / up
  // write the raw gate | up rows to gu instead; a panel-format down then applies
  // SwiGLU in its own prep unless the caller wants the activation rows too,
  // otherwise they are formed from gu first.
  void mlp_pair(GemvArgs g, GemvArgs dn, bool need_act, cudaStream_t s, float* gu_rows = nullptr,
                DevBuf<uint8_t>* ws = nullptr) {
    const uint32_t F = g.rows;
    if (!gu_rows) gu_rows = gu.p;
    const bool gpanel = g.fmt == kQ4KPanel || g.fmt == kQ6KPanel;
    const bool dpanel = dn.fmt == kQ4KPanel || dn.fmt == kQ6KPanel;
    if (!gpanel) {
      RTA_CUDA(launch_gemv(g, s));
      mark(RTA_PROF_GATE_UP, product_bytes(g), s);
      RTA_CUDA(matmul(dn, s, ws));
      mark(RTA_PROF_DOWN, product_bytes(dn), s);
      return;
    }
    float* act_rows = g.y;
    const uint32_t act_stride = g.y_stride ? g.y_stride : F;
    g.epilogue = kStore;
    g.y = gu_rows;
    g.y_stride = 2 * F;  // matrix 1 (up) rows follow matrix 0 (gate) rows
    RTA_CUDA(matmul(g, s, ws));
    mark(RTA_PROF_GATE_UP, product_bytes(g), s);
    if (dpanel && !need_act) {
      dn.prologue = kSwiGLUIn;
      dn.x = gu_rows;
      dn.z = gu_rows + F;
      dn.x_stride = 2 * F;
      dn.z_stride = 2 * F;
    } else {
      RTA_CUDA(launch_swiglu_rows(gu_rows, g.batch, F, 2 * F, act_rows, act_stride, s));
    }
    RTA_CUDA(matmul(dn, s, ws));
    mark(RTA_PROF_DOWN, product_bytes(dn), s);
  }

  // Team mode: every rank's attention / recurrent block outputs (its own rows of
  // delta) are added to the residual rows on every rank; returns launches made.
  uint32_t gather_block_outputs(cudaStream_t s) {
    if (!team) return 0;
    RTA_CUDA(team_gather_add(team, delta.p, state.p, D(), row_start.data(), xblocks, s, &ctrl.p->running,
                             static_cast<uint32_t>(sizeof(Control) / 4)));
    mark(RTA_PROF_EXCHANGE, 4.0 * nseq * D(), s);
    return 1;
  }

  // ---------------------------------------------------------- step recording
  uint32_t record_step(bool decode, bool capture_rows = false) {
    const cudaStream_t s = stream;
    uint32_t n = 0;
    tc_split = split_decode;
    Control* c = ctrl.p;
    const uint32_t* running = &c->running;
    // this rank's sequences (all of them without a team): attention / recurrent blocks
    Control* cl = c + z0;
    const uint32_t* running_l = &cl->running;
    float* state_l = state.p + static_cast<size_t>(z0) * this->D();
    const uint32_t D = this->D(), F = this->F(), hd = spec.attention_head_dim;
    const uint32_t cstep = static_cast<uint32_t>(sizeof(Control) / 4);  // u32 between sequences' control words
    static_assert(sizeof(Control) % 8 == 0, "control blocks must keep 8-byte alignment");
    mark(RTA_PROF_START, 0.0, s);
    if (decode) {
      GemvArgs r;
      r.fmt = lm_fmt;
      r.w0 = lm;
      r.rows = VL();
      r.cols = D;
      r.x = state.p;
      r.prologue = kRmsNorm;
      r.norm_w = out_norm;
      r.eps = spec.norm_epsilon;
      r.batch = nseq;
      r.x_stride = D;
      r.argmax = &c->argkey;
      r.argmax_step = static_cast<uint32_t>(sizeof(Control) / 8);
      r.err = &c->err;
      r.running = running;
      r.running_step = cstep;
      r.pdl = true;
      RTA_CUDA(matmul(r, s));
      mark(RTA_PROF_READOUT, product_bytes(r) - 4.0 * r.batch * r.rows, s);  // logits are not stored
      ++n;
      if (team) {  // the best row of every rank's vocabulary slice -> the global best, in the control blocks
        RTA_CUDA(team_allmax_keys(team, &c->argkey, nseq, static_cast<uint32_t>(sizeof(Control) / 8), v0, xblocks, s));
        mark(RTA_PROF_EXCHANGE, static_cast<double>(nseq) * 8.0 * team_world(team), s);
        ++n;
      }
    }
    EmbedParams e;
    e.table = embed;
    e.fmt = embed_fmt;
    e.D = D;
    e.row_bytes = static_cast<uint32_t>(row_bytes(embed_fmt, D));
    e.vocab = spec.vocabulary_size;
    e.ctrl = c;
    e.prompt = prompt.p;
    e.prompt_stride = capacity;
    e.nseq = nseq;
    e.mode = decode ? kEmbedDecode : kEmbedPrefill;
    e.state = state.p;
    RTA_CUDA(launch_embed(e, s, true));
    mark(RTA_PROF_EMBED, static_cast<double>(nseq) * (e.row_bytes + 4.0 * D), s);
    ++n;
    for (size_t li = 0; li < layers.size(); ++li) {
      Layer& L = *layers[li];
      if (L.full) {
        GemvArgs g;
        g.fmt = L.qkvg_fmt;
        g.w0 = L.qkvg.p;
        g.rows = L.qkvg_rows;
        g.cols = D;
        g.x = state_l;
        g.prologue = kRmsNorm;
        g.norm_w = L.attn_norm;
        g.eps = spec.norm_epsilon;
        g.y = proj.p;
        g.batch = na;
        g.x_stride = D;
        g.y_stride = projw;
        g.running = running_l;
        g.running_step = cstep;
        g.err = &cl->err;
        g.pdl = true;
        RTA_CUDA(matmul(g, s));
        mark(RTA_PROF_QKV, product_bytes(g), s);
        PrepParams pp;
        pp.qkvg = proj.p;
        pp.qnorm = L.qnorm;
        pp.knorm = L.knorm;
        pp.inv_freq = inv_freq.p;
        pp.eps = spec.norm_epsilon;
        pp.heads = spec.attention_heads;
        pp.kvh = spec.kv_heads;
        pp.hd = hd;
        pp.group = spec.attention_heads / spec.kv_heads;
        pp.rotary = spec.rotary_dim;
        pp.qk_norm = spec.qk_norm;
        pp.q_width = Q();
        pp.kv_width = KVW();
        pp.qout = qproc.p;
        const size_t seq_kv = static_cast<size_t>(spec.kv_heads) * capacity * hd;
        const size_t layer_kv = seq_kv * na;
        pp.kcache = kcache.p + L.fi * layer_kv;
        pp.vcache = vcache.p + L.fi * layer_kv;
        pp.capacity = capacity;
        pp.pos = &cl->pos_cur;
        pp.running = running_l;
        pp.nseq = na;
        pp.ctrl_step = cstep;
        pp.qkvg_seq = projw;
        const size_t layer_pkt = static_cast<size_t>(na) * capacity * pbytes;
        if (packet_history) pp.packets = pring.p + L.fi * layer_pkt;
        RTA_CUDA(launch_attn_prep(pp, s, true));
        mark(RTA_PROF_PREP, static_cast<double>(na) * 4.0 * (L.qkvg_rows + Q()) +
                                static_cast<double>(na) * (packet_history ? pbytes : 4.0 * KVW()), s);
        AttnParams ap;
        ap.q = qproc.p;
        ap.k = pp.kcache;
        ap.v = pp.vcache;
        ap.q_seq_stride = Q();
        ap.seq_stride = seq_kv;
        if (packet_history) {
          ap.packets = pp.packets;
          ap.packet_seq_stride = static_cast<size_t>(capacity) * pbytes;
          ap.packet_stride = pbytes;
        }
        ap.kv_stride = static_cast<size_t>(capacity) * hd;
        ap.pos_stride = hd;
        ap.heads = spec.attention_heads;
        ap.kvh = spec.kv_heads;
        ap.hd = hd;
        ap.capacity = capacity;
        ap.pos = &cl->pos_cur;
        ap.ctrl_step = cstep;
        ap.gate = L.gated ? proj.p + Q() + 2 * KVW() : nullptr;
        ap.gate_seq_stride = projw;
        ap.out = att.p;
        ap.out_seq_stride = Q();
        ap.rotary_out = L.rotary_out;
        ap.part_m = part_m.p;
        ap.part_z = part_z.p;
        ap.part_o = part_o.p;
        ap.err = &cl->err;
        ap.running = running_l;
        ap.split_by_length = nseq >= kTcMinSeq ? 1u : 0u;
        RTA_CUDA(launch_attention(ap, nsplit, na, true, s));
        mark(RTA_PROF_ATTENTION, attention_bytes(), s);
        GemvArgs o;
        o.fmt = L.o_fmt;
        o.w0 = L.o;
        o.rows = D;
        o.cols = Q();
        o.x = att.p;
        o.epilogue = team ? kStore : kAccumulate;
        o.y = team ? delta.p + static_cast<size_t>(z0) * D : state.p;
        o.batch = na;
        o.x_stride = Q();
        o.y_stride = D;
        o.running = running_l;
        o.running_step = cstep;
        o.err = &cl->err;
        o.pdl = true;
        RTA_CUDA(matmul(o, s));
        mark(RTA_PROF_O_PROJ, product_bytes(o), s);
        n += 5;
        n += gather_block_outputs(s);
      } else {
        GemvArgs g;
        g.fmt = L.inproj_fmt;
        g.w0 = L.inproj.p;
        g.rows = L.inproj_rows;
        g.cols = D;
        g.x = state_l;
        g.prologue = kRmsNorm;
        g.norm_w = L.attn_norm;
        g.eps = spec.norm_epsilon;
        g.y = proj.p;
        g.batch = na;
        g.x_stride = D;
        g.y_stride = projw;
        g.running = running_l;
        g.running_step = cstep;
        g.err = &cl->err;
        g.pdl = true;
        RTA_CUDA(matmul(g, s));
        mark(RTA_PROF_IN_PROJ, product_bytes(g), s);
        GdnParams gp;
        gp.x = state_l;
        gp.attn_norm = L.gate_w.p + 2ull * spec.state_heads * D;  // aligned copy of L.attn_norm
        gp.eps = spec.norm_epsilon;
        gp.wa = L.wa;
        gp.wb = L.wb;
        gp.a_log = L.a_log;
        gp.dt_bias = L.dt_bias;
        gp.proj = proj.p;
        gp.conv_w = L.conv_w;
        gp.conv_seq = static_cast<size_t>(2) * 3 * S() * 3;
        gp.rec_seq = static_cast<size_t>(spec.state_heads) * 128 * 128;
        gp.conv_state = conv.p + static_cast<size_t>(L.ri) * na * gp.conv_seq;
        gp.rec = rec.p + static_cast<size_t>(L.ri) * na * gp.rec_seq;
        gp.proj_seq = projw;
        gp.nseq = na;
        gp.ctrl_step = cstep;
        gp.out = gdn.p;
        gp.D = D;
        gp.H = spec.state_heads;
        gp.KH = spec.state_key_heads;
        gp.pos = &cl->pos_cur;
        gp.err = &cl->err;
        gp.err_step = cstep;
        gp.running = running_l;
        RTA_CUDA(launch_gdn(gp, s, true));
        mark(RTA_PROF_GATED_DELTA, static_cast<double>(running_sequences()) *
                                       (8.0 * spec.state_heads * 128 * 128 + 4.0 * (2 * K() + 2 * S() + 2 * D)), s);
        GemvArgs o;
        o.fmt = L.out_fmt;
        o.w0 = L.out;
        o.rows = D;
        o.cols = S();
        o.x = gdn.p;
        o.x_stride = S();
        o.batch = na;
        o.prologue = kHeadGate;
        o.z = proj.p + 2 * K() + S();
        o.z_stride = projw;
        o.norm_w = L.ssm_norm;
        o.eps = spec.norm_epsilon;
        o.epilogue = team ? kStore : kAccumulate;
        o.y = team ? delta.p + static_cast<size_t>(z0) * D : state.p;
        o.y_stride = D;
        o.running = running_l;
        o.running_step = cstep;
        o.err = &cl->err;
        o.pdl = true;
        RTA_CUDA(matmul(o, s));
        mark(RTA_PROF_OUT_PROJ, product_bytes(o), s);
        n += 3;
        n += gather_block_outputs(s);
      }
      GemvArgs gu;
      gu.fmt = L.mlp_fmt;
      gu.w0 = L.gate;
      gu.w1 = L.up;
      gu.rows = F;
      gu.cols = D;
      gu.x = state.p;
      gu.prologue = kRmsNorm;
      gu.norm_w = L.post_norm;
      gu.eps = spec.norm_epsilon;
      gu.epilogue = kSwiGLU;
      gu.y = act.p;
      gu.batch = nseq;
      gu.x_stride = D;
      gu.y_stride = F;
      gu.running = running;
      gu.running_step = cstep;
      gu.err = &c->err;
      gu.pdl = true;
      GemvArgs dn;
      dn.fmt = L.down_fmt;
      dn.w0 = L.down;
      dn.rows = D;
      dn.cols = F;
      dn.x = act.p;
      dn.epilogue = team ? kStore : kAccumulate;
      dn.y = team ? partial.p : state.p;
      dn.batch = nseq;
      dn.x_stride = F;
      dn.y_stride = D;
      dn.running = running;
      dn.running_step = cstep;
      dn.err = &c->err;
      dn.pdl = true;
      mlp_pair(gu, dn, false, s);
      n += 2;
      if (team) {  // residual + the partial down projections of every rank, in rank order
        // two-phase (reduce-scatter + all-gather) between ranks: each rank sends
        // 2 (world - 1) / world of its partial rows instead of world - 1 copies
        // (rows of sequences that sat the step out are left alone: their products wrote nothing)
        if (team_world(team) >= 2)
          RTA_CUDA(team_allreduce2(team, partial.p, state.p, state.p, static_cast<size_t>(nseq) * D, xblocks, s,
                                   running, cstep, D));
        else
          RTA_CUDA(team_allreduce(team, partial.p, state.p, state.p, static_cast<size_t>(nseq) * D, xblocks, s,
                                  running, cstep, D));
        mark(RTA_PROF_EXCHANGE, 4.0 * nseq * D * team_world(team), s);
        ++n;
      }
      if (capture_rows) {
        CaptureParams cp;
        cp.state = state.p;
        cp.dst = cap.p + (li + 1) * static_cast<size_t>(capacity) * D;
        cp.ctrl = c;
        cp.D = D;
        cp.capacity = capacity;
        RTA_CUDA(launch_capture_row(cp, s, true));
        ++n;
      }
    }
    if (capture_rows) {  // the final-normed row (op 1 index 2), what the reference's debug prefill returns
      CaptureParams cp;
      cp.state = state.p;
      cp.dst = cap.p;
      cp.ctrl = c;
      cp.norm_w = out_norm;
      cp.eps = spec.norm_epsilon;
      cp.D = D;
      cp.capacity = capacity;
      RTA_CUDA(launch_capture_row(cp, s, true));
      ++n;
    }
    return n;
  }

  // One prefill chunk of a single-sequence handle: kChunk consecutive prompt
  // positions from the control block's pos_next (rows past the prompt sit out).
  uint32_t record_chunk() {
    tc_split = true;  // prefill chunk products on the tensor cores carry x exactly (two fp16 operands)
    const cudaStream_t s = stream;
    uint32_t n = 0;
    Control* c = ctrl.p;
    const uint32_t D = this->D(), F = this->F(), hd = spec.attention_head_dim, C = kChunk;
    const uint32_t* rpos = c_rowctl.p;       // row r: position at rpos[2r]
    const uint32_t* rlive = c_rowctl.p + 1;  // row r: live at rlive[2r]
    ChunkParams cp;
    cp.table = embed;
    cp.fmt = embed_fmt;
    cp.D = D;
    cp.row_bytes = static_cast<uint32_t>(row_bytes(embed_fmt, D));
    cp.vocab = spec.vocabulary_size;
    cp.C = C;
    cp.ctrl = c;
    cp.prompt = prompt.p;
    cp.rowctl = c_rowctl.p;
    cp.rows = c_rows.p;
    cp.state = state.p;
    RTA_CUDA(launch_chunk_begin(cp, s, true));
    ++n;
    // the chunk's products: the panel copy when the matrix has one, else the decode matrix
    auto product = [&](const uint8_t* pc, int pc_fmt, const uint8_t* w, int fmt) {
      GemvArgs a;
      a.fmt = pc_fmt >= 0 ? pc_fmt : fmt;
      a.w0 = pc_fmt >= 0 ? pc : w;
      a.batch = C;
      a.running = rlive;
      a.running_step = 2;
      a.err = &c->err;
      a.pdl = true;
      return a;
    };
    for (size_t li = 0; li < layers.size(); ++li) {
      Layer& L = *layers[li];
      if (L.full) {
        GemvArgs g = product(L.pc_a.p, L.pc_a_fmt, L.qkvg.p, L.qkvg_fmt);
        g.rows = L.qkvg_rows;
        g.cols = D;
        g.x = c_rows.p;
        g.x_stride = D;
        g.prologue = kRmsNorm;
        g.norm_w = L.attn_norm;
        g.eps = spec.norm_epsilon;
        g.y = c_proj.p;
        g.y_stride = projw;
        RTA_CUDA(matmul(g, s, &c_tcws));
        PrepParams pp;
        pp.qkvg = c_proj.p;
        pp.qnorm = L.qnorm;
        pp.knorm = L.knorm;
        pp.inv_freq = inv_freq.p;
        pp.eps = spec.norm_epsilon;
        pp.heads = spec.attention_heads;
        pp.kvh = spec.kv_heads;
        pp.hd = hd;
        pp.group = spec.attention_heads / spec.kv_heads;
        pp.rotary = spec.rotary_dim;
        pp.qk_norm = spec.qk_norm;
        pp.q_width = Q();
        pp.kv_width = KVW();
        pp.qout = c_q.p;
        const size_t layer_kv = static_cast<size_t>(spec.kv_heads) * capacity * hd;  // one sequence
        pp.kcache = kcache.p + L.fi * layer_kv;
        pp.vcache = vcache.p + L.fi * layer_kv;
        pp.capacity = capacity;
        pp.pos = rpos;
        pp.running = rlive;
        pp.nseq = C;
        pp.ctrl_step = 2;
        pp.qkvg_seq = projw;
        pp.ring_seq = 0;  // every row writes the sequence's one ring
        if (packet_history) pp.packets = pring.p + L.fi * static_cast<size_t>(capacity) * pbytes;
        RTA_CUDA(launch_attn_prep(pp, s, true));
        AttnParams ap;
        ap.q = c_q.p;
        ap.k = pp.kcache;
        ap.v = pp.vcache;
        ap.q_seq_stride = Q();
        ap.seq_stride = 0;
        if (packet_history) {
          ap.packets = pp.packets;
          ap.packet_seq_stride = 0;
          ap.packet_stride = pbytes;
        }
        ap.kv_stride = static_cast<size_t>(capacity) * hd;
        ap.pos_stride = hd;
        ap.heads = spec.attention_heads;
        ap.kvh = spec.kv_heads;
        ap.hd = hd;
        ap.capacity = capacity;
        ap.pos = rpos;
        ap.ctrl_step = 2;
        ap.gate = L.gated ? c_proj.p + Q() + 2 * KVW() : nullptr;
        ap.gate_seq_stride = projw;
        ap.out = c_att.p;
        ap.out_seq_stride = Q();
        ap.rotary_out = L.rotary_out;
        ap.part_m = c_pm.p;
        ap.part_z = c_pz.p;
        ap.part_o = c_po.p;
        ap.err = &c->err;
        ap.running = rlive;
        RTA_CUDA(launch_attention(ap, kChunkSplits, C, true, s));
        GemvArgs o = product(L.pc_b.p, L.pc_b_fmt, L.o, L.o_fmt);
        o.rows = D;
        o.cols = Q();
        o.x = c_att.p;
        o.x_stride = Q();
        o.epilogue = kAccumulate;
        o.y = c_rows.p;
        o.y_stride = D;
        RTA_CUDA(matmul(o, s, &c_tcws));
        n += 5;
      } else {
        GemvArgs g = product(L.pc_a.p, L.pc_a_fmt, L.inproj.p, L.inproj_fmt);
        g.rows = L.inproj_rows;
        g.cols = D;
        g.x = c_rows.p;
        g.x_stride = D;
        g.prologue = kRmsNorm;
        g.norm_w = L.attn_norm;
        g.eps = spec.norm_epsilon;
        g.y = c_proj.p;
        g.y_stride = projw;
        RTA_CUDA(matmul(g, s, &c_tcws));
        ++n;
        // the recurrent rows: a parallel pre-pass (gates, convolution, norms of
        // every row), then a scan of the rows in order on register-held state
        GdnChunkParams gc;
        GdnParams& gp = gc.g;
        gp.x = c_rows.p;
        gp.attn_norm = L.gate_w.p + 2ull * spec.state_heads * D;
        gp.eps = spec.norm_epsilon;
        gp.wa = L.wa;
        gp.wb = L.wb;
        gp.a_log = L.a_log;
        gp.dt_bias = L.dt_bias;
        gp.proj = c_proj.p;
        gp.proj_seq = projw;
        gp.conv_w = L.conv_w;
        gp.conv_seq = static_cast<size_t>(2) * 3 * S() * 3;
        gp.rec_seq = static_cast<size_t>(spec.state_heads) * 128 * 128;
        gp.conv_state = conv.p + static_cast<size_t>(L.ri) * gp.conv_seq;
        gp.rec = rec.p + static_cast<size_t>(L.ri) * gp.rec_seq;
        gp.out = c_gdn.p;
        gp.D = D;
        gp.H = spec.state_heads;
        gp.KH = spec.state_key_heads;
        gp.err = &c->err;
        gc.rowctl = c_rowctl.p;
        gc.C = C;
        gc.gates = c_gates.p;
        gc.qk = c_qk.p;
        gc.vc = c_vc.p;
        RTA_CUDA(launch_gdn_chunk(gc, s, true));
        n += 2;
        GemvArgs o = product(L.pc_b.p, L.pc_b_fmt, L.out, L.out_fmt);
        o.rows = D;
        o.cols = S();
        o.x = c_gdn.p;
        o.x_stride = S();
        o.prologue = kHeadGate;
        o.z = c_proj.p + 2 * K() + S();
        o.z_stride = projw;
        o.norm_w = L.ssm_norm;
        o.eps = spec.norm_epsilon;
        o.epilogue = kAccumulate;
        o.y = c_rows.p;
        o.y_stride = D;
        RTA_CUDA(matmul(o, s, &c_tcws));
        ++n;
      }
      GemvArgs gu = product(L.pc_gate.p, L.pc_gate_fmt, L.gate, L.mlp_fmt);
      gu.w1 = L.pc_gate_fmt >= 0 ? L.pc_up.p : L.up;
      gu.rows = F;
      gu.cols = D;
      gu.x = c_rows.p;
      gu.x_stride = D;
      gu.prologue = kRmsNorm;
      gu.norm_w = L.post_norm;
      gu.eps = spec.norm_epsilon;
      gu.epilogue = kSwiGLU;
      gu.y = c_act.p;
      gu.y_stride = F;
      GemvArgs dn = product(L.pc_down.p, L.pc_down_fmt, L.down, L.down_fmt);
      dn.rows = D;
      dn.cols = F;
      dn.x = c_act.p;
      dn.x_stride = F;
      dn.epilogue = kAccumulate;
      dn.y = c_rows.p;
      dn.y_stride = D;
      mlp_pair(gu, dn, false, s, c_gu.p, &c_tcws);
      n += 2;
    }
    RTA_CUDA(launch_chunk_end(cp, s, true));
    return n + 1;
  }

  void capture() {
    if (chunked) {
      cudaGraph_t graph = nullptr;
      RTA_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
      try {
        record_chunk();
      } catch (...) {
        cudaStreamEndCapture(stream, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
      }
      RTA_CUDA(cudaStreamEndCapture(stream, &graph));
      size_t nodes = 0;
      cudaGraphGetNodes(graph, nullptr, &nodes);
      kernels_per_chunk = static_cast<uint32_t>(nodes);
      const cudaError_t e = cudaGraphInstantiate(&g_chunk, graph, 0);
      cudaGraphDestroy(graph);
      RTA_CUDA(e);
    }
    for (int mode = 0; mode < 2; ++mode) {
      uint32_t n = 0;
      cudaGraphExec_t exec = instantiate_step(mode == 1, false, &n);
      if (mode == 1) {
        g_decode = exec;
        kernels_per_decode = n;
      } else {
        g_prefill = exec;
        kernels_per_prefill = n;
      }
    }
  }

  cudaGraphExec_t instantiate_step(bool decode, bool capture_rows, uint32_t* launches) {
    {
      cudaGraph_t graph = nullptr;
      RTA_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
      uint32_t n = 0;
      try {
        n = record_step(decode, capture_rows);
      } catch (...) {
        cudaStreamEndCapture(stream, &graph);
        if (graph) cudaGraphDestroy(graph);
        throw;
      }
      RTA_CUDA(cudaStreamEndCapture(stream, &graph));
      size_t nodes = 0;
      cudaGraphGetNodes(graph, nullptr, &nodes);  // launches per replay (batched GEMVs may split)
      n = static_cast<uint32_t>(nodes);
      cudaGraphExec_t exec = nullptr;
      const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      RTA_CUDA(e);
      if (launches) *launches = n;
      return exec;
    }
  }

  // Sequences that take part in the next step (host mirror of the positions).
  uint32_t running_sequences() const {
    uint32_t r = 0;
    for (uint32_t z = z0; z < z0 + na; ++z) r += positions[z] > 0 ? 1u : 0u;
    return r;
  }
  // Algorithmic bytes of one full layer's attention in the next step: every
  // visible history position of every running sequence once (K and V), plus
  // q, the gate rows and the output.
  double attention_bytes() const {
    const double per_pos = packet_history ? static_cast<double>(pbytes) : 4.0 * KVW();
    double b = 0.0;
    for (uint32_t z = z0; z < z0 + na; ++z)
      if (positions[z] > 0) b += per_pos * std::min(positions[z] + 1u, capacity) + 12.0 * Q();
    return b;
  }

  // One decode step of every sequence through a graph that has an event after
  // every launch group; returns per group its kind, device time and
  // algorithmic bytes.  Events between the launches remove the programmatic
  // overlap of consecutive kernels, so each group is timed on its own.
  void profile_step(uint32_t* kinds, double* ms, double* bytes, size_t cap_groups, size_t* n_groups) {
    bool any = false;
    for (uint32_t z = 0; z < nseq; ++z) {
      ctrl_host[z].running = positions[z] > 0 ? 1u : 0u;
      ctrl_host[z].n_out = 0u;
      ctrl_host[z].stops[0] = stops[0];
      ctrl_host[z].stops[1] = stops[1];
      any = any || positions[z] > 0;
    }
    require(any, "prefill before profiling a decode step", RTA_E_STATE);
    profiling = true;
    cudaGraphExec_t exec = nullptr;
    try {
      exec = instantiate_step(true, false, nullptr);
    } catch (...) {
      profiling = false;
      for (cudaEvent_t e : prof_ev) cudaEventDestroy(e);
      prof_ev.clear(), prof_kind.clear(), prof_bytes.clear();
      throw;
    }
    profiling = false;
    write_headers();
    cudaError_t e = cudaGraphLaunch(exec, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    size_t n = 0;
    for (size_t i = 1; e == cudaSuccess && i < prof_ev.size(); ++i) {
      float t = 0.f;
      e = cudaEventElapsedTime(&t, prof_ev[i - 1], prof_ev[i]);
      if (n < cap_groups) {
        kinds[n] = prof_kind[i];
        ms[n] = t;
        bytes[n] = prof_bytes[i];
      }
      ++n;
    }
    cudaGraphExecDestroy(exec);
    for (cudaEvent_t ev : prof_ev) cudaEventDestroy(ev);
    prof_ev.clear(), prof_kind.clear(), prof_bytes.clear();
    RTA_CUDA(e);
    if (n_groups) *n_groups = n;
    read_control(1);
  }

  // Copy the control blocks back (header plus the first `ids` emitted ids of
  // every sequence) and surface device-side errors.
  void read_control(uint32_t ids = 0) {
    const size_t width = offsetof(Control, ids) + 4ull * std::min(ids, kMaxOut);
    RTA_CUDA(cudaMemcpy2DAsync(ctrl_host, sizeof(Control), ctrl.p, sizeof(Control), width, nseq,
                               cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
    uint32_t err = 0;
    for (uint32_t z = 0; z < nseq; ++z) {
      err |= ctrl_host[z].err;
      positions[z] = ctrl_host[z].pos_next;
    }
    position = positions[0];
    if (team) {  // the exchanges' own error word (a peer that never arrived)
      uint32_t terr = 0;
      RTA_CUDA(cudaMemcpy(&terr, team_error_word(team), 4, cudaMemcpyDeviceToHost));
      err |= terr;
    }
    if (err & RTA_DEVERR_TIMEOUT) throw Failure{RTA_E_TIMEOUT, "device-side wait exceeded its bound"};
    if (err) throw Failure{RTA_E_DEVICE_CHECK, "device error word " + std::to_string(err)};
  }
  void write_headers() {
    RTA_CUDA(cudaMemcpy2DAsync(ctrl.p, sizeof(Control), ctrl_host, sizeof(Control), offsetof(Control, ids), nseq,
                               cudaMemcpyHostToDevice, stream));
  }

  // Prefill every sequence in lockstep: replay i feeds prompt id i of each
  // sequence that has one; a sequence with a shorter prompt sits out the rest.
  void prefill_batch(const uint32_t* ids, const uint32_t* lengths, uint32_t stride, const uint32_t st[2],
                     bool allow_chunks = true) {
    uint32_t longest = 0;
    for (uint32_t z = 0; z < nseq; ++z) {
      require(lengths[z] <= capacity && lengths[z] <= stride, "prefill length must be at most capacity", RTA_E_ARG);
      for (uint32_t i = 0; i < lengths[z]; ++i)
        require(ids[static_cast<size_t>(z) * stride + i] < spec.vocabulary_size, "token id beyond the vocabulary",
                RTA_E_ARG);
      longest = std::max(longest, lengths[z]);
    }
    require(longest >= 1, "prefill needs at least one prompt id", RTA_E_ARG);
    stops[0] = st ? st[0] : 0xffffffffu;
    stops[1] = st ? st[1] : 0xffffffffu;
    reset_sequence();
    std::vector<uint32_t> rows(static_cast<size_t>(nseq) * capacity, 0u);
    for (uint32_t z = 0; z < nseq; ++z)
      std::copy_n(ids + static_cast<size_t>(z) * stride, lengths[z], rows.begin() + static_cast<size_t>(z) * capacity);
    RTA_CUDA(cudaMemcpyAsync(prompt.p, rows.data(), rows.size() * 4ull, cudaMemcpyHostToDevice, stream));
    std::memset(ctrl_host, 0, sizeof(Control) * nseq);
    for (uint32_t z = 0; z < nseq; ++z) {
      ctrl_host[z].running = lengths[z] > 0 ? 1u : 0u;
      ctrl_host[z].prompt_len = lengths[z];
      ctrl_host[z].stops[0] = stops[0];
      ctrl_host[z].stops[1] = stops[1];
    }
    write_headers();
    RTA_CUDA(cudaEventRecord(ev0, stream));
    if (chunked && g_chunk && allow_chunks)  // kChunk prompt positions per replay
      for (uint32_t i = 0; i < longest; i += kChunk) RTA_CUDA(cudaGraphLaunch(g_chunk, stream));
    else
      for (uint32_t i = 0; i < longest; ++i) RTA_CUDA(cudaGraphLaunch(g_prefill, stream));
    RTA_CUDA(cudaEventRecord(ev1, stream));
    read_control();
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    last_gpu_ms = ms;
  }

  // Debug prefill: the same steps through the capture graph, then the
  // final-normed row of every position (states [n][D]) and, when layers is not
  // NULL, every layer's output row ([depth][n][D]).
  void prefill_capture(const uint32_t* ids, uint32_t n, const uint32_t st[2], float* states, float* layer_rows) {
    invalidate_cache(true);  // layer capture recomputes the prompt outside the caches
    require(nseq == 1 && !team, "debug prefill serves single-sequence handles", RTA_E_STATE);
    require(n >= 1 && n <= capacity, "prefill length must be 1..capacity", RTA_E_ARG);
    require(states != nullptr, "debug prefill needs the state rows", RTA_E_ARG);
    const size_t rows = static_cast<size_t>(capacity) * D();
    if (!g_prefill_cap) {
      cap.alloc((spec.depth + 1ull) * rows);
      g_prefill_cap = instantiate_step(false, true, nullptr);
    }
    std::swap(g_prefill, g_prefill_cap);  // prefill_batch replays g_prefill
    try {
      prefill_batch(ids, &n, n, st, false);
    } catch (...) {
      std::swap(g_prefill, g_prefill_cap);
      throw;
    }
    std::swap(g_prefill, g_prefill_cap);
    RTA_CUDA(cudaMemcpyAsync(states, cap.p, static_cast<size_t>(n) * D() * 4, cudaMemcpyDeviceToHost, stream));
    if (layer_rows)
      for (uint32_t l = 0; l < spec.depth; ++l)
        RTA_CUDA(cudaMemcpyAsync(layer_rows + static_cast<size_t>(l) * n * D(), cap.p + (l + 1ull) * rows,
                                 static_cast<size_t>(n) * D() * 4, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
  }

  void prefill(const uint32_t* ids, uint32_t n, const uint32_t st[2]) {
    require(nseq == 1, "this handle decodes several sequences: use the batch prefill", RTA_E_STATE);
    require(n >= 1 && n <= capacity, "prefill length must be 1..capacity", RTA_E_ARG);
    prefill_batch(ids, &n, n, st);
  }

  // Synthetic histories for throughput runs: every ring slot, recurrent state,
  // conv history and residual row is filled with seeded values and sequence z
  // resumes at position lengths[z] (as if it had been prefilled that far).
  void seed_history(const uint32_t* lengths, uint64_t seed) {
    for (uint32_t z = 0; z < nseq; ++z) require(lengths[z] >= 1, "history lengths must be positive", RTA_E_ARG);
    reset_sequence();
    if (packet_history) {
      RTA_CUDA(launch_random_packets(seed, pring.n / pbytes, spec.kv_heads, pring.p, stream));
    } else {
      RTA_CUDA(launch_random_normal_half(seed, 1.0f, kcache.n, kcache.p, stream));
      RTA_CUDA(launch_random_normal_half(seed + 1, 1.0f, vcache.n, vcache.p, stream));
    }
    RTA_CUDA(launch_random_normal(seed + 2, 0.02f, 0.0f, rec.n, rec.p, stream));
    RTA_CUDA(launch_random_normal(seed + 3, 1.0f, 0.0f, conv.n, conv.p, stream));
    RTA_CUDA(launch_random_normal(seed + 4, 1.0f, 0.0f, state.n, state.p, stream));
    std::memset(ctrl_host, 0, sizeof(Control) * nseq);
    for (uint32_t z = 0; z < nseq; ++z) {
      ctrl_host[z].pos_next = lengths[z];
      ctrl_host[z].pos_cur = lengths[z] - 1u;
      ctrl_host[z].stops[0] = ctrl_host[z].stops[1] = 0xffffffffu;
    }
    stops[0] = stops[1] = 0xffffffffu;
    write_headers();
    read_control();
  }

  // `count` greedy tokens for every sequence that has a history; a sequence
  // stops on its own at a stop id.  ids_out: [nseq][count].
  void generate_batch(uint32_t count, uint32_t* ids_out, uint32_t* n_out) {
    require(count >= 1 && count <= kMaxOut, "generate count must be 1..4096", RTA_E_ARG);
    bool any = false;
    for (uint32_t z = 0; z < nseq; ++z) {
      ctrl_host[z].running = positions[z] > 0 ? 1u : 0u;
      ctrl_host[z].n_out = 0u;
      ctrl_host[z].stops[0] = stops[0];
      ctrl_host[z].stops[1] = stops[1];
      any = any || positions[z] > 0;
    }
    require(any, "prefill before generate", RTA_E_STATE);
    write_headers();
    RTA_CUDA(cudaEventRecord(ev0, stream));
    for (uint32_t i = 0; i < count; ++i) RTA_CUDA(cudaGraphLaunch(g_decode, stream));
    RTA_CUDA(cudaEventRecord(ev1, stream));
    read_control(count);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    last_gpu_ms = ms;
    for (uint32_t z = 0; z < nseq; ++z) {
      const uint32_t got = std::min(ctrl_host[z].n_out, count);
      if (ids_out) std::memcpy(ids_out + static_cast<size_t>(z) * count, ctrl_host[z].ids, got * 4ull);
      if (n_out) n_out[z] = got;
    }
  }

  void generate(uint32_t count, uint32_t* ids_out, uint32_t* n_out) {
    require(nseq == 1, "this handle decodes several sequences: use the batch generate", RTA_E_STATE);
    require(position > 0, "prefill before generate", RTA_E_STATE);
    generate_batch(count, ids_out, n_out);
  }

  // ------------------------------------------------------------ cache logic
  // whole: the sequence bookkeeping is void (the state moved outside the
  // caches); else only boundaries stop being saved / restored.
  void invalidate_cache(bool whole) {
    if (!cache) return;
    cache->prefix_ok = false;
    if (whole) {
      cache->ready = false;
      cache->address_ok = false;
    }
  }
  bool is_stop(uint32_t t) const { return t == stops[0] || t == stops[1]; }
  // generated tokens the device state has to consume (a trailing stop id has no step)
  uint32_t consumable() const {
    const auto& g = cache->gen;
    return static_cast<uint32_t>(g.size()) - (!g.empty() && is_stop(g.back()) ? 1u : 0u);
  }

  // The state address of the live sequence into addresses[slot] (device).
  void digest(uint32_t slot) { digest_at(cache->addresses.p + slot * 8ull, nullptr, 1u); }
  // ... into out, or into out[*counter] (counter advanced, `slots` at most).
  void digest_at(uint32_t* out, uint32_t* counter, uint32_t slots) {
    Caches& c = *cache;
    DigestArgs a;
    a.words[0] = reinterpret_cast<const uint32_t*>(state.p);
    a.count[0] = state.n;
    a.words[1] = reinterpret_cast<const uint32_t*>(rec.p);
    a.count[1] = n_rec ? rec.n : 0u;
    a.words[2] = reinterpret_cast<const uint32_t*>(conv.p);
    a.count[2] = n_rec ? conv.n : 0u;
    a.n_full = n_full;
    a.kvh = spec.kv_heads;
    a.hd = spec.attention_head_dim;
    a.capacity = capacity;
    if (packet_history) {
      a.packets = pring.p;
      a.pbytes = pbytes;
    } else {
      a.kcache = kcache.p;
      a.vcache = vcache.p;
      a.layer_kv = static_cast<size_t>(spec.kv_heads) * capacity * spec.attention_head_dim * na;
    }
    a.slot_hash = c.slot_hash.p;
    a.cursor = c.cursor.p;
    a.pos_next = &ctrl.p->pos_next;
    a.partial = c.partial.p;
    a.out = out;
    a.slot = counter;
    a.slots = slots;
    a.seed[0] = c.epoch;
    a.seed[1] = capacity;
    a.seed[2] = stops[0];
    a.seed[3] = stops[1];
    RTA_CUDA(launch_state_digest(a, stream));
    ++c.info[RTA_CACHE_DIGESTS];
  }
  // The decode step followed by the digest of its result into addresses[1 +
  // *slot]: one graph per token while the reply tree records.
  cudaGraphExec_t instantiate_digest_step() {
    Caches& c = *cache;
    cudaGraph_t graph = nullptr;
    RTA_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeRelaxed));
    try {
      record_step(true, false);
      digest_at(c.addresses.p + 8u, c.slot.p, kMaxOut);
    } catch (...) {
      cudaStreamEndCapture(stream, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    RTA_CUDA(cudaStreamEndCapture(stream, &graph));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    RTA_CUDA(e);
    --c.info[RTA_CACHE_DIGESTS];  // the capture launched nothing
    return exec;
  }
  std::vector<Key256> read_addresses(uint32_t first, uint32_t n) {
    std::vector<Key256> out(n);
    if (n)
      RTA_CUDA(cudaMemcpyAsync(out.data(), cache->addresses.p + first * 8ull, n * sizeof(Key256),
                               cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
    return out;
  }

  // History rows of every full layer, positions [b.first, b.first + b.count),
  // between the ring and the block's own copy ([layer][K, V][kvh][count][hd]
  // halves, or [layer][count][packet]).
  size_t block_bytes(uint32_t count) const {
    const size_t row = packet_history ? pbytes : 4ull * spec.kv_heads * spec.attention_head_dim;
    return static_cast<size_t>(n_full) * count * row;
  }
  void block_segments(const HistoryBlock& b, bool to_ring, std::vector<CopySeg>& out, uint64_t& longest) {
    const uint32_t hd = spec.attention_head_dim, kvh = spec.kv_heads;
    uint8_t* mine = static_cast<uint8_t*>(b.rows.p);
    auto push = [&](void* ring, uint8_t* own, uint64_t bytes) {
      out.push_back(to_ring ? CopySeg{own, ring, bytes} : CopySeg{ring, own, bytes});
      longest = std::max(longest, bytes);
    };
    for (uint32_t fi = 0; fi < n_full; ++fi) {
      if (packet_history) {
        const uint64_t bytes = static_cast<uint64_t>(b.count) * pbytes;
        push(pring.p + (static_cast<size_t>(fi) * capacity + b.first) * pbytes, mine + fi * bytes, bytes);
      } else {
        const size_t layer_kv = static_cast<size_t>(kvh) * capacity * hd;
        const uint64_t bytes = static_cast<uint64_t>(b.count) * hd * 2u;
        for (uint32_t kv = 0; kv < 2; ++kv)
          for (uint32_t h = 0; h < kvh; ++h)
            push((kv ? vcache.p : kcache.p) + fi * layer_kv + (static_cast<size_t>(h) * capacity + b.first) * hd,
                 mine + ((static_cast<size_t>(fi) * 2u + kv) * kvh + h) * bytes, bytes);
      }
    }
  }
  void run_segments(const std::vector<CopySeg>& segs, uint64_t longest) {
    Caches& c = *cache;
    for (size_t first = 0; first < segs.size(); first += c.segs.n) {
      const size_t n = std::min(c.segs.n, segs.size() - first);
      RTA_CUDA(cudaMemcpyAsync(c.segs.p, segs.data() + first, n * sizeof(CopySeg), cudaMemcpyHostToDevice, stream));
      RTA_CUDA(launch_copy_segments(c.segs.p, static_cast<uint32_t>(n), longest, stream));
    }
  }

  // Boundary e (ids = the live sequence): the state words, and the history of
  // [0, n) in 16-position blocks, copied out of the ring only for blocks no
  // other boundary holds already.
  void save_boundary(HistoryEntry& e, const std::vector<Key256>& keys) {
    Caches& c = *cache;
    const size_t sb = state.n * 4u, rb = rec.n * 4u, cb = conv.n * 4u;
    RTA_CUDA(e.snapshot.alloc(sb + rb + cb, stream));
    uint8_t* d = static_cast<uint8_t*>(e.snapshot.p);
    RTA_CUDA(cudaMemcpyAsync(d, state.p, sb, cudaMemcpyDeviceToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(d + sb, rec.p, rb, cudaMemcpyDeviceToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(d + sb + rb, conv.p, cb, cudaMemcpyDeviceToDevice, stream));
    std::vector<CopySeg> segs;
    uint64_t longest = 0;
    const uint32_t n = static_cast<uint32_t>(e.ids.size());
    e.blocks.clear();
    if (n_full)
      for (uint32_t first = 0; first < n; first += 16u) {
        const uint32_t cnt = std::min(16u, n - first);
        bool fresh = false;
        auto b = c.index.block(keys[first + cnt], first, cnt, &fresh);
        if (fresh) {
          RTA_CUDA(b->rows.alloc(block_bytes(cnt), stream));
          block_segments(*b, false, segs, longest);
          b->ready = true;
        }
        e.blocks.push_back(std::move(b));
      }
    run_segments(segs, longest);
    e.saved = true;
  }
  // Make boundary e the live state: its state words, its history blocks into
  // the ring, and a control block that resumes at its length.
  void attach(const HistoryEntry& e) {
    Caches& c = *cache;
    const size_t sb = state.n * 4u, rb = rec.n * 4u, cb = conv.n * 4u;
    const uint8_t* d = static_cast<const uint8_t*>(e.snapshot.p);
    RTA_CUDA(cudaMemcpyAsync(state.p, d, sb, cudaMemcpyDeviceToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(rec.p, d + sb, rb, cudaMemcpyDeviceToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(conv.p, d + sb + rb, cb, cudaMemcpyDeviceToDevice, stream));
    std::vector<CopySeg> segs;
    uint64_t longest = 0;
    for (const auto& b : e.blocks) block_segments(*b, true, segs, longest);
    run_segments(segs, longest);
    const uint32_t n = static_cast<uint32_t>(e.ids.size());
    std::memset(ctrl_host, 0, sizeof(Control));
    ctrl_host[0].pos_next = n;
    ctrl_host[0].pos_cur = n - 1u;
    ctrl_host[0].stops[0] = stops[0];
    ctrl_host[0].stops[1] = stops[1];
    write_headers();
    c.cursor.zero(stream);
    c.attached = e.blocks;
    read_control();
  }
  // Feed ids[from, to) to the state at position `from` through the prefill
  // graphs, without the reset: chunks, or one position per replay (per_token,
  // the decode step's own kernels without the readout).
  void extend(const uint32_t* ids, uint32_t from, uint32_t to, bool per_token) {
    require(from < to && to <= capacity, "cached extension must stay inside the ring", RTA_E_ARG);
    RTA_CUDA(cudaMemcpyAsync(prompt.p + from, ids + from, (to - from) * 4ull, cudaMemcpyHostToDevice, stream));
    std::memset(ctrl_host, 0, sizeof(Control));
    ctrl_host[0].running = 1u;
    ctrl_host[0].prompt_len = to;
    ctrl_host[0].pos_next = from;
    ctrl_host[0].pos_cur = from ? from - 1u : 0u;
    ctrl_host[0].stops[0] = stops[0];
    ctrl_host[0].stops[1] = stops[1];
    write_headers();
    if (chunked && g_chunk && !per_token)
      for (uint32_t i = from; i < to; i += kChunk) RTA_CUDA(cudaGraphLaunch(g_chunk, stream));
    else
      for (uint32_t i = from; i < to; ++i) RTA_CUDA(cudaGraphLaunch(g_prefill, stream));
    read_control();
  }

  // Worker ops 1 / 11 / 12 with the caches (Resident::prefill,
  // optical_resident.cpp:635-699): restore the longest saved boundary that
  // prefixes the prompt, compute the rest, save the prompt's end as a boundary
  // (when anything was computed), and take the state address.
  void prefill_cached(const uint32_t* ids, uint32_t n, const uint32_t st[2], uint32_t boundary) {
    require(n >= 1 && n <= capacity, "prefill length must be 1..capacity", RTA_E_ARG);
    require(boundary >= 1 && boundary <= n, "checkpoint boundary must lie in 1..n", RTA_E_ARG);
    for (uint32_t i = 0; i < n; ++i) require(ids[i] < spec.vocabulary_size, "token id beyond the vocabulary", RTA_E_ARG);
    Caches& c = *cache;
    std::fill(c.info, c.info + RTA_CACHE_INFO_WORDS, 0ull);
    c.info[RTA_CACHE_TREE_LEAF] = 0xffffffffull;
    c.ready = c.prefix_ok = c.address_ok = false;
    stops[0] = st ? st[0] : 0xffffffffu;
    stops[1] = st ? st[1] : 0xffffffffu;
    const auto t0 = std::chrono::steady_clock::now();
    const std::vector<Key256> keys = prefix_identities(ids, n, c.epoch);
    uint32_t lookups = 0;
    std::shared_ptr<HistoryEntry> hit = c.index.find(ids, n, keys, 1u, &lookups);
    c.ms[0] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    const uint32_t reused = hit ? static_cast<uint32_t>(hit->ids.size()) : 0u;
    const bool address_hit = hit && reused == n && hit->address_ready && hit->stops[0] == stops[0] &&
                             hit->stops[1] == stops[1];
    const uint32_t rows = n - reused;
    std::shared_ptr<HistoryEntry> entry = rows ? c.index.reserve(ids, n, 1u, keys[n]) : nullptr;
    Key256 address{};
    try {
      RTA_CUDA(cudaEventRecord(ev0, stream));
      if (hit) {
        attach(*hit);
      } else {
        reset_sequence();
        c.attached.clear();
      }
      if (rows) extend(ids, reused, n, false);
      if (entry) save_boundary(*entry, keys);
      if (!address_hit) digest(0);
      RTA_CUDA(cudaEventRecord(ev1, stream));
      address = address_hit ? hit->address : read_addresses(0, 1)[0];
    } catch (...) {
      c.index.erase(entry);
      throw;
    }
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    last_gpu_ms = ms;
    HistoryEntry* at_end = entry ? entry.get() : (reused == n ? hit.get() : nullptr);
    if (at_end) {
      at_end->address = address;
      at_end->address_ready = true;
      at_end->stops[0] = stops[0];
      at_end->stops[1] = stops[1];
    }
    c.prefix.assign(ids, ids + n);
    c.gen.clear();
    c.fwd = 0;
    c.address = address;
    c.ready = c.prefix_ok = c.address_ok = true;
    const uint64_t held = c.index.evict(c.budget, entry.get(), hit.get());
    c.info[RTA_CACHE_PREFILL_HIT] = hit ? 1u : 0u;
    c.info[RTA_CACHE_REUSED_TOKENS] = reused;
    c.info[RTA_CACHE_STABLE_TOKENS] = boundary;
    c.info[RTA_CACHE_SNAPSHOT_KIND] = !hit ? 0u : reused == n ? 1u : reused == boundary ? 2u : 3u;
    c.info[RTA_CACHE_SHARED_BLOCKS] = hit ? hit->blocks.size() : 0u;
    c.info[RTA_CACHE_SAVED_BOUNDARIES] = entry ? 1u : 0u;
    c.info[RTA_CACHE_BOUNDARIES] = c.index.size();
    c.info[RTA_CACHE_LOOKUPS] = lookups;
    c.info[RTA_CACHE_COMPUTED_TOKENS] = rows;
    c.info[RTA_CACHE_EVICTIONS] = c.index.evictions;
    c.info[RTA_CACHE_ADDRESS_HIT] = address_hit ? 1u : 0u;
    c.info[RTA_CACHE_BYTES] = held;
    c.info[RTA_CACHE_TREE_NODES] = c.tree.size();
    c.info[RTA_CACHE_TREE_CAPACITY] = ReplyTree::kCapacity;
  }

  // Bring the device state level with every emitted token: from the longest
  // saved boundary past it, if any, then one prefill step per token (the
  // decode step's kernels, so the state is the one decoding would have left).
  void materialize() {
    Caches& c = *cache;
    const uint32_t target = consumable();
    if (c.fwd >= target) return;
    const uint32_t n = static_cast<uint32_t>(c.prefix.size());
    std::vector<uint32_t> seq(c.prefix);
    seq.insert(seq.end(), c.gen.begin(), c.gen.begin() + target);
    RTA_CUDA(cudaEventRecord(ev0, stream));
    bool restored = false;
    if (c.prefix_ok) {
      const std::vector<Key256> keys = prefix_identities(seq.data(), seq.size(), c.epoch);
      uint32_t lookups = 0;
      std::shared_ptr<HistoryEntry> b = c.index.find(seq.data(), seq.size(), keys, n + c.fwd + 1u, &lookups);
      if (b) {
        attach(*b);
        c.fwd = static_cast<uint32_t>(b->ids.size()) - n;
        restored = true;
      }
    }
    c.info[RTA_CACHE_RESTORED_TOKENS] = target - c.fwd;
    c.info[RTA_CACHE_CHECKPOINT_RESTORED] = restored ? 1u : 0u;
    if (c.fwd < target) extend(seq.data(), n + c.fwd, n + target, true);
    RTA_CUDA(cudaEventRecord(ev1, stream));
    RTA_CUDA(cudaEventSynchronize(ev1));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    c.ms[2] = ms;
    c.fwd = target;
  }

  // Worker op 2 with the caches (Resident::generatePacket,
  // optical_resident.cpp:770-853): follow the reply tree from the state
  // address, then decode the rest with the address of every step's result and
  // record those steps.  The tree serves positions inside the ring.
  void generate_cached(uint32_t count, uint32_t* ids_out, uint32_t* n_out) {
    require(count >= 1 && count <= kMaxOut, "generate count must be 1..4096", RTA_E_ARG);
    Caches& c = *cache;
    for (int k = RTA_CACHE_REPLAYED_TOKENS; k <= RTA_CACHE_CHECKPOINT_RESTORED; ++k) c.info[k] = 0u;
    c.info[RTA_CACHE_TREE_LEAF] = 0xffffffffull;
    c.info[RTA_CACHE_DIGESTS] = 0u;
    c.ms[1] = c.ms[2] = 0.0;
    std::vector<uint32_t> out;
    out.reserve(count);
    uint32_t p = static_cast<uint32_t>(c.prefix.size()) + consumable();
    const bool tree = c.address_ok && static_cast<uint64_t>(p) + count <= capacity;
    bool stopped = false;
    uint32_t replayed = 0, queries = 0;
    const auto t0 = std::chrono::steady_clock::now();
    if (tree) {
      Key256 key = c.address;
      while (replayed < count) {
        ++queries;
        uint32_t slot = 0;
        const ReplyTree::Node* nd = c.tree.find(key, p, &slot);
        if (!nd) break;
        out.push_back(nd->token);
        c.gen.push_back(nd->token);
        ++replayed;
        c.info[RTA_CACHE_TREE_LEAF] = slot;
        if (is_stop(nd->token)) {
          stopped = true;
          break;
        }
        key = nd->next;
        ++p;
      }
      c.address = key;
    }
    c.ms[1] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    double gpu = 0.0;
    if (replayed < count && !stopped) {
      materialize();
      const uint32_t rest = count - replayed;
      ctrl_host[0].running = 1u;
      ctrl_host[0].n_out = 0u;
      ctrl_host[0].stops[0] = stops[0];
      ctrl_host[0].stops[1] = stops[1];
      write_headers();
      if (tree) {
        if (c.g_step && (c.g_step_stops[0] != stops[0] || c.g_step_stops[1] != stops[1])) {
          cudaGraphExecDestroy(c.g_step);  // the stop ids are part of the address
          c.g_step = nullptr;
        }
        if (!c.g_step) {
          c.g_step = instantiate_digest_step();
          c.g_step_stops[0] = stops[0];
          c.g_step_stops[1] = stops[1];
        }
        RTA_CUDA(cudaMemsetAsync(c.slot.p, 0, 4, stream));
      }
      RTA_CUDA(cudaEventRecord(ev0, stream));
      for (uint32_t i = 0; i < rest; ++i) RTA_CUDA(cudaGraphLaunch(tree ? c.g_step : g_decode, stream));
      RTA_CUDA(cudaEventRecord(ev1, stream));
      if (tree) c.info[RTA_CACHE_DIGESTS] += rest;
      read_control(rest);
      float ms = 0.f;
      cudaEventElapsedTime(&ms, ev0, ev1);
      gpu = ms;
      const uint32_t got = std::min(ctrl_host[0].n_out, rest);
      const uint32_t* tok = ctrl_host[0].ids;
      if (tree) {
        const std::vector<Key256> addr = read_addresses(1u, got);
        Key256 prev = c.address;
        for (uint32_t i = 0; i < got; ++i) {
          c.tree.record(prev, p + i, tok[i], addr[i]);
          prev = addr[i];
        }
        c.address = prev;
      } else {
        c.address_ok = false;  // past the ring: the tree stays out until the next prefill
      }
      for (uint32_t i = 0; i < got; ++i) {
        out.push_back(tok[i]);
        c.gen.push_back(tok[i]);
      }
      c.fwd = consumable();
    }
    last_gpu_ms = gpu + c.ms[2];
    c.info[RTA_CACHE_REPLAYED_TOKENS] = replayed;
    c.info[RTA_CACHE_TREE_QUERIES] = queries;
    c.info[RTA_CACHE_TREE_NODES] = c.tree.size();
    c.info[RTA_CACHE_TREE_CAPACITY] = ReplyTree::kCapacity;
    c.info[RTA_CACHE_BOUNDARIES] = c.index.size();
    c.info[RTA_CACHE_EVICTIONS] = c.index.evictions;
    if (ids_out) std::copy(out.begin(), out.end(), ids_out);
    if (n_out) *n_out = static_cast<uint32_t>(out.size());
  }

  // Worker op 13 (Resident::finishHistory, optical_resident.cpp:743-759).
  void finish_history(uint64_t* saved, uint64_t* tokens, uint64_t* boundaries) {
    Caches& c = *cache;
    c.info[RTA_CACHE_FINISH_SAVED] = c.info[RTA_CACHE_FINISH_TOKENS] = 0u;
    const uint32_t n = static_cast<uint32_t>(c.prefix.size()), m = consumable();
    if (c.ready && c.prefix_ok && !c.gen.empty() && c.fwd == m && n + m <= capacity) {
      std::vector<uint32_t> ids(c.prefix);
      ids.insert(ids.end(), c.gen.begin(), c.gen.begin() + m);
      const uint32_t t = static_cast<uint32_t>(ids.size());
      c.info[RTA_CACHE_FINISH_TOKENS] = t;
      const std::vector<Key256> keys = prefix_identities(ids.data(), t, c.epoch);
      std::shared_ptr<HistoryEntry> e = c.index.reserve(ids.data(), t, 2u, keys[t]);
      if (e) {
        try {
          save_boundary(*e, keys);
          RTA_CUDA(cudaStreamSynchronize(stream));
        } catch (...) {
          c.index.erase(e);
          throw;
        }
        if (c.address_ok) {
          e->address = c.address;
          e->address_ready = true;
          e->stops[0] = stops[0];
          e->stops[1] = stops[1];
        }
        c.info[RTA_CACHE_FINISH_SAVED] = 1u;
        c.info[RTA_CACHE_BYTES] = c.index.evict(c.budget, e.get(), nullptr);
      }
    }
    c.info[RTA_CACHE_BOUNDARIES] = c.index.size();
    c.info[RTA_CACHE_EVICTIONS] = c.index.evictions;
    if (saved) *saved = c.info[RTA_CACHE_FINISH_SAVED];
    if (tokens) *tokens = c.info[RTA_CACHE_FINISH_TOKENS];
    if (boundaries) *boundaries = c.index.size();
  }

  // The address of the live state, level with every emitted token.
  Key256 state_address() {
    require(cache != nullptr, "the handle was opened without RTA_MODEL_CACHE", RTA_E_STATE);
    if (cache->ready) materialize();
    digest(0);
    return read_addresses(0, 1)[0];
  }

  // Worker op 14 (attentionCheck, resident_attention_runtime.inl:646-753): the
  // full-attention detector of one full layer over a supplied causal history.
  // K/V rows are packed into the reference's history packets (returned), the
  // detector runs over the packets with one split per newest-first group of
  // `block` positions, and every (row, group, head) record becomes one dense
  // receipt (verify_attention_receipts.py:140-203 reads them).
  void attention_check(uint32_t layer, const float* q, const float* k, const float* v, const float* gate,
                       uint32_t rows, uint32_t count, uint32_t query_start, uint32_t history_start, uint32_t block,
                       float* out, float* phys, uint8_t* packets_out, uint32_t* receipts, uint32_t* n_records,
                       double* timing) {
    invalidate_cache(false);
    const uint32_t H = spec.attention_heads, KVH = spec.kv_heads, hd = spec.attention_head_dim;
    require(!team, "diagnostics are served by single-GPU handles", RTA_E_STATE);
    require(layer < spec.depth && layers[layer]->full, "attention diagnostic needs a full-attention layer", RTA_E_ARG);
    require(rows >= 1 && rows <= 32 && count >= 1 && count <= capacity, "attention rows 1..32, count 1..capacity",
            RTA_E_ARG);
    require(query_start >= history_start &&
                static_cast<uint64_t>(query_start) + rows <= static_cast<uint64_t>(history_start) + count,
            "query times must lie inside the supplied causal history", RTA_E_ARG);
    require(block == 128 || block == 256 || block == 512, "attention block must be 128, 256 or 512", RTA_E_ARG);
    const size_t nq = static_cast<size_t>(rows) * H * hd, nk = static_cast<size_t>(count) * KVH * hd;
    for (size_t i = 0; i < nq; ++i)
      require(std::isfinite(q[i]) && std::isfinite(gate[i]), "attention values must be finite", RTA_E_ARG);
    for (size_t i = 0; i < nk; ++i)
      require(std::isfinite(k[i]) && std::isfinite(v[i]), "attention values must be finite", RTA_E_ARG);
    // visible positions and receipt groups per row
    std::vector<uint32_t> visible(rows), times(rows);
    uint32_t groups = 0, records = 0;
    for (uint32_t r = 0; r < rows; ++r) {
      times[r] = query_start + r;
      visible[r] = std::min(times[r] - history_start + 1u, capacity);
      const uint32_t g = (visible[r] + block - 1u) / block;
      groups = std::max(groups, g);
      records += g * H;
    }
    DevBuf<float> dq, dk, dv, dg, dout, dphys, pm, pz, po;
    DevBuf<uint8_t> dpk;
    DevBuf<uint32_t> dt, derr;
    dq.alloc(nq);
    dg.alloc(nq);
    dk.alloc(nk);
    dv.alloc(nk);
    dout.alloc(nq);
    dphys.alloc(static_cast<size_t>(rows) * H * 2);
    const size_t recs = static_cast<size_t>(rows) * KVH * groups * 4;
    pm.alloc(recs);
    pz.alloc(recs);
    po.alloc(recs * hd);
    dpk.alloc(static_cast<size_t>(count) * pbytes);
    dt.alloc(rows);
    derr.alloc(1);
    derr.zero(stream);
    RTA_CUDA(cudaMemcpyAsync(dq.p, q, nq * 4, cudaMemcpyHostToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(dg.p, gate, nq * 4, cudaMemcpyHostToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(dk.p, k, nk * 4, cudaMemcpyHostToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(dv.p, v, nk * 4, cudaMemcpyHostToDevice, stream));
    RTA_CUDA(cudaMemcpyAsync(dt.p, times.data(), rows * 4ull, cudaMemcpyHostToDevice, stream));
    RTA_CUDA(cudaEventRecord(ev0, stream));
    RTA_CUDA(launch_pack_history(dk.p, dv.p, count, KVH, dpk.p, stream));
    AttnParams ap;
    ap.q = dq.p;
    ap.q_seq_stride = static_cast<size_t>(H) * hd;
    ap.heads = H;
    ap.kvh = KVH;
    ap.hd = hd;
    ap.capacity = capacity;
    ap.history_start = history_start;
    ap.pos = dt.p;
    ap.ctrl_step = 1;
    ap.gate = spec.attention_gate ? dg.p : nullptr;
    ap.gate_seq_stride = static_cast<size_t>(H) * hd;
    ap.out = dout.p;
    ap.out_seq_stride = static_cast<size_t>(H) * hd;
    ap.phys = dphys.p;
    ap.part_m = pm.p;
    ap.part_z = pz.p;
    ap.part_o = po.p;
    ap.err = derr.p;
    ap.packets = dpk.p;
    ap.packet_seq_stride = 0;  // every row reads the same supplied history
    ap.packet_stride = pbytes;
    ap.packet_base = history_start;
    ap.group_block = block;
    RTA_CUDA(launch_attention(ap, groups, rows, false, stream));
    RTA_CUDA(cudaEventRecord(ev1, stream));
    std::vector<float> hm(recs), hz(recs), ho(recs * hd);
    RTA_CUDA(cudaMemcpyAsync(out, dout.p, nq * 4, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaMemcpyAsync(phys, dphys.p, static_cast<size_t>(rows) * H * 8, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaMemcpyAsync(packets_out, dpk.p, static_cast<size_t>(count) * pbytes, cudaMemcpyDeviceToHost,
                             stream));
    RTA_CUDA(cudaMemcpyAsync(hm.data(), pm.p, recs * 4, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaMemcpyAsync(hz.data(), pz.p, recs * 4, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaMemcpyAsync(ho.data(), po.p, recs * hd * 4, cudaMemcpyDeviceToHost, stream));
    uint32_t err = 0;
    RTA_CUDA(cudaMemcpyAsync(&err, derr.p, 4, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    if (timing) timing[0] = ms;
    require(err == 0, "attention diagnostic device error " + std::to_string(err), RTA_E_DEVICE_CHECK);
    // dense receipts in the reference's order: row, group (newest first), head
    const uint32_t words = block / 32u, stride = hd + 8u + words;
    size_t at = 0;
    for (uint32_t r = 0; r < rows; ++r) {
      const uint32_t ng = (visible[r] + block - 1u) / block;
      for (uint32_t g = 0; g < ng; ++g) {
        const uint32_t cnt = std::min(block, visible[r] - g * block);
        for (uint32_t h = 0; h < H; ++h) {
          const uint32_t kv = h / (H / KVH), hq = h % (H / KVH);
          const size_t rec = ((static_cast<size_t>(r) * KVH + kv) * groups + g) * 4 + hq;
          uint32_t* w = receipts + at * stride;
          const float m = hm[rec], zz = hz[rec];
          bool finite = std::isfinite(m) && std::isfinite(zz);
          for (uint32_t d = 0; d < hd; ++d) finite = finite && std::isfinite(ho[rec * hd + d]);
          std::memcpy(&w[0], &m, 4);
          std::memcpy(&w[1], &zz, 4);
          w[2] = cnt;          // positions in the group
          w[3] = cnt;          // exponentials: one per position
          w[4] = cnt;          // value rows accumulated one by one (no vector grouping)
          w[5] = cnt;          // weight contributions
          // history-traversal counter of the reference's record (head 0 carries
          // it): 2 + one per 16-position tile, the tiling this kernel also uses
          w[6] = h == 0 ? 2u + (cnt + 15u) / 16u : 0u;
          w[7] = finite ? 3u : 1u;  // bit 0: verified, bit 1: finite
          for (uint32_t i = 0; i < words; ++i) {
            const uint32_t bits = std::min(32u, cnt > 32u * i ? cnt - 32u * i : 0u);
            w[8 + i] = bits == 32u ? 0xffffffffu : (1u << bits) - 1u;
          }
          std::memcpy(&w[8 + words], &ho[rec * hd], hd * 4ull);
          ++at;
        }
      }
    }
    if (n_records) *n_records = records;
  }

  // Inputs and output of the last full-attention layer of the last step for
  // sequence z (q after QK-norm and RoPE, the gate row, the detector output in
  // o-projection axis order) and that layer's visible history packets, oldest
  // first: what a test needs to recompute the layer's attention independently.
  uint32_t debug_attention(uint32_t z, float* q, float* gate, float* att, uint8_t* packets) {
    require(packet_history && !team, "needs a single-GPU packet-history handle", RTA_E_STATE);
    require(z < nseq && positions[z] > 0, "sequence has no history", RTA_E_ARG);
    uint32_t fi = 0;
    bool any = false;
    for (auto& L : layers)
      if (L->full) {
        fi = L->fi;
        any = true;
      }
    require(any, "model has no full-attention layer", RTA_E_STATE);
    const uint32_t t = positions[z] - 1u, n = std::min(t + 1u, capacity), lo = t + 1u - n;
    RTA_CUDA(cudaMemcpyAsync(q, qproc.p + static_cast<size_t>(z) * Q(), Q() * 4ull, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaMemcpyAsync(gate, proj.p + static_cast<size_t>(z) * projw + Q() + 2 * KVW(), Q() * 4ull,
                             cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaMemcpyAsync(att, this->att.p + static_cast<size_t>(z) * Q(), Q() * 4ull, cudaMemcpyDeviceToHost,
                             stream));
    const uint8_t* ring = pring.p + (static_cast<size_t>(fi) * nseq + z) * capacity * pbytes;
    for (uint32_t i = 0; i < n; ++i)
      RTA_CUDA(cudaMemcpyAsync(packets + static_cast<size_t>(i) * pbytes,
                               ring + static_cast<size_t>((lo + i) % capacity) * pbytes, pbytes,
                               cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
    return n;
  }

  void mlp(uint32_t layer, const float* x, uint32_t rows, float* y, float* a) {
    invalidate_cache(false);  // diagnostics end prefix reuse (optical_resident.cpp:969, ops 4/5/6/14)
    require(!team, "diagnostics are served by single-GPU handles", RTA_E_STATE);
    require(layer < spec.depth, "layer out of range", RTA_E_ARG);
    require(rows >= 1 && rows <= 32, "MLP check supports 1..32 rows", RTA_E_ARG);
    const uint32_t D = this->D(), F = spec.middle_size;
    for (size_t i = 0; i < static_cast<size_t>(rows) * D; ++i)
      require(std::isfinite(x[i]), "MLP input must be finite", RTA_E_ARG);
    Layer& L = *layers[layer];
    RTA_CUDA(cudaMemcpyAsync(scratch_x.p, x, static_cast<size_t>(rows) * D * 4, cudaMemcpyHostToDevice, stream));
    if (L.mlp_fmt == kQ4KPanel || L.mlp_fmt == kQ6KPanel) {  // tensor-core handle: all rows in one pair
      GemvArgs gu;
      gu.fmt = L.mlp_fmt;
      gu.w0 = L.gate;
      gu.w1 = L.up;
      gu.rows = F;
      gu.cols = D;
      gu.x = scratch_x.p;
      gu.x_stride = D;
      gu.batch = rows;
      gu.epilogue = kSwiGLU;
      gu.y = scratch_y.p;
      gu.y_stride = F;
      GemvArgs dn;
      dn.fmt = L.down_fmt;
      dn.w0 = L.down;
      dn.rows = D;
      dn.cols = F;
      dn.x = scratch_y.p;
      dn.x_stride = F;
      dn.batch = rows;
      dn.y = scratch_x.p;  // x no longer needed
      dn.y_stride = D;
      mlp_pair(gu, dn, true, stream);
      RTA_CUDA(cudaMemcpyAsync(a, scratch_y.p, static_cast<size_t>(rows) * F * 4, cudaMemcpyDeviceToHost, stream));
      RTA_CUDA(cudaMemcpyAsync(y, scratch_x.p, static_cast<size_t>(rows) * D * 4, cudaMemcpyDeviceToHost, stream));
      RTA_CUDA(cudaStreamSynchronize(stream));
      return;
    }
    for (uint32_t r0 = 0; r0 < rows; r0 += 8) {  // 8-row launches keep the activation tables in shared memory
      const uint32_t nb = std::min(8u, rows - r0);
      GemvArgs gu;
      gu.fmt = L.mlp_fmt;
      gu.w0 = L.gate;
      gu.w1 = L.up;
      gu.rows = F;
      gu.cols = D;
      gu.x = scratch_x.p + static_cast<size_t>(r0) * D;
      gu.x_stride = D;
      gu.batch = nb;
      gu.epilogue = kSwiGLU;
      gu.y = scratch_y.p + static_cast<size_t>(r0) * F;
      gu.y_stride = F;
      RTA_CUDA(launch_gemv(gu, stream));
    }
    RTA_CUDA(cudaMemcpyAsync(a, scratch_y.p, static_cast<size_t>(rows) * F * 4, cudaMemcpyDeviceToHost, stream));
    for (uint32_t r0 = 0; r0 < rows; r0 += 8) {
      const uint32_t nb = std::min(8u, rows - r0);
      GemvArgs dn;
      dn.fmt = L.down_fmt;
      dn.w0 = L.down;
      dn.rows = D;
      dn.cols = F;
      dn.x = scratch_y.p + static_cast<size_t>(r0) * F;
      dn.x_stride = F;
      dn.batch = nb;
      dn.y = scratch_x.p + static_cast<size_t>(r0) * D;  // x no longer needed
      dn.y_stride = D;
      RTA_CUDA(launch_gemv(dn, stream));
    }
    RTA_CUDA(cudaMemcpyAsync(y, scratch_x.p, static_cast<size_t>(rows) * D * 4, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
  }

  void vocabulary(const float* hidden, float* logits, uint32_t* argmax, float* best) {
    invalidate_cache(false);
    require(!team, "diagnostics are served by single-GPU handles", RTA_E_STATE);
    const uint32_t D = this->D(), V = spec.vocabulary_size;
    for (uint32_t i = 0; i < D; ++i) require(std::isfinite(hidden[i]), "vocabulary input must be finite", RTA_E_ARG);
    RTA_CUDA(cudaMemcpyAsync(scratch_x.p, hidden, D * 4ull, cudaMemcpyHostToDevice, stream));
    unsigned long long* key = reinterpret_cast<unsigned long long*>(scratch_y.p);
    RTA_CUDA(cudaMemsetAsync(key, 0, 8, stream));
    DevBuf<float> lg;
    if (logits) lg.alloc(V);
    GemvArgs r;
    r.fmt = lm_fmt;
    r.w0 = lm;
    r.rows = V;
    r.cols = D;
    r.x = scratch_x.p;
    r.y = logits ? lg.p : nullptr;
    r.argmax = key;
    RTA_CUDA(matmul(r, stream));
    unsigned long long k = 0;
    RTA_CUDA(cudaMemcpyAsync(&k, key, 8, cudaMemcpyDeviceToHost, stream));
    if (logits) RTA_CUDA(cudaMemcpyAsync(logits, lg.p, V * 4ull, cudaMemcpyDeviceToHost, stream));
    RTA_CUDA(cudaStreamSynchronize(stream));
    const uint32_t id = ~static_cast<uint32_t>(k & 0xffffffffu);
    require(k != 0 && id < V, "readout produced no valid row", RTA_E_DEVICE_CHECK);
    *argmax = id;
    if (best) {
      const uint32_t ok = static_cast<uint32_t>(k >> 32);
      const uint32_t bits = (ok & 0x80000000u) ? (ok & 0x7fffffffu) : ~ok;
      std::memcpy(best, &bits, 4);
    }
  }
};

rta_status fail_model(const Failure& f) {
  g_model_error = f.msg;
  return f.code;
}

bool read_file(const std::string& path, std::vector<char>& out) {
  std::ifstream f(path, std::ios::binary | std::ios::ate);
  if (!f) return false;
  const std::streamsize n = f.tellg();
  f.seekg(0);
  out.resize(static_cast<size_t>(n));
  return static_cast<bool>(f.read(out.data(), n));
}

}  // namespace
}  // namespace rta

struct rta_model {
  rta::Engine engine;
};

extern "C" {

const char* rta_model_last_error(void) { return rta::g_model_error.c_str(); }

rta_status rta_model_open_ex(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                             const void* matrices, size_t matrix_bytes, const void* basis, size_t basis_bytes,
                             uint32_t capacity, uint32_t sequences, uint32_t flags, int device, rta_model** out) {
  if (!spec || !params || !matrices || !basis || !out) {
    rta::g_model_error = "rta_model_open: null argument";
    return RTA_E_ARG;
  }
  *out = nullptr;
  auto* m = new (std::nothrow) rta_model;
  if (!m) return RTA_E_CUDA;
  try {
    m->engine.load(*spec, params, n_params, matrices, matrix_bytes, basis, basis_bytes, capacity, sequences, flags,
                   device);
  } catch (const rta::Failure& f) {
    delete m;
    return rta::fail_model(f);
  }
  *out = m;
  return RTA_OK;
}

rta_status rta_model_open_team(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                               const void* matrices, size_t matrix_bytes, const void* basis, size_t basis_bytes,
                               uint32_t capacity, uint32_t sequences, const uint32_t* sequence_starts,
                               rta_team* team, uint32_t flags, int device, rta_model** out) {
  if (!spec || !params || !matrices || !basis || !out || !team || !sequence_starts) {
    rta::g_model_error = "rta_model_open_team: null argument";
    return RTA_E_ARG;
  }
  *out = nullptr;
  auto* m = new (std::nothrow) rta_model;
  if (!m) return RTA_E_CUDA;
  try {
    m->engine.load(*spec, params, n_params, matrices, matrix_bytes, basis, basis_bytes, capacity, sequences, flags,
                   device, team, sequence_starts);
  } catch (const rta::Failure& f) {
    delete m;
    return rta::fail_model(f);
  }
  *out = m;
  return RTA_OK;
}

rta_status rta_model_open_batch(const rta_model_spec* spec, const uint32_t* params, size_t n_params,
                                const void* matrices, size_t matrix_bytes, const void* basis, size_t basis_bytes,
                                uint32_t capacity, uint32_t sequences, int device, rta_model** out) {
  return rta_model_open_ex(spec, params, n_params, matrices, matrix_bytes, basis, basis_bytes, capacity, sequences, 0u,
                           device, out);
}

rta_status rta_model_open(const rta_model_spec* spec, const uint32_t* params, size_t n_params, const void* matrices,
                          size_t matrix_bytes, const void* basis, size_t basis_bytes, uint32_t capacity, int device,
                          rta_model** out) {
  return rta_model_open_batch(spec, params, n_params, matrices, matrix_bytes, basis, basis_bytes, capacity, 1u, device,
                              out);
}

rta_status rta_model_open_files(const rta_model_spec* spec, const char* optical_model_bin, const char* geometry_bin,
                                const char* vocabulary_bin, uint32_t capacity, int device, rta_model** out) {
  return rta_model_open_files_ex(spec, optical_model_bin, geometry_bin, vocabulary_bin, capacity, 1u, 0u, device, out);
}

rta_status rta_model_open_files_ex(const rta_model_spec* spec, const char* optical_model_bin,
                                   const char* geometry_bin, const char* vocabulary_bin, uint32_t capacity,
                                   uint32_t sequences, uint32_t flags, int device, rta_model** out) {
  if (!spec || !optical_model_bin || !geometry_bin || !vocabulary_bin || !out) {
    rta::g_model_error = "rta_model_open_files: null argument";
    return RTA_E_ARG;
  }
  std::vector<char> model, geo, voc;
  if (!rta::read_file(optical_model_bin, model) || !rta::read_file(geometry_bin, geo) ||
      !rta::read_file(vocabulary_bin, voc)) {
    rta::g_model_error = "cannot read the model payload files";
    return RTA_E_ASSET;
  }
  // optical_model.bin: 'RTRES004' + <9I d, depth, depth, middle, V, 4, n_params, matrix_words, 0> + params
  if (model.size() < 44 || std::memcmp(model.data(), "RTRES004", 8) != 0) {
    rta::g_model_error = "optical_model.bin: bad magic";
    return RTA_E_ASSET;
  }
  uint32_t hdr[9];
  std::memcpy(hdr, model.data() + 8, sizeof hdr);
  if (hdr[0] != spec->hidden_size || hdr[1] != spec->depth || hdr[3] != spec->middle_size ||
      hdr[4] != spec->vocabulary_size || model.size() < 44 + static_cast<size_t>(hdr[6]) * 4 ||
      geo.size() < static_cast<size_t>(hdr[7]) * 4) {
    rta::g_model_error = "optical_model.bin header does not match the model spec or the payload sizes";
    return RTA_E_ASSET;
  }
  // vocabulary.bin: 'RTBASQ01' + <2I V, D> + raw rows
  uint32_t vh[2];
  if (voc.size() < 16 || std::memcmp(voc.data(), "RTBASQ01", 8) != 0) {
    rta::g_model_error = "vocabulary.bin: bad magic";
    return RTA_E_ASSET;
  }
  std::memcpy(vh, voc.data() + 8, 8);
  if (vh[0] != spec->vocabulary_size || vh[1] != spec->hidden_size) {
    rta::g_model_error = "vocabulary.bin header does not match the model spec";
    return RTA_E_ASSET;
  }
  return rta_model_open_ex(spec, reinterpret_cast<const uint32_t*>(model.data() + 44), hdr[6], geo.data(),
                           static_cast<size_t>(hdr[7]) * 4, voc.data() + 16, voc.size() - 16, capacity, sequences,
                           flags, device, out);
}

void rta_model_close(rta_model* m) { delete m; }

rta_status rta_model_prefill(rta_model* m, const uint32_t* ids, uint32_t n, const uint32_t stops[2], double* gpu_ms) {
  return rta_model_prefill_checkpoint(m, ids, n, stops, n, gpu_ms);
}

rta_status rta_model_prefill_checkpoint(rta_model* m, const uint32_t* ids, uint32_t n, const uint32_t stops[2],
                                        uint32_t boundary, double* gpu_ms) {
  if (!m || !ids) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    if (m->engine.cache)
      m->engine.prefill_cached(ids, n, stops, boundary);
    else
      m->engine.prefill(ids, n, stops);
    if (gpu_ms) *gpu_ms = m->engine.last_gpu_ms;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_prefill_capture(rta_model* m, const uint32_t* ids, uint32_t n, const uint32_t stops[2],
                                     float* states, float* layers, double* gpu_ms) {
  if (!m || !ids || !states) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.prefill_capture(ids, n, stops, states, layers);
    if (gpu_ms) *gpu_ms = m->engine.last_gpu_ms;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_profile_step(rta_model* m, uint32_t* kinds, double* ms, double* bytes, size_t capacity,
                                  size_t* n_groups) {
  if (!m || !kinds || !ms || !bytes || !n_groups) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.profile_step(kinds, ms, bytes, capacity, n_groups);
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_generate(rta_model* m, uint32_t count, uint32_t* ids, uint32_t* n_out, double* gpu_ms) {
  if (!m) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    if (m->engine.cache && m->engine.cache->ready)
      m->engine.generate_cached(count, ids, n_out);
    else
      m->engine.generate(count, ids, n_out);
    if (gpu_ms) *gpu_ms = m->engine.last_gpu_ms;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_prefill_batch(rta_model* m, const uint32_t* ids, const uint32_t* lengths, uint32_t stride,
                                   const uint32_t stops[2], double* gpu_ms) {
  if (!m || !ids || !lengths) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.invalidate_cache(true);  // the batch calls move the state outside the caches
    m->engine.prefill_batch(ids, lengths, stride, stops);
    if (gpu_ms) *gpu_ms = m->engine.last_gpu_ms;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_seed_history(rta_model* m, const uint32_t* lengths, uint64_t seed) {
  if (!m || !lengths) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.invalidate_cache(true);
    m->engine.seed_history(lengths, seed);
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_generate_batch(rta_model* m, uint32_t count, uint32_t* ids, uint32_t* n_out, double* gpu_ms) {
  if (!m) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.invalidate_cache(true);
    m->engine.generate_batch(count, ids, n_out);
    if (gpu_ms) *gpu_ms = m->engine.last_gpu_ms;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_attention(rta_model* m, uint32_t layer, const float* q, const float* k, const float* v,
                               const float* gate, uint32_t rows, uint32_t count, uint32_t query_start,
                               uint32_t history_start, uint32_t block, float* out, float* phys, uint8_t* packets,
                               uint32_t* receipts, uint32_t* n_records, double* gpu_ms) {
  if (!m || !q || !k || !v || !gate || !out || !phys || !packets || !receipts) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.attention_check(layer, q, k, v, gate, rows, count, query_start, history_start, block, out, phys,
                              packets, receipts, n_records, gpu_ms);
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_debug_attention(rta_model* m, uint32_t seq, float* q, float* gate, float* att,
                                     uint8_t* packets, uint32_t* n_positions) {
  if (!m || !q || !gate || !att || !packets) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    const uint32_t n = m->engine.debug_attention(seq, q, gate, att, packets);
    if (n_positions) *n_positions = n;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_mlp(rta_model* m, uint32_t layer, const float* x, uint32_t rows, float* y, float* act) {
  if (!m || !x || !y || !act) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.mlp(layer, x, rows, y, act);
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_vocabulary(rta_model* m, const float* hidden, float* logits, uint32_t* argmax, float* best) {
  if (!m || !hidden || !argmax) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    m->engine.vocabulary(hidden, logits, argmax, best);
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_state(rta_model* m, float* state, uint32_t* position) {
  if (!m || !state) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    if (m->engine.cache && m->engine.cache->ready) m->engine.materialize();
    RTA_CUDA(cudaMemcpyAsync(state, m->engine.state.p, m->engine.D() * 4ull, cudaMemcpyDeviceToHost,
                             m->engine.stream));
    RTA_CUDA(cudaStreamSynchronize(m->engine.stream));
    if (position) *position = m->engine.position;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_cache_info(rta_model* m, uint64_t* out, size_t n, double* ms) {
  if (!m || (!out && n)) return RTA_E_ARG;
  if (!m->engine.cache) {
    rta::g_model_error = "the handle was opened without RTA_MODEL_CACHE";
    return RTA_E_STATE;
  }
  const auto& c = *m->engine.cache;
  for (size_t i = 0; i < n && i < RTA_CACHE_INFO_WORDS; ++i) out[i] = c.info[i];
  if (ms)
    for (int i = 0; i < 3; ++i) ms[i] = c.ms[i];
  return RTA_OK;
}

rta_status rta_model_finish_history(rta_model* m, uint64_t* saved, uint64_t* tokens, uint64_t* boundaries) {
  if (!m) return RTA_E_ARG;
  if (!m->engine.cache) {
    rta::g_model_error = "the handle was opened without RTA_MODEL_CACHE";
    return RTA_E_STATE;
  }
  try {
    cudaSetDevice(m->engine.device);
    m->engine.finish_history(saved, tokens, boundaries);
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_cache_limit(rta_model* m, uint64_t bytes) {
  if (!m) return RTA_E_ARG;
  if (!m->engine.cache) {
    rta::g_model_error = "the handle was opened without RTA_MODEL_CACHE";
    return RTA_E_STATE;
  }
  try {
    cudaSetDevice(m->engine.device);
    auto& c = *m->engine.cache;
    c.budget = bytes;
    c.info[RTA_CACHE_BYTES] = c.index.evict(bytes, nullptr, nullptr);
    c.info[RTA_CACHE_BOUNDARIES] = c.index.size();
    c.info[RTA_CACHE_EVICTIONS] = c.index.evictions;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_state_address(rta_model* m, uint32_t address[8], uint32_t* position) {
  if (!m || !address) return RTA_E_ARG;
  try {
    cudaSetDevice(m->engine.device);
    const rta::Key256 k = m->engine.state_address();
    for (int i = 0; i < 8; ++i) address[i] = k[i];
    if (position) *position = m->engine.position;
  } catch (const rta::Failure& f) {
    return rta::fail_model(f);
  }
  return RTA_OK;
}

rta_status rta_model_resources(rta_model* m, uint64_t* out, size_t n) {
  if (!m || !out) return RTA_E_ARG;
  const rta::Engine& e = m->engine;
  size_t layer_bytes = 0;
  for (auto& L : e.layers) layer_bytes += L->qkvg.n + L->inproj.n;
  layer_bytes += e.lm_tiled.n;
  const uint64_t v[] = {
      e.payload_bytes,
      layer_bytes,
      e.packet_history ? e.pring.n : e.kcache.n * 2ull + e.vcache.n * 2ull,
      e.rec.n * 4ull + e.conv.n * 4ull,
      e.capacity,
      e.nsplit,
      e.kernels_per_decode,
      e.kernels_per_prefill,
      e.position,
      e.nseq,
      e.panel_matrices,
  };
  for (size_t i = 0; i < n && i < sizeof(v) / sizeof(v[0]); ++i) out[i] = v[i];
  return RTA_OK;
}

}  // extern "C"
