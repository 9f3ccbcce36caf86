// attention.h -- parameters of the split-K decode attention (attention.cu).
#pragma once
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

namespace rta {

struct AttnParams {
  const float* q = nullptr;      // [nseq][heads][hd] fp32 (normed, rotated)
  size_t q_seq_stride = 0;       // floats between sequences
  const __half* k = nullptr;     // key cache base (fp16)
  const __half* v = nullptr;     // value cache base (fp16)
  size_t seq_stride = 0;         // halves between sequences' caches
  size_t kv_stride = 0;          // halves between KV heads
  size_t pos_stride = 0;         // halves between ring slots
  uint32_t heads = 16, kvh = 4, hd = 256;
  uint32_t capacity = 0;         // ring slots (position p lives in slot p % capacity)
  uint32_t history_start = 0;    // oldest age present
  uint32_t t = 0;                // current absolute time (used when pos == nullptr)
  const uint32_t* pos = nullptr; // device-side current times (graph replay): sequence z reads pos[z * ctrl_step]
  uint32_t ctrl_step = 1;        // u32 elements between sequences' pos / running words
  const float* gate = nullptr;   // [nseq] x ([heads][hd] at gate_seq_stride) or null
  size_t gate_seq_stride = 0;
  float* out = nullptr;          // [nseq][heads][hd]
  size_t out_seq_stride = 0;
  uint32_t rotary_out = 0;       // >0: write outputs in original (un-paired) axis order
  float* phys = nullptr;         // [nseq][heads][2] = (m + 20, Z) or null
  float* part_m = nullptr;       // split records [nseq][kvh][nsplit][4]
  float* part_z = nullptr;
  float* part_o = nullptr;       // [nseq][kvh][nsplit][4][hd]
  uint32_t* err = nullptr;
  const uint32_t* running = nullptr;  // optional: sequence z skipped when running[z * ctrl_step] == 0
  // History packets instead of fp16 K/V (the reference's format): per position
  // kvh Q4_K key blocks then kvh Q6_K value blocks; age a lives in packet row
  // (a - packet_base) % capacity, rows packet_stride bytes apart, sequences
  // packet_seq_stride bytes apart.
  const uint8_t* packets = nullptr;
  size_t packet_seq_stride = 0;
  uint32_t packet_stride = 0, packet_base = 0;
  // 0: splits cut the visible window into equal chunks; > 0: split g covers the
  // g-th newest group of `group_block` positions (the reference's receipt groups).
  uint32_t group_block = 0;
  // fp16 history, several sequences: sequence z uses only the first
  // ceil(n_z * nsplit / capacity) splits of the launch (n_z its visible
  // history), so every split covers about capacity / nsplit positions; the
  // unused splits leave at once and the merge reads only the used records.
  uint32_t split_by_length = 0;
};

size_t attention_smem_bytes(int stages, int warps, int tile);
cudaError_t launch_attention(const AttnParams& p, uint32_t nsplit, uint32_t nseq, bool pdl, cudaStream_t s);
uint32_t attention_default_splits(uint32_t history, uint32_t kvh, int sms);

}  // namespace rta
