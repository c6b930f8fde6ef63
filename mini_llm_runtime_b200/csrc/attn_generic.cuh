// Parameters shared by the paged-attention launchers.
#pragma once
#include "common.cuh"

namespace pa {

// One "row" is one query token (decode: one per sequence; prefill: one per
// packed chunk token).  Pools are one layer viewed as [num_slots, Hkv, D].
struct GenericParams {
  const void* q;
  int64_t q_s0, q_s1;
  const void* kp;
  const void* vp;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  void* out;
  int64_t o_s0, o_s1;
  const int64_t* context_lens;
  const int64_t* cu_q;  // nullptr for decode
  int num_seqs;
  int64_t num_rows;
  int64_t num_blocks;  // physical blocks per layer; ids outside [0, num_blocks) read as zeros
  int Hq, Hkv, D, bs, group;
  float scale;      // score scale (for FP8 pools already times the K scale)
  float out_scale;  // output factor: 1, or the V scale of an FP8 pool
  int split_tokens, max_splits;
  float* part_ml;  // [rows, Hq, max_splits, 2]
  float* part_o;   // [rows, Hq, max_splits, D]
  int* tickets;    // [rows, Hq]
  int* status;
};

// Workspace layout used by both decode kernels:
//   [0, 256)            int status word (+ padding)
//   tickets             int32[B * Hq]
//   part_ml             float[B * Hq * S * 2]
//   part_o              float[B * Hq * S * D]
struct WorkspaceLayout {
  size_t tickets, part_ml, part_o, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline WorkspaceLayout workspace_layout(int64_t batch, int hq, int d, int splits) {
  WorkspaceLayout w;
  w.tickets = 256;
  w.part_ml = w.tickets + align256(sizeof(int) * (size_t)batch * hq);
  w.part_o = w.part_ml + align256(sizeof(float) * 2 * (size_t)batch * hq * splits);
  w.total = w.part_o + align256(sizeof(float) * (size_t)batch * hq * splits * d);
  return w;
}

// dtype: q / out; kv_dtype: the pools (dtype itself, or PA_DTYPE_FP8_E4M3).
int launch_attn_generic(const GenericParams& p, int dtype, int splits, cudaStream_t st, int kv_dtype = -1);
int generic_chunk_tokens();

}  // namespace pa
