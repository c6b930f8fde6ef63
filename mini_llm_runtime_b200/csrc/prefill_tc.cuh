// tcgen05 (5th-gen tensor core) causal chunk-prefill: launcher interface.
#pragma once
#include "common.cuh"

namespace pa {

struct PrefillTcArgs {
  const void* q;
  int64_t q_s0, q_s1;
  const int64_t* cu_q;
  const int64_t* context_lens;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  const void* kp;
  const void* vp;
  int64_t num_blocks;
  int bs, Hkv, Hq, group, D;
  void* out;
  int64_t o_s0, o_s1;
  int num_seqs;
  int64_t total_q;
  int max_q_len;
  float scale;
  int dtype;
  int* control;  // PA_PREFILL_CONTROL_INTS device ints (status, claim, finish), may be null
};

bool prefill_tc_supported(const PrefillTcArgs& a);
int launch_prefill_tc(const PrefillTcArgs& a, cudaStream_t st);

}  // namespace pa
