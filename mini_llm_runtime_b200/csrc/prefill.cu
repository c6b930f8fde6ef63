// Causal chunk-prefill over a paged cache (entry point + dispatch).
//
// Replaces paged_attention_prefill_chunk_tiled / _tiled_reference
// (kernels/reference/paged_attention.py:282-434), batched over sequences
// with varlen metadata (cu_q_lens = ModelBatch.query_start_loc,
// runtime/model_runner.py:14-27).  BF16/F16 with head_dim 64 or 128 and block
// sizes that are a multiple of 16 go to the tcgen05 kernel in prefill_tc.cu
// (when the pointers and strides suit its TMA maps); everything
// else (F32 — the CUDA-core path the parity contract asks for — and odd
// shapes) runs the CUDA-core kernel in attn_generic.cu, one query row per
// CTA with context = prefix + i + 1.
#include "attn_generic.cuh"
#include "prefill_tc.cuh"

namespace {
int chunk_prefill_impl(const void* q, int64_t q_s0, int64_t q_s1, const int64_t* cu_q_lens,
                                const int64_t* context_lens, const int64_t* block_tables, int64_t bt_stride,
                                int64_t bt_width, const void* k_pool_layer, const void* v_pool_layer,
                                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, void* out,
                                int64_t o_s0, int64_t o_s1, int num_seqs, int64_t total_q, int max_q_len,
                                int num_q_heads, float scale, int dtype, int* control, void* stream, int kv_dtype,
                                float k_scale, float v_scale) {
  using namespace pa;
  if (num_seqs < 0 || total_q < 0 || max_q_len < 0 || num_kv_heads <= 0 || num_q_heads <= 0 ||
      num_q_heads % num_kv_heads != 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0 || bt_width <= 0)
    return PA_ERR_INVALID;
  if (num_seqs == 0 || total_q == 0) return PA_OK;
  if (q == nullptr || cu_q_lens == nullptr || context_lens == nullptr || block_tables == nullptr ||
      k_pool_layer == nullptr || v_pool_layer == nullptr || out == nullptr)
    return PA_ERR_INVALID;
  if (dtype != PA_DTYPE_F32 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16) return PA_ERR_UNSUPPORTED;
  const bool kv8 = kv_dtype == PA_DTYPE_FP8_E4M3;
  if (kv8 && (!(k_scale > 0.f) || !(v_scale > 0.f) || isinf(k_scale) || isinf(v_scale))) return PA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int group = num_q_heads / num_kv_heads;

  PrefillTcArgs a;
  a.q = q;
  a.q_s0 = q_s0;
  a.q_s1 = q_s1;
  a.cu_q = cu_q_lens;
  a.context_lens = context_lens;
  a.bt = block_tables;
  a.bt_stride = bt_stride;
  a.bt_width = bt_width;
  a.kp = k_pool_layer;
  a.vp = v_pool_layer;
  a.num_blocks = num_blocks;
  a.bs = block_size;
  a.Hkv = num_kv_heads;
  a.Hq = num_q_heads;
  a.group = group;
  a.D = head_dim;
  a.out = out;
  a.o_s0 = o_s0;
  a.o_s1 = o_s1;
  a.num_seqs = num_seqs;
  a.total_q = total_q;
  a.max_q_len = max_q_len;
  a.scale = scale;
  a.dtype = dtype;
  a.control = control;
  // FP8 pools run on CUDA cores (the tensor-core kernel stages 16-bit K/V).
  if (!kv8 && prefill_tc_supported(a)) return launch_prefill_tc(a, st);

  GenericParams g;
  g.q = q;
  g.q_s0 = q_s0;
  g.q_s1 = q_s1;
  g.kp = k_pool_layer;
  g.vp = v_pool_layer;
  g.bt = block_tables;
  g.bt_stride = bt_stride;
  g.bt_width = bt_width;
  g.out = out;
  g.o_s0 = o_s0;
  g.o_s1 = o_s1;
  g.context_lens = context_lens;
  g.cu_q = cu_q_lens;
  g.num_seqs = num_seqs;
  g.num_blocks = num_blocks;
  g.num_rows = total_q;
  g.Hq = num_q_heads;
  g.Hkv = num_kv_heads;
  g.D = head_dim;
  g.bs = block_size;
  g.group = group;
  g.scale = kv8 ? scale * k_scale : scale;
  g.out_scale = kv8 ? v_scale : 1.f;
  // One split covering the whole context: the CTA walks it in chunks.
  const int chunk = generic_chunk_tokens();
  const int64_t max_tok = bt_width * (int64_t)block_size;
  g.split_tokens = static_cast<int>((max_tok + chunk - 1) / chunk * chunk);
  g.max_splits = 1;
  g.part_ml = nullptr;
  g.part_o = nullptr;
  g.tickets = nullptr;
  g.status = nullptr;
  return launch_attn_generic(g, dtype, 1, st, kv8 ? PA_DTYPE_FP8_E4M3 : dtype);
}
}  // namespace

extern "C" int pa_chunk_prefill(const void* q, int64_t q_s0, int64_t q_s1, const int64_t* cu_q_lens,
                                const int64_t* context_lens, const int64_t* block_tables, int64_t bt_stride,
                                int64_t bt_width, const void* k_pool_layer, const void* v_pool_layer,
                                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, void* out,
                                int64_t o_s0, int64_t o_s1, int num_seqs, int64_t total_q, int max_q_len,
                                int num_q_heads, float scale, int dtype, int* control, void* stream) {
  return chunk_prefill_impl(q, q_s0, q_s1, cu_q_lens, context_lens, block_tables, bt_stride, bt_width, k_pool_layer,
                            v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim, out, o_s0, o_s1, num_seqs,
                            total_q, max_q_len, num_q_heads, scale, dtype, control, stream, dtype, 1.f, 1.f);
}

extern "C" int pa_chunk_prefill_fp8(const void* q, int64_t q_s0, int64_t q_s1, const int64_t* cu_q_lens,
                                    const int64_t* context_lens, const int64_t* block_tables, int64_t bt_stride,
                                    int64_t bt_width, const void* k_pool_layer, const void* v_pool_layer,
                                    int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, void* out,
                                    int64_t o_s0, int64_t o_s1, int num_seqs, int64_t total_q, int max_q_len,
                                    int num_q_heads, float scale, int dtype, float k_scale, float v_scale,
                                    void* stream) {
  return chunk_prefill_impl(q, q_s0, q_s1, cu_q_lens, context_lens, block_tables, bt_stride, bt_width, k_pool_layer,
                            v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim, out, o_s0, o_s1, num_seqs,
                            total_q, max_q_len, num_q_heads, scale, dtype, nullptr, stream, PA_DTYPE_FP8_E4M3, k_scale,
                            v_scale);
}
