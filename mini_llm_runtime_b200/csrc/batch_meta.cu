// ModelBatch metadata built on the device.
//
// Replaces the tensor assembly of build_model_batch
// (runtime/model_runner.py:37-143): per scheduled token its position and KV
// slot (append_slots, :56-66, a Python loop per token there), the cumulative
// query starts, the context lengths and the block tables padded with -1 to
// the widest table (:117-129).  The host sends one packed int64 buffer of
// per-request numbers, the concatenated block tables and the token ids; one
// CTA per request writes that request's rows of every output.
//
// Packed layout for R requests (int64):
//   [0, R)        first scheduled position (num_computed_tokens)
//   [R, 2R)       scheduled tokens
//   [2R, 3R)      offset of the request's block table in the table area
//   [3R, 4R)      length of that block table
//   [4R, 4R + E)  the block tables, concatenated (E entries)
//   then T token ids, in request order.
// A position beyond its request's block table (the reference raises
// ValueError on the host for it, :58-63) gets slot -1 and records
// PA_ERR_INVALID in *status; the host checks the same condition before the
// launch, so the word only guards callers that skip that check.
#include "common.cuh"

namespace pa {
namespace {

constexpr int kMetaThreads = 256;

__global__ void __launch_bounds__(kMetaThreads) build_batch_metadata_kernel(
    const int64_t* __restrict__ packed, int R, int64_t E, int64_t T, int block_size, int64_t width,
    int64_t* __restrict__ query_start_loc, int64_t* __restrict__ positions, int64_t* __restrict__ context_lens,
    int64_t* __restrict__ block_tables, int64_t* __restrict__ slot_mapping, int64_t* __restrict__ input_token_ids,
    int* status) {
  __shared__ int64_t warp_sums[kMetaThreads / 32];
  const int r = blockIdx.x, tid = threadIdx.x;
  const int64_t* start = packed;
  const int64_t* nsched = packed + R;
  const int64_t* toff = packed + 2 * (int64_t)R;
  const int64_t* tlen = packed + 3 * (int64_t)R;
  const int64_t* tables = packed + 4 * (int64_t)R;
  const int64_t* tokens = tables + E;

  // This request's first packed row: the scheduled tokens of requests before it.
  int64_t part = 0;
  for (int i = tid; i < r; i += kMetaThreads) part += nsched[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  if ((tid & 31) == 0) warp_sums[tid >> 5] = part;
  __syncthreads();
  int64_t q0 = 0;
#pragma unroll
  for (int w = 0; w < kMetaThreads / 32; ++w) q0 += warp_sums[w];

  const int64_t s0 = start[r], n = nsched[r], off = toff[r], len = tlen[r];
  if (tid == 0) {
    query_start_loc[r] = q0;
    if (r == R - 1) query_start_loc[R] = q0 + n;
    context_lens[r] = s0 + n;
  }
  for (int64_t j = tid; j < width; j += kMetaThreads)
    block_tables[(int64_t)r * width + j] = j < len ? tables[off + j] : -1;
  for (int64_t i = tid; i < n; i += kMetaThreads) {
    const int64_t row = q0 + i;
    if (row >= T) break;  // inconsistent counts: the host sized T from the same numbers
    const int64_t pos = s0 + i, lb = pos / block_size;
    positions[row] = pos;
    input_token_ids[row] = tokens[row];
    if (lb < len) {
      slot_mapping[row] = tables[off + lb] * block_size + pos % block_size;
    } else {
      slot_mapping[row] = -1;
      if (status != nullptr) atomicCAS(status, 0, PA_ERR_INVALID);
    }
  }
}

}  // namespace
}  // namespace pa

extern "C" PA_API int pa_build_batch_metadata(const int64_t* packed, int num_requests, int64_t num_table_entries,
                                              int64_t total_tokens, int block_size, int64_t width,
                                              int64_t* query_start_loc, int64_t* positions, int64_t* context_lens,
                                              int64_t* block_tables, int64_t* slot_mapping,
                                              int64_t* input_token_ids, int* status, void* stream) {
  if (num_requests < 0 || num_table_entries < 0 || total_tokens < 0 || width < 0 || block_size <= 0)
    return PA_ERR_INVALID;
  if (num_requests == 0) return PA_OK;
  if (packed == nullptr || query_start_loc == nullptr || context_lens == nullptr ||
      (width > 0 && block_tables == nullptr) ||
      (total_tokens > 0 && (positions == nullptr || slot_mapping == nullptr || input_token_ids == nullptr)))
    return PA_ERR_INVALID;
  pa::build_batch_metadata_kernel<<<num_requests, pa::kMetaThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, num_requests, num_table_entries, total_tokens, block_size, width, query_start_loc, positions,
      context_lens, block_tables, slot_mapping, input_token_ids, status);
  PA_CHECK_LAUNCH();
  return PA_OK;
}
