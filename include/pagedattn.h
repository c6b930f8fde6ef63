/*
 * pagedattn.h — C ABI of libpagedattn.so, the B200 (sm_100a) paged-attention
 * hot path of mini-llm-runtime.
 *
 * Conventions for every entry point:
 *   - Pointers are device pointers unless stated otherwise; the caller owns
 *     and allocates every buffer (outputs and workspaces included).  The
 *     library never allocates device memory.
 *   - Strides are in ELEMENTS.  The innermost (head_dim) dimension of every
 *     tensor argument must be contiguous.
 *   - `stream` is a cudaStream_t passed as void*.  Launches are asynchronous
 *     on that stream; no entry point synchronises the host.
 *   - The return value is PA_OK (0) or a negative PA_ERR_* code.  Argument
 *     errors are detected on the host before anything is launched, so a
 *     non-zero return means no device memory was modified.
 *   - Block tables and context lengths are int64 (torch.long), matching the
 *     reference's metadata tensors (model/qwen2.py:566-579).
 *
 * Citations are paths inside the mini-llm-runtime project
 * (src/mini_llm_runtime/...).
 */
#ifndef PAGEDATTN_H_
#define PAGEDATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PA_API __attribute__((visibility("default")))
#else
#define PA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define PA_OK 0
#define PA_ERR_INVALID (-1)     /* bad shape / stride / size argument          */
#define PA_ERR_UNSUPPORTED (-2) /* valid but not implemented (dtype, head_dim) */
#define PA_ERR_CUDA (-3)        /* CUDA runtime reported a launch error        */
#define PA_ERR_WORKSPACE (-4)   /* workspace missing or too small              */
#define PA_ERR_CAPACITY (-5)    /* request exceeds a fixed built-in capacity   */

/* Device-side status codes written into the workspace status word when a
 * bounded wait inside a kernel gives up (never expected in normal runs). */
#define PA_DEVICE_TIMEOUT_TMA 101
#define PA_DEVICE_TIMEOUT_MMA 102
#define PA_DEVICE_TIMEOUT_PEER 103 /* a peer GPU did not raise its flag in time (pa_head_allgather) */

/* Element types (torch dtype mapping in mini_llm_runtime_b200/_lib.py). */
#define PA_DTYPE_F32 0
#define PA_DTYPE_F16 1
#define PA_DTYPE_BF16 2
#define PA_DTYPE_F64 3
#define PA_DTYPE_FP8_E4M3 4 /* KV pools only (torch.float8_e4m3fn), with a scale per pool */

/* Flags of pa_paged_decode_ex. */
#define PA_DECODE_EARLY_INPUTS 1 /* metadata and pools may be read before the PDL wait */
#define PA_DECODE_EARLY_QUERY 2  /* with EARLY_INPUTS: q may be read before it too */

/* Ranks and IPC handle size of the peer head all-gather. */
#define PA_PEER_MAX_RANKS 8
#define PA_IPC_HANDLE_BYTES 64

/* Ints in the control block of pa_chunk_prefill. */
#define PA_PREFILL_CONTROL_INTS 4

/* Human-readable name of a status code (static storage). */
PA_API const char* pa_status_string(int status);

/* ABI version of this library; bumps when a signature changes. */
PA_API int pa_abi_version(void);

/*
 * Batched KV-cache write: scatter rows k[t], v[t] ([num_kv_heads, head_dim])
 * into flat slot slot_mapping[t] of one layer's pools, converting to the pool
 * dtype with round-to-nearest-even exactly as torch's `.to(dtype)` does.
 *
 * Replaces PagedKVCache.write_slots (runtime/paged_kv_cache.py:194-249):
 * the two `index_copy_` calls at :243-249.  The range / duplicate checks at
 * :228-239 stay on the host (the Python mirror runs them before calling).
 *
 * k, v          : [T, Hkv, D] with element strides (s0, s1, s2) of src_dtype
 *                 (F32/F16/BF16/F64), any layout.
 * slot_mapping  : [T] int32 (slot_is_int64 = 0) or int64 (slot_is_int64 = 1)
 * k_pool_layer  : this layer's pool viewed as [num_slots, Hkv, D] contiguous,
 *                 num_slots = num_blocks * block_size (slot = block*bs + off).
 * Slots outside [0, num_slots) are skipped on the device (never written).
 */
PA_API int pa_kv_scatter(const void* k, int64_t k_s0, int64_t k_s1, int64_t k_s2, const void* v, int64_t v_s0,
                  int64_t v_s1, int64_t v_s2, int src_dtype, const void* slot_mapping, int slot_is_int64,
                  int64_t num_tokens, void* k_pool_layer, void* v_pool_layer, int64_t num_slots,
                  int num_kv_heads, int head_dim, int pool_dtype, void* stream);

/*
 * FP8 KV-cache pools (PA_DTYPE_FP8_E4M3, torch.float8_e4m3fn) — a storage
 * format of the reference's PagedKVCache (runtime/paged_kv_cache.py:25-35)
 * that halves the bytes decode streams; the reference has no FP8 pool, so
 * these entry points extend its write_slots / decode / prefill contracts
 * with one scale per pool (k_scale, v_scale > 0, finite): a stored element
 * is clamp(x / scale, -448, 448) rounded to nearest even (the division in
 * FP32), and attention reads it back as element * scale.
 *
 * pa_kv_scatter_fp8: pa_kv_scatter into FP8 pools (any source dtype and
 * strides; slots outside the pool skipped).  Replaces
 * PagedKVCache.write_slots (runtime/paged_kv_cache.py:194-249) for FP8 pools.
 */
PA_API int pa_kv_scatter_fp8(const void* k, int64_t k_s0, int64_t k_s1, int64_t k_s2, const void* v, int64_t v_s0,
                             int64_t v_s1, int64_t v_s2, int src_dtype, const void* slot_mapping, int slot_is_int64,
                             int64_t num_tokens, void* k_pool_layer, void* v_pool_layer, int64_t num_slots,
                             int num_kv_heads, int head_dim, float k_scale, float v_scale, void* stream);

/*
 * pa_paged_decode_ex over FP8 pools: q, out, new_k and new_v in `dtype`
 * (F32 / F16 / BF16); the fused write quantizes the new token exactly as
 * pa_kv_scatter_fp8 does.  BF16/F16 with head_dim 64/128, block_size % 16 == 0
 * and batch <= 1024 run the balanced kernel (FP8 tiles by TMA, dequantized to
 * f16 in shared memory, f16 tensor-core MMAs with FP32 softmax, k_scale
 * folded into the score scale and v_scale into the output); F32 and odd
 * shapes run the CUDA-core kernel.  Workspace as pa_decode_workspace_bytes
 * with dtype = the query dtype.  Replaces paged_attention_decode_batch_parallel
 * (kernels/reference/paged_attention.py:178-254) for FP8 pools.
 */
PA_API int pa_paged_decode_fp8(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k, const void* new_v,
                               const int64_t* slot_mapping, void* k_pool_layer, void* v_pool_layer,
                               int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                               const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                               const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                               int num_q_heads, float scale, int dtype, float k_scale, float v_scale,
                               int partition_tokens, int flags, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Bytes of workspace pa_paged_decode needs for exactly these arguments
 * (0 on invalid arguments).  The workspace holds a status word, the split
 * tickets and FP32 partial results:
 *   [0, 256)                         int status (PA_DEVICE_TIMEOUT_* or 0)
 *   [256, 256 + 4*batch*Hq)          int32 tickets — must read 0 when a call
 *                                    starts; every call leaves them 0
 *   [256 + align256(4*batch*Hq), ..) partials (scratch)
 * Zero the buffer once at allocation; when a later call uses a larger
 * batch*Hq than earlier calls on the same buffer, re-zero its ticket range
 * first (it may hold older partials).  Calls sharing a workspace must be
 * ordered on one stream.
 */
PA_API size_t pa_decode_workspace_bytes(int batch, int num_kv_heads, int num_q_heads, int head_dim, int block_size,
                                        int64_t bt_width, int partition_tokens, int dtype);

/*
 * Batched single-token paged decode with split-KV and a log-sum-exp merge.
 *
 *   out[b, h, :] = softmax(scale * q[b, h] . K_b^T) V_b
 * where K_b, V_b are the first context_lens[b] tokens of sequence b gathered
 * through block_tables[b] from the layer pools [num_blocks, block_size, Hkv, D]
 * and q head h reads KV head h / (Hq / Hkv) (GQA / MQA).
 *
 * Replaces paged_attention_decode_batch_parallel
 * (kernels/reference/paged_attention.py:178-254) — same inputs, same output
 * [B, Hq, D] in the input dtype — and, with partition_tokens > 0, the Triton
 * split-KV stage-1 + merge pair (kernels/triton/paged_attention.py:24-213,
 * :528-700, :1530-1618) generalised to a batch.
 *
 * q            : [B, Hq, D], element strides (q_s0, q_s1), last dim contiguous
 * block_tables : [B, bt_width] int64, row stride bt_stride; entries past a
 *                sequence's last block are ignored (the reference pads -1)
 * context_lens : [B] int64, includes the token being decoded (> 0)
 * out          : [B, Hq, D], element strides (o_s0, o_s1)
 * dtype        : F32, F16 or BF16 for q, pools and out (all the same)
 * partition_tokens : BF16/F16 with head_dim 64/128 and batch <= 1024 take
 *                the balanced kernel whatever its value: the batch's KV is
 *                cut into equal ranges per CTA and the pieces of a sequence
 *                are LSE-merged, so the value (accepted for the Triton
 *                split-KV signature) changes nothing beyond FP32 rounding.
 *                Elsewhere > 0 cuts every sequence into partitions of this
 *                many tokens, LSE-merged; 0 lets the library choose.
 * workspace    : >= pa_decode_workspace_bytes(...) bytes, 256-byte aligned,
 *                see pa_decode_workspace_bytes for the zeroing rule.
 */
PA_API int pa_paged_decode(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer,
                    const void* v_pool_layer, int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                    const int64_t* block_tables, int64_t bt_stride, int64_t bt_width, const int64_t* context_lens,
                    void* out, int64_t o_s0, int64_t o_s1, int batch, int num_q_heads, float scale, int dtype,
                    int partition_tokens, void* workspace, size_t workspace_bytes, void* stream);

/*
 * KV write of the new token fused with batched decode: the effect of
 * pa_kv_scatter(new_k, new_v -> slot_mapping) followed by pa_paged_decode,
 * in one launch where it can be fused.  Replaces the pair the reference runs
 * per layer, PagedKVCache.write_slots (runtime/paged_kv_cache.py:194-249)
 * then paged_attention_decode_batch_parallel
 * (kernels/reference/paged_attention.py:178-254), as called by
 * Qwen2Attention.forward_decode_batch_with_cache (model/qwen2.py:608-621).
 *
 * new_k, new_v : [batch, num_kv_heads, head_dim], contiguous, pool dtype
 * slot_mapping : [batch] int64; slot_mapping[b] must be the slot of
 *                position context_lens[b] - 1 of sequence b's block table
 *                (the reference checks this, qwen2.py:594-600) and the
 *                slots distinct; other sequences must not map that slot
 *                into their context.
 * The decode kernel patches the new token's rows into the K/V it stages and
 * stores them to the pools; the output and the pools end up equal to the
 * unfused pair (bit for bit).  Falls back to the two calls where the fused
 * kernel does not apply (F32, odd head_dim or block size, misalignment).
 * Workspace as for pa_paged_decode with partition_tokens = 0.
 */
PA_API int pa_paged_decode_write(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k, const void* new_v,
                          const int64_t* slot_mapping, void* k_pool_layer, void* v_pool_layer, int64_t num_blocks,
                          int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                          int64_t bt_stride, int64_t bt_width, const int64_t* context_lens, void* out, int64_t o_s0,
                          int64_t o_s1, int batch, int num_q_heads, float scale, int dtype, void* workspace,
                          size_t workspace_bytes, void* stream);

/*
 * pa_paged_decode and pa_paged_decode_write in one entry point, with flags.
 * new_k, new_v and slot_mapping are all NULL (decode only, as
 * pa_paged_decode, partition_tokens as there) or all set (the fused write of
 * pa_paged_decode_write; partition_tokens must be 0).  Replaces the same
 * reference pair as those two entry points
 * (runtime/paged_kv_cache.py:194-249, kernels/reference/paged_attention.py:
 * 178-254, as called by model/qwen2.py:608-621).
 *
 * flags = PA_DECODE_EARLY_INPUTS: the caller vouches that the kernel launched
 * just before this call on `stream` (if any) writes none of context_lens,
 * block_tables, slot_mapping or the pool rows other than the new tokens'.
 * The balanced kernel then reads them (and starts its first K/V copies)
 * before waiting for that kernel under programmatic dependent launch, so its
 * start-up overlaps the previous kernel's tail — e.g. the previous layer's
 * decode in a captured multi-layer step.  q, new_k and new_v are still read,
 * and everything is written, only after the wait.  Without the flag the
 * kernel waits before its first global access.
 *
 * flags |= PA_DECODE_EARLY_QUERY (only with PA_DECODE_EARLY_INPUTS): the
 * caller also vouches that q is complete when the kernel is launched — no
 * kernel that may still be running writes it (q comes from a copy or a
 * kernel the launch is fully ordered after, as in a captured step whose
 * per-layer queries are inputs).  The balanced kernel then loads its first
 * query rows before the wait as well.  Not for a model's layer loop, where
 * the kernel just before computes q.
 */
PA_API int pa_paged_decode_ex(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k, const void* new_v,
                              const int64_t* slot_mapping, void* k_pool_layer, void* v_pool_layer,
                              int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                              const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                              const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                              int num_q_heads, float scale, int dtype, int partition_tokens, int flags,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * pa_paged_decode without a caller-supplied workspace: for callers that
 * cannot allocate device memory (a host runtime that owns every device byte
 * through its own arena, an FFI host with no device allocator, a serving
 * loop that must not let cudaMalloc synchronise the device).  No counterpart
 * in the reference: its decode is PyTorch code that allocates freely.
 *
 * The scratch is a fixed 16 MiB array inside the library (held on every GPU
 * that loads it until exit); calls whose pa_decode_workspace_bytes(...)
 * exceeds 16 MiB return PA_ERR_CAPACITY.  The first call on a device looks
 * the array's address up with cudaGetSymbolAddress, so make it before any
 * stream capture.  Every call clears the scratch's status word and tickets
 * on `stream` and then shares the array: calls that overlap on the GPU race.
 * Arguments and results are those of pa_paged_decode.  Allocates nothing.
 */
PA_API int pa_paged_decode_noalloc(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer,
                                   const void* v_pool_layer, int64_t num_blocks, int block_size, int num_kv_heads,
                                   int head_dim, const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                                   const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                                   int num_q_heads, float scale, int dtype, int partition_tokens, void* stream);

/*
 * Copies the status word of pa_paged_decode_noalloc's built-in scratch to
 * *status_out (host memory) in `stream` order: 0, or PA_DEVICE_TIMEOUT_* when
 * a bounded wait of the last call on this device gave up (its output is then
 * garbage).  Read *status_out after synchronising `stream`.  Allocates
 * nothing; no counterpart in the reference (its decode has no device waits).
 */
PA_API int pa_decode_noalloc_status(int* status_out, void* stream);

/*
 * Self-test of the device-side failure path (no counterpart in the
 * reference): launches one bounded wait on an mbarrier that nothing arrives
 * on.  After limit_ns (1 us .. 2 s) of %globaltimer the wait gives up, writes
 * PA_DEVICE_TIMEOUT_TMA into *status (device int, left alone if already
 * non-zero) and the kernel returns — the same path every kernel here takes
 * when a TMA copy or tensor-core step never completes.  No fault, no hang.
 */
PA_API int pa_selftest_wait_timeout(int* status, int64_t limit_ns, void* stream);

/*
 * Causal chunk-prefill over a paged cache, batched over sequences.
 *
 * Sequence s owns packed query rows [cu_q_lens[s], cu_q_lens[s+1]) of q; its
 * chunk is the last (cu_q_lens[s+1]-cu_q_lens[s]) tokens of a context of
 * context_lens[s] tokens (prefix = context_len - chunk_len).  Query i of the
 * chunk attends to cached keys at absolute positions <= prefix + i.  The
 * chunk's own K/V must already be in the pools (written by pa_kv_scatter).
 *
 * Replaces paged_attention_prefill_chunk_tiled and its dense reference
 * (kernels/reference/paged_attention.py:282-434); the single-request
 * signature is the nseq = 1 case.  BF16/F16 run on tcgen05 tensor cores with
 * the accumulators in tensor memory; F32 runs on CUDA cores.
 *
 * q            : [total_q, Hq, D], element strides (q_s0, q_s1)
 * cu_q_lens    : [num_seqs + 1] int64 (query_start_loc, model_runner.py:14-27)
 * context_lens : [num_seqs] int64
 * block_tables : [num_seqs, bt_width] int64, row stride bt_stride
 * out          : [total_q, Hq, D], element strides (o_s0, o_s1)
 * max_q_len    : upper bound of any chunk length (sizes the work list)
 * control      : optional device int[PA_PREFILL_CONTROL_INTS], all zero
 *                before the first call (may be NULL).  control[0] receives
 *                PA_DEVICE_TIMEOUT_* if a bounded wait of the tensor-core
 *                kernel gives up; control[1..2] are the work-claim counters
 *                of its dynamic schedule, which every call leaves at zero
 *                again.  Calls that share a control block must not overlap
 *                on the GPU (same stream, or ordered by events).  With NULL
 *                the kernel falls back to a static schedule.
 */
PA_API int pa_chunk_prefill(const void* q, int64_t q_s0, int64_t q_s1, const int64_t* cu_q_lens,
                     const int64_t* context_lens, const int64_t* block_tables, int64_t bt_stride,
                     int64_t bt_width, const void* k_pool_layer, const void* v_pool_layer, int64_t num_blocks,
                     int block_size, int num_kv_heads, int head_dim, void* out, int64_t o_s0, int64_t o_s1,
                     int num_seqs, int64_t total_q, int max_q_len, int num_q_heads, float scale, int dtype,
                     int* control, void* stream);

/*
 * pa_chunk_prefill over FP8 pools (q / out in dtype), on CUDA cores.
 * Replaces paged_attention_prefill_chunk_tiled
 * (kernels/reference/paged_attention.py:346-434) for FP8 pools.
 */
PA_API int pa_chunk_prefill_fp8(const void* q, int64_t q_s0, int64_t q_s1, const int64_t* cu_q_lens,
                                const int64_t* context_lens, const int64_t* block_tables, int64_t bt_stride,
                                int64_t bt_width, const void* k_pool_layer, const void* v_pool_layer,
                                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, void* out,
                                int64_t o_s0, int64_t o_s1, int num_seqs, int64_t total_q, int max_q_len,
                                int num_q_heads, float scale, int dtype, float k_scale, float v_scale, void* stream);

/*
 * ModelBatch metadata on the device: positions, KV slots, cumulative query
 * starts, context lengths and padded block tables of one scheduler step.
 *
 * Replaces the tensor assembly of build_model_batch
 * (runtime/model_runner.py:37-143; slots :56-66, padding :117-129).
 * `packed` (device, int64) holds for R = num_requests requests: first
 * scheduled position [R], scheduled tokens [R], block-table offset [R] and
 * length [R], then the concatenated block tables (num_table_entries), then
 * the total_tokens token ids in request order.  Outputs (device, int64):
 * query_start_loc[R + 1], positions[T], context_lens[R] (= position +
 * scheduled), block_tables[R][width] padded with -1, slot_mapping[T],
 * input_token_ids[T].  A position past its request's table gets slot -1
 * and PA_ERR_INVALID in *status (device int, may be null).
 */
PA_API int pa_build_batch_metadata(const int64_t* packed, int num_requests, int64_t num_table_entries,
                                   int64_t total_tokens, int block_size, int64_t width, int64_t* query_start_loc,
                                   int64_t* positions, int64_t* context_lens, int64_t* block_tables,
                                   int64_t* slot_mapping, int64_t* input_token_ids, int* status, void* stream);

/*
 * FP32 P.V accumulator: out[b, d] = sum_n p[b, n] * v[b, n, d] for N = 64,
 * D = 256, contiguous inputs.
 *
 * Replaces paged_attention_accumulator_cuda
 * (kernels/cuda/accumulator.py:21-37 -> paged_attention_accumulator.cu:72-90).
 */
PA_API int pa_accumulate_pv(const float* p, const float* v, float* out, int64_t batch, void* stream);

/*
 * All-gather of attention head outputs over NVLink peer memory, for decode
 * sharded by KV head across the GPUs of one node (rank r of `world` decodes
 * query heads [r*heads_local, (r+1)*heads_local) of every sequence).
 *
 * Replaces, on the KV-head-sharded path, the all-gather of the [B, Hq/g, D]
 * head outputs that torch.distributed / NCCL would run; the reference runs
 * one process on one device (runtime/model_runner.py:146-288) and has no
 * counterpart.  The per-rank decode it follows is
 * paged_attention_decode_batch_parallel (kernels/reference/paged_attention.py:178-254).
 *
 * Each rank allocates one exchange area of pa_peer_gather_bytes(world,
 * B_max * heads_local * head_dim * esize) bytes (256-byte aligned), zeroes it,
 * exports it with pa_ipc_export, and maps every peer's area with
 * pa_ipc_import; `areas` (HOST array of `world` device pointers) holds every
 * rank's area as seen from this process, its own at [rank].  All ranks must
 * have zeroed and mapped all areas before the first call (a host barrier).
 *
 * pa_head_allgather: part [batch, heads_local, head_dim] with element strides
 * (p_s0, p_s1); out [batch, world*heads_local, head_dim] with (o_s0, o_s1);
 * dtype F16/BF16/F32 (head_dim * esize, strides and pointers 16-byte
 * aligned).  One kernel (launched with programmatic dependent launch) stores
 * `part` into `out` and, as 16-byte lines that carry 8 data bytes and the
 * call's number twice, into every peer's area; it then polls its own area
 * until every peer's lines of this call have arrived (bounded: wait_limit_ns,
 * 0 = 500 ms; on expiry the area's status word at byte 136 becomes
 * PA_DEVICE_TIMEOUT_PEER and `out` keeps only the heads that arrived) and
 * decodes them into `out`.  Every rank must make the same sequence of calls;
 * calls on one rank must be ordered on one stream.  CUDA-graph capture works:
 * the call number lives in the area, not in the launch arguments.  After a
 * timeout the exchange is out of step: zero the areas on every rank (between
 * a host barrier and the next call) before reusing them.
 */
PA_API size_t pa_peer_gather_bytes(int world, int64_t slice_bytes);
PA_API int pa_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
PA_API int pa_ipc_import(const void* handle, uint64_t offset, void** dev_ptr_out, void** base_out);
PA_API int pa_ipc_close(void* base);
PA_API int pa_head_allgather(const void* part, int64_t p_s0, int64_t p_s1, int batch, int heads_local, int head_dim,
                             int dtype, int rank, int world, void* const* areas, int64_t area_bytes, void* out,
                             int64_t o_s0, int64_t o_s1, int64_t wait_limit_ns, void* stream);

/*
 * Batched decode with the all-gather of head outputs fused into it, for
 * decode sharded by KV head across `world` GPUs of one node (the exchange of
 * pa_head_allgather, done by the decode's own merge kernel: each of its CTAs
 * stores its finished output rows into every peer's exchange area and polls
 * its own area for the peers' rows of the same sequence and heads).
 *
 * Replaces, on the KV-head-sharded path, paged_attention_decode_batch_parallel
 * (kernels/reference/paged_attention.py:178-254) on this rank's heads
 * followed by an all-gather; the reference has no multi-GPU decode.
 *
 * Arguments as pa_paged_decode_ex (partition_tokens 0; new_k / new_v /
 * slot_mapping all null, or all set for the fused KV write), with `out`
 * pointing at THIS rank's first head inside the [batch, world * num_q_heads,
 * head_dim] output of all ranks (strides o_s0, o_s1 of that tensor): rank q's
 * heads are written num_q_heads * (q - rank) heads away.  num_q_heads and
 * num_kv_heads are this rank's.  `areas` is the host array of every rank's
 * exchange area (see pa_head_allgather; the two share the areas and their
 * call number), each of at least pa_decode_allgather_bytes(...) bytes.  On
 * expiry of a wait (wait_limit_ns, 0 = 500 ms) PA_DEVICE_TIMEOUT_PEER goes to
 * the area's status word and the workspace status word.
 *
 * Returns PA_ERR_UNSUPPORTED, with nothing launched, when the call cannot
 * take the balanced kernel (F32, head_dim other than 64/128, batch > 1024,
 * unaligned views) or when the merge kernel's grid does not fit on the device
 * at once (every CTA waits for its peers, so all must be resident): the
 * caller then decodes with pa_paged_decode_ex and exchanges with
 * pa_head_allgather.  Every rank must make the same sequence of calls.
 */
PA_API size_t pa_decode_allgather_bytes(int batch, int num_kv_heads, int num_q_heads, int head_dim, int world);
PA_API int pa_paged_decode_allgather(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k, const void* new_v,
                                     const int64_t* slot_mapping, void* k_pool_layer, void* v_pool_layer,
                                     int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                                     const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                                     const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                                     int num_q_heads, float scale, int dtype, int flags, int rank, int world,
                                     void* const* areas, int64_t area_bytes, int64_t wait_limit_ns, void* workspace,
                                     size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDATTN_H_ */
