// Allocation-free variant of the batched paged decode.
//
// Some callers cannot hand the library a workspace: a host runtime that owns
// every device byte through its own arena and forbids stray allocations, an
// FFI host (cgo / JNI / ctypes) that has no device allocator of its own, or a
// latency-critical serving loop where a cudaMalloc would synchronise the
// device.  pa_paged_decode_noalloc serves them with the decode scratch
// (status word, split tickets, FP32 partial results) taken from a fixed
// array compiled into the library, so the call itself allocates nothing.
//
// Set-up: the first call on a device resolves the array's device address
// with cudaGetSymbolAddress (with that device current) and caches it; make
// that first call before any stream capture.  The array is shared by every
// call on a device and keeps the previous call's contents, so each call
// clears the status word and the ticket range it is about to use; calls that
// overlap on the GPU (different streams, no ordering) race on the array.
#include <mutex>

#include "common.cuh"

namespace pa {
namespace {

// Fixed scratch per device that loads this library (held until exit).
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

// Device address of g_decode_scratch on the current device (set up once).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_decode_scratch) != cudaSuccess || ptr == nullptr) return PA_ERR_CUDA;
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return PA_OK;
}

}  // namespace
}  // namespace pa

extern "C" int pa_paged_decode_noalloc(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer,
                                       const void* v_pool_layer, int64_t num_blocks, int block_size,
                                       int num_kv_heads, int head_dim, const int64_t* block_tables,
                                       int64_t bt_stride, int64_t bt_width, const int64_t* context_lens, void* out,
                                       int64_t o_s0, int64_t o_s1, int batch, int num_q_heads, float scale,
                                       int dtype, int partition_tokens, void* stream) {
  using namespace pa;
  if (batch < 0) return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  const size_t need = pa_decode_workspace_bytes(batch, num_kv_heads, num_q_heads, head_dim, block_size, bt_width,
                                                partition_tokens, dtype);
  if (need == 0) return PA_ERR_INVALID;
  if (need > kNoAllocScratchBytes) return PA_ERR_CAPACITY;
  void* scratch = nullptr;
  const int r = scratch_address(&scratch);
  if (r != PA_OK) return r;
  // Status word + split tickets must read zero when the kernels start.
  const size_t clear = 256 + ((sizeof(int) * (size_t)batch * num_q_heads + 255) & ~size_t(255));
  if (cudaMemsetAsync(scratch, 0, clear, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return PA_ERR_CUDA;
  return pa_paged_decode(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim,
                         block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch, num_q_heads, scale,
                         dtype, partition_tokens, scratch, kNoAllocScratchBytes, stream);
}

// The status word of the built-in scratch (0, or PA_DEVICE_TIMEOUT_* when a
// bounded wait of the last pa_paged_decode_noalloc call on this device gave
// up), copied to host memory in stream order.  Allocates nothing.
extern "C" int pa_decode_noalloc_status(int* status_out, void* stream) {
  using namespace pa;
  if (status_out == nullptr) return PA_ERR_INVALID;
  void* scratch = nullptr;
  const int r = scratch_address(&scratch);
  if (r != PA_OK) return r;
  if (cudaMemcpyAsync(status_out, scratch, sizeof(int), cudaMemcpyDeviceToHost,
                      reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return PA_ERR_CUDA;
  return PA_OK;
}
