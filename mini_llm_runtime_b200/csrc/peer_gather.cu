// All-gather of attention head outputs over NVLink peer memory, for decode
// sharded by KV head (rank r of g decodes query heads [r*Hq/g, (r+1)*Hq/g)
// of every sequence and every rank needs all Hq heads).
//
// One kernel does the exchange, in the "low-latency" line format: every
// 16-byte store carries 8 bytes of data and the call's number twice
// ({w0, n, w1, n}), so a receiver knows a line has arrived when both number
// words read n; no fence, flag or second round trip is needed.  Each rank
// stores its [B, Hq/g, D] slice, so encoded, straight into every peer's
// exchange area (16-byte stores through a CUDA IPC mapping of the peer's
// memory), copies it into its own [B, Hq, D] output, then polls its own area
// (bounded) for the peers' lines and decodes them into the output.  The
// slice is a few KB per layer: the exchange is latency-bound, one launch and
// one NVLink crossing.
//
// Exchange area of each rank (one device allocation, mapped on every peer):
//   [0, 128)     reserved
//   [128, 256)   uint32 arrivals (CTAs of the current call past their
//                stores), uint32 calls (calls made), int status
//                (PA_DEVICE_TIMEOUT_PEER after a wait gave up); local use
//   [256, ...)   2 slots x world x 2 * slice bytes of lines; call n uses slot
//                n & 1, so a peer that runs one call ahead writes the other
//                slot, and a line left from call n - 2 reads as not arrived.
//                Call numbers are never 0 (next_call_number), so a line never
//                written since the area was zeroed never reads as arrived.
// A peer can run at most one call ahead: it finishes a call only after it
// has received this rank's lines of that call, which this rank stores only
// after it has finished the call before.
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace pa {
namespace {

constexpr int kGatherThreads = 256;
constexpr int kGatherMaxCtas = 32;  // every CTA of the grid waits: all must be resident at once
constexpr int kAreaHeader = 256;

struct GatherParams {
  const uint8_t* part;
  int64_t p_s0, p_s1;  // bytes
  uint8_t* out;
  int64_t o_s0, o_s1;  // bytes
  uint8_t* areas[PA_PEER_MAX_RANKS];
  int B, hl, row_vecs;  // batch, heads per rank, 16-byte vectors per head row
  int rank, world;
  int64_t slice_bytes;
  uint64_t limit_ns;
};

__device__ __forceinline__ void st_line(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_line(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(kGatherThreads) head_allgather_kernel(GatherParams p) {
  // Launched with PDL right behind the kernel that writes `part`: wait for
  // it, and let the next kernel launch (its own wait orders it after this
  // one) so its start-up overlaps the exchange.
  grid_dep_wait();
  grid_dep_launch();
  uint8_t* mine = p.areas[p.rank];
  uint32_t* arrivals = reinterpret_cast<uint32_t*>(mine + 128);
  uint32_t* calls = arrivals + 1;
  int* status = reinterpret_cast<int*>(mine + 136);
  __shared__ uint32_t call_s;
  if (threadIdx.x == 0) call_s = next_call_number(*reinterpret_cast<volatile uint32_t*>(calls));
  __syncthreads();
  const uint32_t n = call_s;
  const int64_t lines_per_rank = 2 * p.slice_bytes;  // bytes of lines per rank's slice
  const int64_t slot_off = kAreaHeader + (int64_t)(n & 1u) * p.world * lines_per_rank;
  const int64_t units = (int64_t)p.B * p.hl * p.row_vecs;  // 16-byte data vectors of a slice
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;

  // This rank's slice: into its own output, and as lines into every peer's area.
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units; u += stride) {
    const int64_t row = u / p.row_vecs;
    const int v = static_cast<int>(u - row * p.row_vecs);
    const int b = static_cast<int>(row / p.hl), h = static_cast<int>(row - (int64_t)b * p.hl);
    const int4 val = *reinterpret_cast<const int4*>(p.part + b * p.p_s0 + h * p.p_s1 + v * 16);
    *reinterpret_cast<int4*>(p.out + b * p.o_s0 + (int64_t)(p.rank * p.hl + h) * p.o_s1 + v * 16) = val;
    for (int q = 0; q < p.world; ++q) {
      if (q == p.rank) continue;
      uint8_t* line = p.areas[q] + slot_off + p.rank * lines_per_rank + u * 32;
      st_line(line, (uint32_t)val.x, n, (uint32_t)val.y, n);
      st_line(line + 16, (uint32_t)val.z, n, (uint32_t)val.w, n);
    }
  }
  // The call counter advances once every CTA has read it.
  if (threadIdx.x == 0 && atomicAdd(arrivals, 1u) == gridDim.x - 1) {
    *reinterpret_cast<volatile uint32_t*>(arrivals) = 0u;
    *reinterpret_cast<volatile uint32_t*>(calls) = n;
  }
  // The peers' lines, polled (bounded) and decoded into the output.
  const uint8_t* slot = mine + slot_off;
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  for (int r = 0; r < p.world && ok; ++r) {
    if (r == p.rank) continue;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < units && ok; u += stride) {
      const uint8_t* line = slot + r * lines_per_rank + u * 32;
      uint4 a, c;
      for (uint32_t i = 0;; ++i) {
        a = ld_line(line);
        c = ld_line(line + 16);
        if (a.y == n && a.w == n && c.y == n && c.w == n) break;
        if ((i & 63) == 63 && globaltimer_ns() - t0 > p.limit_ns) {
          record_status(status, PA_DEVICE_TIMEOUT_PEER);
          ok = false;
          break;
        }
      }
      if (!ok) break;
      const int64_t row = u / p.row_vecs;
      const int v = static_cast<int>(u - row * p.row_vecs);
      const int b = static_cast<int>(row / p.hl), h = static_cast<int>(row - (int64_t)b * p.hl);
      *reinterpret_cast<int4*>(p.out + b * p.o_s0 + (int64_t)(r * p.hl + h) * p.o_s1 + v * 16) =
          make_int4((int)a.x, (int)a.z, (int)c.x, (int)c.z);
    }
  }
}

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

AddressRangeFn get_address_range() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* q = nullptr;
    cudaDriverEntryPointQueryResult r;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &q, cudaEnableDefault, &r) == cudaSuccess &&
        r == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(q);
  });
  return fn;
}

}  // namespace
}  // namespace pa

extern "C" size_t pa_peer_gather_bytes(int world, int64_t slice_bytes) {
  if (world < 1 || world > PA_PEER_MAX_RANKS || slice_bytes < 0) return 0;
  // Two slots of lines: 32 bytes of lines per 16 bytes of data.
  return static_cast<size_t>(pa::kAreaHeader + 2 * (int64_t)world * 2 * ((slice_bytes + 15) / 16 * 16));
}

extern "C" int pa_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  if (dev_ptr == nullptr || handle_out == nullptr || offset_out == nullptr) return PA_ERR_INVALID;
  pa::AddressRangeFn range = pa::get_address_range();
  if (range == nullptr) return PA_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return PA_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return PA_ERR_CUDA;
  static_assert(sizeof(cudaIpcMemHandle_t) == PA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return PA_OK;
}

extern "C" int pa_ipc_import(const void* handle, uint64_t offset, void** dev_ptr_out, void** base_out) {
  if (handle == nullptr || dev_ptr_out == nullptr || base_out == nullptr) return PA_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return PA_ERR_CUDA;
  *base_out = base;
  *dev_ptr_out = static_cast<uint8_t*>(base) + offset;
  return PA_OK;
}

extern "C" int pa_ipc_close(void* base) {
  if (base == nullptr) return PA_ERR_INVALID;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? PA_OK : PA_ERR_CUDA;
}

extern "C" int pa_head_allgather(const void* part, int64_t p_s0, int64_t p_s1, int batch, int heads_local,
                                 int head_dim, int dtype, int rank, int world, void* const* areas,
                                 int64_t area_bytes, void* out, int64_t o_s0, int64_t o_s1, int64_t wait_limit_ns,
                                 void* stream) {
  using namespace pa;
  const int es = dtype_size(dtype);
  if (part == nullptr || out == nullptr || areas == nullptr || es == 0) return PA_ERR_INVALID;
  if (batch < 0 || heads_local <= 0 || head_dim <= 0 || world < 1 || world > PA_PEER_MAX_RANKS || rank < 0 ||
      rank >= world)
    return PA_ERR_INVALID;
  const int64_t row_bytes = (int64_t)head_dim * es;
  if (row_bytes % 16 || (p_s0 * es) % 16 || (p_s1 * es) % 16 || (o_s0 * es) % 16 || (o_s1 * es) % 16 ||
      (reinterpret_cast<uintptr_t>(part) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return PA_ERR_INVALID;
  if (wait_limit_ns < 0 || wait_limit_ns > 2000000000LL) return PA_ERR_INVALID;
  GatherParams p{};
  p.slice_bytes = (int64_t)batch * heads_local * row_bytes;
  if ((size_t)area_bytes < pa_peer_gather_bytes(world, p.slice_bytes)) return PA_ERR_CAPACITY;
  for (int r = 0; r < world; ++r) {
    if (areas[r] == nullptr || (reinterpret_cast<uintptr_t>(areas[r]) & 255)) return PA_ERR_INVALID;
    p.areas[r] = static_cast<uint8_t*>(areas[r]);
  }
  p.part = static_cast<const uint8_t*>(part);
  p.p_s0 = p_s0 * es;
  p.p_s1 = p_s1 * es;
  p.out = static_cast<uint8_t*>(out);
  p.o_s0 = o_s0 * es;
  p.o_s1 = o_s1 * es;
  p.B = batch;
  p.hl = heads_local;
  p.row_vecs = static_cast<int>(row_bytes / 16);
  p.rank = rank;
  p.world = world;
  p.limit_ns = wait_limit_ns == 0 ? kWaitLimitNs : static_cast<uint64_t>(wait_limit_ns);
  const int64_t units = (int64_t)batch * heads_local * p.row_vecs;
  // At least 8 vectors per thread: one CTA for slices up to 32 KB.
  int grid = static_cast<int>((units + 8 * kGatherThreads - 1) / (8 * kGatherThreads));
  grid = grid < 1 ? 1 : (grid > kGatherMaxCtas ? kGatherMaxCtas : grid);
  return launch_pdl(head_allgather_kernel, dim3(grid), dim3(kGatherThreads), 0,
                    reinterpret_cast<cudaStream_t>(stream), p);
}
