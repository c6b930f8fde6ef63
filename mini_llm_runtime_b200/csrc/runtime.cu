// Library-wide host helpers: status strings, ABI version, tensor-map
// encoding through the driver entry point, SM count cache.
#include <mutex>

#include "common.cuh"

namespace pa {

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int make_map_3d(CUtensorMap* map, int dtype, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promotion) {
  EncodeTiledFn enc = get_encode_tiled();
  if (enc == nullptr) return PA_ERR_CUDA;
  CUtensorMapDataType t = dtype == PA_DTYPE_BF16        ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                          : dtype == PA_DTYPE_FP8_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, t, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, promotion, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PA_OK : PA_ERR_CUDA;
}

int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (cached[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0) n = 148;
    cached[device] = n;
  }
  return cached[device];
}

// One bounded wait on an mbarrier that nothing ever arrives on: the wait runs
// out after limit_ns and records PA_DEVICE_TIMEOUT_TMA in *status, the path
// every kernel takes when a copy or tensor-core step never completes.
__global__ void wait_timeout_selftest_kernel(int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait(&bar, 0, status, PA_DEVICE_TIMEOUT_TMA, limit_ns);
  }
}

}  // namespace pa

extern "C" int pa_selftest_wait_timeout(int* status, int64_t limit_ns, void* stream) {
  if (status == nullptr || limit_ns < 1000 || limit_ns > 2000000000LL) return PA_ERR_INVALID;
  pa::wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      status, static_cast<uint64_t>(limit_ns));
  PA_CHECK_LAUNCH();
  return PA_OK;
}

extern "C" const char* pa_status_string(int status) {
  switch (status) {
    case PA_OK: return "ok";
    case PA_ERR_INVALID: return "invalid argument";
    case PA_ERR_UNSUPPORTED: return "unsupported configuration";
    case PA_ERR_CUDA: return "CUDA launch error";
    case PA_ERR_WORKSPACE: return "workspace missing or too small";
    case PA_ERR_CAPACITY: return "request exceeds built-in capacity";
    case PA_DEVICE_TIMEOUT_TMA: return "device: bounded wait for a TMA copy gave up";
    case PA_DEVICE_TIMEOUT_MMA: return "device: bounded wait for a tensor-core step gave up";
    case PA_DEVICE_TIMEOUT_PEER: return "device: bounded wait for a peer GPU's flag gave up";
    default: return "unknown status";
  }
}

extern "C" int pa_abi_version(void) { return 3; }
