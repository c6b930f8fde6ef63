// Shared definitions for the paged-attention kernels (sm_100a only).
//
// Everything here is plain CUDA C++ plus inline PTX.  Device helpers cover
// the three data paths the kernels use:
//   * mbarrier + cp.async.bulk.tensor (TMA) for block-table-indirected K/V
//     staging into shared memory,
//   * ldmatrix + mma.sync (m16n8k16, fp32 accumulate) for the small per-block
//     contractions of single-token decode,
//   * element conversions whose rounding matches torch's `Tensor.to(dtype)`
//     (round-to-nearest-even; f64 sources go through f32 first, as c10 does).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/pagedattn.h"

namespace pa {

// ---------------------------------------------------------------------------
// Element types
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  __device__ __forceinline__ static float to_f32(float x) { return x; }
  __device__ __forceinline__ static float from_f32(float x) { return x; }
};
template <> struct Elem<__half> {
  __device__ __forceinline__ static float to_f32(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f32(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};

// FP8 (e4m3, "fn": no infinities, max finite 448) KV-pool element.  Stored
// values are the source divided by the pool's scale, saturated to +-448 and
// rounded to nearest even — clamp(x / scale, -448, 448) cast to
// torch.float8_e4m3fn; a NaN is stored as 0x7f.  Reads return the stored value; the
// kernels apply the scale (to the scores for K, to the output for V).
struct Fp8E4M3 {
  uint8_t bits;
};
template <> struct Elem<Fp8E4M3> {
  __device__ __forceinline__ static float to_f32(Fp8E4M3 x) {
    return __half2float(__half(__nv_cvt_fp8_to_halfraw(x.bits, __NV_E4M3)));
  }
  __device__ __forceinline__ static Fp8E4M3 from_f32(float x) {
    return Fp8E4M3{static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3))};
  }
};

inline int dtype_size(int dt) {
  switch (dt) {
    case PA_DTYPE_F32: return 4;
    case PA_DTYPE_F16: return 2;
    case PA_DTYPE_BF16: return 2;
    case PA_DTYPE_F64: return 8;
    case PA_DTYPE_FP8_E4M3: return 1;
    default: return 0;
  }
}

#define PA_CHECK_LAUNCH()                                   \
  do {                                                      \
    cudaError_t e__ = cudaGetLastError();                   \
    if (e__ != cudaSuccess) return PA_ERR_CUDA;             \
  } while (0)

// ---------------------------------------------------------------------------
// Bounded waits.  Every spin in these kernels gives up after kWaitLimitNs of
// wall-clock time (%globaltimer), records why in the caller-visible status
// word and lets the kernel run to its end, so a lost arrival can never hang
// the GPU.  Legitimate waits (a TMA copy, one tensor-core tile) take
// microseconds.
// ---------------------------------------------------------------------------
constexpr uint64_t kWaitLimitNs = 500ull * 1000 * 1000;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// A waiting thread is suspended in hardware until the phase completes or
// the hint (ns) runs out, so waiting warps do not spin on the issue slots
// their neighbours compute with.
#ifndef PA_WAIT_SUSPEND_NS
#define PA_WAIT_SUSPEND_NS 20000
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(PA_WAIT_SUSPEND_NS)
      : "memory");
  return ok != 0;
}

// Returns false (and records `code`) when the phase did not complete within
// limit_ns (kWaitLimitNs unless a self-test asks for less).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > limit_ns) break;
  }
  record_status(status, code);
  return false;
}

// Same, polling with test_wait (no suspension): for a thread on the
// critical path whose wake-up latency matters more than the issue slots it
// takes while it polls.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 255) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  record_status(status, code);
  return false;
}

// 3-D tiled TMA load into this CTA: the box lands densely in shared memory and
// completes `bar`'s transaction count.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// The same, with an L2 cache policy for the copied lines (from
// createpolicy, e.g. l2_evict_first_policy()).
__device__ __forceinline__ void tma_load_3d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                                 int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// L2 policy for data read once: its lines are the first evicted, so a
// stream does not push out what other accesses will read again.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Number of the next call of a peer exchange, from the last one made: the
// exchange areas start zeroed and the call number marks arrived lines, so it
// is never 0 (after 0xffffffff comes 2, which keeps the slot parity n & 1
// alternating).
__device__ __forceinline__ uint32_t next_call_number(uint32_t last) {
  const uint32_t n = last + 1u;
  return n == 0u ? 2u : n;
}

// Cache hint: bring the 128-byte line holding `ptr` into L2.  It reads no
// value, so it may precede the wait for the kernel that writes the line: that
// write lands in the same L2 line.
__device__ __forceinline__ void prefetch_l2(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(ptr));
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Programmatic dependent launch.  A kernel launched with the
// programmatic-stream-serialization attribute may start while the previous
// kernel in the stream is still running; grid_dep_wait() blocks until that
// kernel has completed and its memory is visible, so every kernel here calls
// it before its first global-memory access.  grid_dep_launch() lets the next
// PDL-launched kernel start early (it still waits for this one to finish).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Warp-level matrix helpers (legacy tensor path; used only by the
// memory-bound decode kernel where the math is a few percent of the budget).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Transpose of an 8x8 matrix of 16-bit elements held in MMA fragment layout
// (lane l: row l / 4, columns 2 (l % 4), +1): lane l receives row l / 4 of
// the transpose.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};
template <> struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// Two adjacent 16-bit elements from global memory as one 32-bit register.
template <typename T>
__device__ __forceinline__ uint32_t load_pair_u32(const T* p) {
  return *reinterpret_cast<const uint32_t*>(p);
}

// ---------------------------------------------------------------------------
// Host: tensor-map creation through the driver entry point (no libcuda link).
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_tiled();

// Encodes a 3-D map of bf16 / f16 / fp8 (as uint8) elements (dims innermost
// first).  Returns PA_OK or
// PA_ERR_CUDA.
int make_map_3d(CUtensorMap* map, int dtype, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promotion = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

int num_sms(int device);

// Launch `kern` on `st` with programmatic stream serialization (PDL) enabled.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? PA_OK : PA_ERR_CUDA;
}

}  // namespace pa
