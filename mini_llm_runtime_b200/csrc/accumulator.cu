// FP32 P.V accumulator: out[b, d] = sum_n p[b, n] * v[b, n, d], N = 64, D = 256.
//
// Same contract as paged_attention_accumulator_cuda
// (kernels/cuda/accumulator.py:21-37, paged_attention_accumulator.cu:15-94):
// contiguous FP32 inputs [B, 64] and [B, 64, 256], output [B, 256].
//
// Layout on B200: the op is a pure stream of v (64 KB per batch row), so it is
// HBM-bound.  One CTA of 256 threads per batch row; thread t owns float4
// column (t & 63) and token quarter (t >> 6) — every warp reads whole 512-byte
// row segments (fully coalesced 16-byte loads, 4 rows in flight per thread).
// The four quarter-sums are added in shared memory in a fixed order.
#include "common.cuh"

namespace pa {
namespace {

constexpr int kN = 64;
constexpr int kD = 256;
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) accumulate_pv_kernel(const float* __restrict__ p,
                                                                 const float* __restrict__ v,
                                                                 float* __restrict__ out) {
  __shared__ float4 part[4][kD / 4];
  const int64_t b = blockIdx.x;
  const int col = threadIdx.x & 63;  // float4 column
  const int quarter = threadIdx.x >> 6;
  const float* pb = p + b * kN + quarter * (kN / 4);
  const float4* vb = reinterpret_cast<const float4*>(v + b * kN * kD) + (int64_t)quarter * (kN / 4) * (kD / 4) + col;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int n = 0; n < kN / 4; ++n) {
    const float w = __ldg(pb + n);
    const float4 x = __ldg(vb + n * (kD / 4));
    acc.x = fmaf(w, x.x, acc.x);
    acc.y = fmaf(w, x.y, acc.y);
    acc.z = fmaf(w, x.z, acc.z);
    acc.w = fmaf(w, x.w, acc.w);
  }
  part[quarter][col] = acc;
  __syncthreads();
  if (threadIdx.x < kD / 4) {
    float4 r = part[0][threadIdx.x];
#pragma unroll
    for (int q = 1; q < 4; ++q) {
      const float4 y = part[q][threadIdx.x];
      r.x += y.x;
      r.y += y.y;
      r.z += y.z;
      r.w += y.w;
    }
    reinterpret_cast<float4*>(out + b * kD)[threadIdx.x] = r;
  }
}

}  // namespace
}  // namespace pa

extern "C" int pa_accumulate_pv(const float* p, const float* v, float* out, int64_t batch, void* stream) {
  if (batch < 0) return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  if (p == nullptr || v == nullptr || out == nullptr) return PA_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(v) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(p) & 3))
    return PA_ERR_INVALID;
  if (batch > 0x7fffffffLL) return PA_ERR_INVALID;
  pa::accumulate_pv_kernel<<<static_cast<unsigned>(batch), pa::kThreads, 0,
                             reinterpret_cast<cudaStream_t>(stream)>>>(p, v, out);
  PA_CHECK_LAUNCH();
  return PA_OK;
}
