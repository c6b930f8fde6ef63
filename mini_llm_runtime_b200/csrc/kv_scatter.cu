// Batched KV-cache write (scatter of new K/V rows into flat pool slots).
//
// Mirrors PagedKVCache.write_slots (runtime/paged_kv_cache.py:194-249): the
// layer pool is viewed as [num_slots, Hkv, D] with slot = block*bs + offset
// (:241-244) and row t of k/v goes to slot slot_mapping[t] after a dtype
// conversion equal to `k.to(pool dtype)` (:246-247).  Both K and V are written
// by the same launch.
//
// Two kernels:
//  * scatter_rows_vec: source dtype == pool dtype and each token's [Hkv, D]
//    row contiguous and 16-byte aligned — one 16-byte load/store per thread,
//    K and V handled in the same grid (HBM-bound copy).
//  * scatter_rows_cvt: any strides / any source dtype — element-wise with
//    round-to-nearest-even conversion (f64 goes through f32 like c10 does).
#include "common.cuh"

namespace pa {
namespace {

template <typename I>
__device__ __forceinline__ int64_t load_slot(const void* slots, int64_t t) {
  return static_cast<int64_t>(reinterpret_cast<const I*>(slots)[t]);
}

// One thread per 16-byte chunk of a token row; blockIdx.y selects K (0) or V (1).
template <typename I>
__global__ void scatter_rows_vec(const uint8_t* __restrict__ k, const uint8_t* __restrict__ v, int64_t k_row_bytes,
                                 int64_t v_row_bytes, const void* __restrict__ slots, int64_t num_tokens,
                                 uint8_t* __restrict__ k_pool, uint8_t* __restrict__ v_pool, int64_t num_slots,
                                 int row_chunks) {
  grid_dep_wait();  // PDL launch: the previous kernel has finished
  grid_dep_launch();
  const uint8_t* src = blockIdx.y == 0 ? k : v;
  const int64_t src_row = blockIdx.y == 0 ? k_row_bytes : v_row_bytes;
  uint8_t* dst = blockIdx.y == 0 ? k_pool : v_pool;
  const int64_t total = num_tokens * row_chunks;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / row_chunks;
    const int c = static_cast<int>(i - t * row_chunks);
    const int64_t slot = load_slot<I>(slots, t);
    if (slot < 0 || slot >= num_slots) continue;
    const int4 val = *reinterpret_cast<const int4*>(src + t * src_row + (int64_t)c * 16);
    *reinterpret_cast<int4*>(dst + slot * (int64_t)row_chunks * 16 + (int64_t)c * 16) = val;
  }
}

template <typename S> struct SrcLoad {
  __device__ __forceinline__ static float get(const S* p) { return Elem<S>::to_f32(*p); }
};
template <> struct SrcLoad<double> {
  __device__ __forceinline__ static float get(const double* p) { return static_cast<float>(*p); }
};

template <typename S, typename Dt, typename I>
__global__ void scatter_rows_cvt(const S* __restrict__ k, int64_t ks0, int64_t ks1, int64_t ks2,
                                 const S* __restrict__ v, int64_t vs0, int64_t vs1, int64_t vs2,
                                 const void* __restrict__ slots, int64_t num_tokens, Dt* __restrict__ k_pool,
                                 Dt* __restrict__ v_pool, int64_t num_slots, int hkv, int d) {
  grid_dep_wait();  // PDL launch: the previous kernel has finished
  grid_dep_launch();
  const int64_t row = static_cast<int64_t>(hkv) * d;
  const int64_t total = num_tokens * row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / row;
    const int64_t r = i - t * row;
    const int h = static_cast<int>(r / d);
    const int e = static_cast<int>(r - (int64_t)h * d);
    const int64_t slot = load_slot<I>(slots, t);
    if (slot < 0 || slot >= num_slots) continue;
    const float kv = SrcLoad<S>::get(k + t * ks0 + h * ks1 + e * ks2);
    const float vv = SrcLoad<S>::get(v + t * vs0 + h * vs1 + e * vs2);
    k_pool[slot * row + r] = Elem<Dt>::from_f32(kv);
    v_pool[slot * row + r] = Elem<Dt>::from_f32(vv);
  }
}

// FP8 pools: element = clamp(x / scale, -448, 448) rounded to nearest even,
// the division in FP32 (x converted first, f64 through f32).
template <typename S, typename I>
__global__ void scatter_rows_fp8(const S* __restrict__ k, int64_t ks0, int64_t ks1, int64_t ks2,
                                 const S* __restrict__ v, int64_t vs0, int64_t vs1, int64_t vs2,
                                 const void* __restrict__ slots, int64_t num_tokens, Fp8E4M3* __restrict__ k_pool,
                                 Fp8E4M3* __restrict__ v_pool, int64_t num_slots, int hkv, int d, float k_scale,
                                 float v_scale) {
  grid_dep_wait();  // PDL launch: the previous kernel has finished
  grid_dep_launch();
  const int64_t row = static_cast<int64_t>(hkv) * d;
  const int64_t total = num_tokens * row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / row;
    const int64_t r = i - t * row;
    const int h = static_cast<int>(r / d);
    const int e = static_cast<int>(r - (int64_t)h * d);
    const int64_t slot = load_slot<I>(slots, t);
    if (slot < 0 || slot >= num_slots) continue;
    const float kv = __fdiv_rn(SrcLoad<S>::get(k + t * ks0 + h * ks1 + e * ks2), k_scale);
    const float vv = __fdiv_rn(SrcLoad<S>::get(v + t * vs0 + h * vs1 + e * vs2), v_scale);
    k_pool[slot * row + r] = Elem<Fp8E4M3>::from_f32(kv);
    v_pool[slot * row + r] = Elem<Fp8E4M3>::from_f32(vv);
  }
}

template <typename S>
int launch_fp8_idx(const void* k, int64_t ks0, int64_t ks1, int64_t ks2, const void* v, int64_t vs0, int64_t vs1,
                   int64_t vs2, const void* slots, int slot64, int64_t T, void* kp, void* vp, int64_t num_slots,
                   int hkv, int d, float k_scale, float v_scale, cudaStream_t st) {
  const int64_t total = T * hkv * d;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (slot64)
    return launch_pdl(scatter_rows_fp8<S, int64_t>, dim3((unsigned)blocks), dim3(threads), 0, st, (const S*)k, ks0,
                      ks1, ks2, (const S*)v, vs0, vs1, vs2, slots, T, (Fp8E4M3*)kp, (Fp8E4M3*)vp, num_slots, hkv, d,
                      k_scale, v_scale);
  return launch_pdl(scatter_rows_fp8<S, int32_t>, dim3((unsigned)blocks), dim3(threads), 0, st, (const S*)k, ks0,
                    ks1, ks2, (const S*)v, vs0, vs1, vs2, slots, T, (Fp8E4M3*)kp, (Fp8E4M3*)vp, num_slots, hkv, d,
                    k_scale, v_scale);
}

// f32 -> f32 and f64 -> f32 keep full precision without the float detour
// mattering (identity / single rounding), so the generic kernel is exact.

template <typename S, typename Dt>
int launch_cvt_idx(const void* k, int64_t ks0, int64_t ks1, int64_t ks2, const void* v, int64_t vs0, int64_t vs1,
                   int64_t vs2, const void* slots, int slot64, int64_t T, void* kp, void* vp, int64_t num_slots,
                   int hkv, int d, cudaStream_t st) {
  const int64_t total = T * hkv * d;
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (slot64)
    return launch_pdl(scatter_rows_cvt<S, Dt, int64_t>, dim3((unsigned)blocks), dim3(threads), 0, st, (const S*)k,
                      ks0, ks1, ks2, (const S*)v, vs0, vs1, vs2, slots, T, (Dt*)kp, (Dt*)vp, num_slots, hkv, d);
  return launch_pdl(scatter_rows_cvt<S, Dt, int32_t>, dim3((unsigned)blocks), dim3(threads), 0, st, (const S*)k, ks0,
                    ks1, ks2, (const S*)v, vs0, vs1, vs2, slots, T, (Dt*)kp, (Dt*)vp, num_slots, hkv, d);
}

template <typename Dt>
int launch_cvt_src(int src_dtype, const void* k, int64_t ks0, int64_t ks1, int64_t ks2, const void* v, int64_t vs0,
                   int64_t vs1, int64_t vs2, const void* slots, int slot64, int64_t T, void* kp, void* vp,
                   int64_t num_slots, int hkv, int d, cudaStream_t st) {
  switch (src_dtype) {
    case PA_DTYPE_F32:
      return launch_cvt_idx<float, Dt>(k, ks0, ks1, ks2, v, vs0, vs1, vs2, slots, slot64, T, kp, vp, num_slots, hkv,
                                       d, st);
    case PA_DTYPE_F16:
      return launch_cvt_idx<__half, Dt>(k, ks0, ks1, ks2, v, vs0, vs1, vs2, slots, slot64, T, kp, vp, num_slots, hkv,
                                        d, st);
    case PA_DTYPE_BF16:
      return launch_cvt_idx<__nv_bfloat16, Dt>(k, ks0, ks1, ks2, v, vs0, vs1, vs2, slots, slot64, T, kp, vp,
                                               num_slots, hkv, d, st);
    case PA_DTYPE_F64:
      return launch_cvt_idx<double, Dt>(k, ks0, ks1, ks2, v, vs0, vs1, vs2, slots, slot64, T, kp, vp, num_slots, hkv,
                                        d, st);
    default:
      return PA_ERR_UNSUPPORTED;
  }
}

}  // namespace
}  // namespace pa

extern "C" int pa_kv_scatter_fp8(const void* k, int64_t k_s0, int64_t k_s1, int64_t k_s2, const void* v,
                                 int64_t v_s0, int64_t v_s1, int64_t v_s2, int src_dtype, const void* slot_mapping,
                                 int slot_is_int64, int64_t num_tokens, void* k_pool_layer, void* v_pool_layer,
                                 int64_t num_slots, int num_kv_heads, int head_dim, float k_scale, float v_scale,
                                 void* stream) {
  using namespace pa;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots < 0) return PA_ERR_INVALID;
  if (!(k_scale > 0.f) || !(v_scale > 0.f) || isinf(k_scale) || isinf(v_scale)) return PA_ERR_INVALID;
  if (num_tokens == 0) return PA_OK;
  if (k == nullptr || v == nullptr || slot_mapping == nullptr || k_pool_layer == nullptr || v_pool_layer == nullptr)
    return PA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (src_dtype) {
    case PA_DTYPE_F32:
      return launch_fp8_idx<float>(k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping, slot_is_int64, num_tokens,
                                   k_pool_layer, v_pool_layer, num_slots, num_kv_heads, head_dim, k_scale, v_scale, st);
    case PA_DTYPE_F16:
      return launch_fp8_idx<__half>(k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping, slot_is_int64, num_tokens,
                                    k_pool_layer, v_pool_layer, num_slots, num_kv_heads, head_dim, k_scale, v_scale,
                                    st);
    case PA_DTYPE_BF16:
      return launch_fp8_idx<__nv_bfloat16>(k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping, slot_is_int64,
                                           num_tokens, k_pool_layer, v_pool_layer, num_slots, num_kv_heads, head_dim,
                                           k_scale, v_scale, st);
    case PA_DTYPE_F64:
      return launch_fp8_idx<double>(k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping, slot_is_int64, num_tokens,
                                    k_pool_layer, v_pool_layer, num_slots, num_kv_heads, head_dim, k_scale, v_scale,
                                    st);
    default:
      return PA_ERR_UNSUPPORTED;
  }
}

extern "C" int pa_kv_scatter(const void* k, int64_t k_s0, int64_t k_s1, int64_t k_s2, const void* v, int64_t v_s0,
                             int64_t v_s1, int64_t v_s2, int src_dtype, const void* slot_mapping, int slot_is_int64,
                             int64_t num_tokens, void* k_pool_layer, void* v_pool_layer, int64_t num_slots,
                             int num_kv_heads, int head_dim, int pool_dtype, void* stream) {
  using namespace pa;
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || num_slots < 0) return PA_ERR_INVALID;
  if (num_tokens == 0) return PA_OK;  // empty writes are allowed (paged_kv_cache.py:203)
  if (k == nullptr || v == nullptr || slot_mapping == nullptr || k_pool_layer == nullptr || v_pool_layer == nullptr)
    return PA_ERR_INVALID;
  if (dtype_size(src_dtype) == 0 || dtype_size(pool_dtype) == 0 || pool_dtype == PA_DTYPE_F64 ||
      src_dtype == PA_DTYPE_FP8_E4M3 || pool_dtype == PA_DTYPE_FP8_E4M3)
    return PA_ERR_UNSUPPORTED;  // FP8 pools take pa_kv_scatter_fp8 (they need a scale)
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int es = dtype_size(pool_dtype);
  const int64_t row = static_cast<int64_t>(num_kv_heads) * head_dim;
  const int64_t row_bytes = row * es;

  const bool same = src_dtype == pool_dtype;
  const bool dense = k_s2 == 1 && v_s2 == 1 && k_s1 == head_dim && v_s1 == head_dim;
  const bool aligned = (row_bytes % 16 == 0) && ((k_s0 * es) % 16 == 0) && ((v_s0 * es) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(k) % 16 == 0) && (reinterpret_cast<uintptr_t>(v) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(k_pool_layer) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(v_pool_layer) % 16 == 0);
  if (same && dense && aligned) {
    const int chunks = static_cast<int>(row_bytes / 16);
    const int64_t total = num_tokens * chunks;
    const int threads = 256;
    int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 148 * 16) blocks = 148 * 16;
    dim3 grid(static_cast<unsigned>(blocks), 2);
    if (slot_is_int64)
      return launch_pdl(scatter_rows_vec<int64_t>, grid, dim3(threads), 0, st, (const uint8_t*)k, (const uint8_t*)v,
                        k_s0 * es, v_s0 * es, slot_mapping, num_tokens, (uint8_t*)k_pool_layer,
                        (uint8_t*)v_pool_layer, num_slots, chunks);
    return launch_pdl(scatter_rows_vec<int32_t>, grid, dim3(threads), 0, st, (const uint8_t*)k, (const uint8_t*)v,
                      k_s0 * es, v_s0 * es, slot_mapping, num_tokens, (uint8_t*)k_pool_layer, (uint8_t*)v_pool_layer,
                      num_slots, chunks);
  }
  switch (pool_dtype) {
    case PA_DTYPE_F32:
      return launch_cvt_src<float>(src_dtype, k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping, slot_is_int64,
                                   num_tokens, k_pool_layer, v_pool_layer, num_slots, num_kv_heads, head_dim, st);
    case PA_DTYPE_F16:
      return launch_cvt_src<__half>(src_dtype, k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping, slot_is_int64,
                                    num_tokens, k_pool_layer, v_pool_layer, num_slots, num_kv_heads, head_dim, st);
    case PA_DTYPE_BF16:
      return launch_cvt_src<__nv_bfloat16>(src_dtype, k, k_s0, k_s1, k_s2, v, v_s0, v_s1, v_s2, slot_mapping,
                                           slot_is_int64, num_tokens, k_pool_layer, v_pool_layer, num_slots,
                                           num_kv_heads, head_dim, st);
    default:
      return PA_ERR_UNSUPPORTED;
  }
}
