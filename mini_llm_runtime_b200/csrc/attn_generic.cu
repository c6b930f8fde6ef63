// CUDA-core paged attention for any dtype (F32/F16/BF16), any head_dim up to
// 256, any block size and any GQA group.
//
// This is the FP32 path the parity contract asks for (1e-5 relative against
// the reference's FP32 PyTorch path) and the fallback for shapes the tensor-
// core kernels do not cover (head_dim outside {64, 128}, block sizes that are
// not a multiple of 16).  It serves both entry points:
//   * decode: one query row per sequence, context = context_lens[b]
//     (paged_attention_decode_batch_parallel, reference/paged_attention.py:178-254)
//   * chunk-prefill: one query row per packed chunk token, context of row i
//     = prefix + i + 1, i.e. the causal mask `pos_k <= prefix + i`
//     (paged_attention_prefill_chunk_tiled, reference/paged_attention.py:346-434).
//
// A CTA owns (query row, KV head, head tile of <= 8 query heads, KV split).
// It walks its token range in chunks of kChunk tokens: scores into shared
// memory (one warp per token, lanes across head_dim), FP32 softmax with a
// running max (natural-log domain, expf, like torch.softmax(dtype=float32)),
// then P.V with one thread per (head, dim) pair.  Splits of one row are
// merged by the CTA that takes the last ticket (log-sum-exp merge of
// (m, l, acc) partials, the Triton merge kernel's math at
// kernels/triton/paged_attention.py:1530-1618); nothing ever waits.
#include "attn_generic.cuh"

namespace pa {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxD = 256;
constexpr int kHeadTile = 8;
constexpr int kChunk = 256;
constexpr int kPairsPerThread = kHeadTile * kMaxD / kThreads;  // 16

// T: q / out elements; TK: pool elements (T, or FP8 with scales).
template <typename T, typename TK>
__global__ void __launch_bounds__(kThreads) attn_generic_kernel(GenericParams p) {
  __shared__ float q_s[kHeadTile][kMaxD];
  __shared__ float sc[kHeadTile][kChunk];
  __shared__ float m_s[kHeadTile], l_s[kHeadTile], alpha_s[kHeadTile];
  __shared__ int last_s;

  const int64_t row = blockIdx.x;
  const int head_tiles = (p.group + kHeadTile - 1) / kHeadTile;
  const int kvh = blockIdx.y / head_tiles;
  const int ht = blockIdx.y - kvh * head_tiles;
  const int split = blockIdx.z;
  const int h0 = kvh * p.group + ht * kHeadTile;
  const int hn = min(kHeadTile, p.group - ht * kHeadTile);
  const int D = p.D;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // Which sequence / how many keys this row sees.
  int64_t seq = row, ctx;
  if (p.cu_q == nullptr) {
    ctx = p.context_lens[row];
  } else {
    int lo = 0, hi = p.num_seqs - 1;  // last s with cu_q[s] <= row
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.cu_q[mid] <= row) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    ctx = p.context_lens[lo] - (p.cu_q[lo + 1] - 1 - row);
  }
  const int64_t cap = p.bt_width * (int64_t)p.bs;
  if (ctx > cap) ctx = cap;
  if (ctx <= 0) return;
  const int64_t t_begin = (int64_t)split * p.split_tokens;
  if (t_begin >= ctx) return;
  const int64_t t_end = min(ctx, t_begin + (int64_t)p.split_tokens);
  const int nsplits = static_cast<int>((ctx + p.split_tokens - 1) / p.split_tokens);

  const T* q = reinterpret_cast<const T*>(p.q);
  const TK* kp = reinterpret_cast<const TK*>(p.kp);
  const TK* vp = reinterpret_cast<const TK*>(p.vp);
  const int64_t* bt = p.bt + seq * p.bt_stride;
  const int64_t kv_row = (int64_t)p.Hkv * D;

  for (int i = tid; i < kHeadTile * kMaxD; i += kThreads) {
    const int h = i / kMaxD, d = i - h * kMaxD;
    q_s[h][d] = (h < hn && d < D) ? Elem<T>::to_f32(q[row * p.q_s0 + (int64_t)(h0 + h) * p.q_s1 + d]) : 0.f;
  }
  if (tid < kHeadTile) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  float acc[kPairsPerThread];
#pragma unroll
  for (int i = 0; i < kPairsPerThread; ++i) acc[i] = 0.f;
  __syncthreads();

  for (int64_t c0 = t_begin; c0 < t_end; c0 += kChunk) {
    const int n = static_cast<int>(min((int64_t)kChunk, t_end - c0));
    // Scores: one warp per token, lanes stride head_dim.
    for (int j = warp; j < n; j += kWarps) {
      const int64_t pos = c0 + j;
      const int64_t pb = bt[pos / p.bs];
      const bool in_pool = pb >= 0 && pb < p.num_blocks;
      const TK* krow = kp + (pb * p.bs + pos % p.bs) * kv_row + (int64_t)kvh * D;
      float part[kHeadTile];
#pragma unroll
      for (int h = 0; h < kHeadTile; ++h) part[h] = 0.f;
      for (int d = lane; d < D && in_pool; d += 32) {
        const float kd = Elem<TK>::to_f32(krow[d]);
#pragma unroll
        for (int h = 0; h < kHeadTile; ++h) part[h] = fmaf(q_s[h][d], kd, part[h]);
      }
#pragma unroll
      for (int h = 0; h < kHeadTile; ++h) {
        float s = part[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sc[h][j] = s * p.scale;
      }
    }
    __syncthreads();
    // Running max / sum per head.
    for (int h = warp; h < hn; h += kWarps) {
      float mx = -INFINITY;
      for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc[h][j]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = m_s[h];
      const float m_new = fmaxf(m_old, mx);
      float sum = 0.f;
      for (int j = lane; j < n; j += 32) {
        const float e = expf(sc[h][j] - m_new);
        sc[h][j] = e;
        sum += e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (lane == 0) {
        const float a = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        alpha_s[h] = a;
        l_s[h] = l_s[h] * a + sum;
        m_s[h] = m_new;
      }
    }
    __syncthreads();
    // acc[h][d] = acc * alpha + sum_j p[h][j] * v[j][d]
#pragma unroll
    for (int i = 0; i < kPairsPerThread; ++i) {
      const int h = (tid + i * kThreads) / D;
      if (h < hn) acc[i] *= alpha_s[h];
    }
    for (int j = 0; j < n; ++j) {
      const int64_t pos = c0 + j;
      const int64_t pb = bt[pos / p.bs];
      if (pb < 0 || pb >= p.num_blocks) continue;  // zero V row contributes nothing
      const TK* vrow = vp + (pb * p.bs + pos % p.bs) * kv_row + (int64_t)kvh * D;
#pragma unroll
      for (int i = 0; i < kPairsPerThread; ++i) {
        const int pi = tid + i * kThreads;
        const int h = pi / D, d = pi - h * D;
        if (h < hn) acc[i] = fmaf(sc[h][j], Elem<TK>::to_f32(vrow[d]), acc[i]);
      }
    }
    __syncthreads();
  }

  T* out = reinterpret_cast<T*>(p.out);
  if (nsplits == 1) {
#pragma unroll
    for (int i = 0; i < kPairsPerThread; ++i) {
      const int pi = tid + i * kThreads;
      const int h = pi / D, d = pi - h * D;
      if (h < hn) out[row * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d] = Elem<T>::from_f32(acc[i] * p.out_scale / l_s[h]);
    }
    return;
  }

  // Publish this split's partial, then the CTA holding the last ticket merges.
  const int64_t base_rh = row * p.Hq + h0;  // (row, first head of tile)
#pragma unroll
  for (int i = 0; i < kPairsPerThread; ++i) {
    const int pi = tid + i * kThreads;
    const int h = pi / D, d = pi - h * D;
    if (h < hn) p.part_o[((base_rh + h) * p.max_splits + split) * D + d] = acc[i];
  }
  if (tid < hn) {
    p.part_ml[((base_rh + tid) * p.max_splits + split) * 2 + 0] = m_s[tid];
    p.part_ml[((base_rh + tid) * p.max_splits + split) * 2 + 1] = l_s[tid];
  }
  __threadfence();
  __syncthreads();
  int* ticket = p.tickets + row * ((int64_t)p.Hkv * head_tiles) + blockIdx.y;
  if (tid == 0) last_s = (atomicAdd(ticket, 1) == nsplits - 1);
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  for (int i = tid; i < hn * D; i += kThreads) {
    const int h = i / D, d = i - h * D;
    const float* ml = p.part_ml + (base_rh + h) * p.max_splits * 2;
    float mx = -INFINITY;
    for (int s = 0; s < nsplits; ++s) mx = fmaxf(mx, __ldcg(ml + 2 * s));
    float l = 0.f, o = 0.f;
    for (int s = 0; s < nsplits; ++s) {
      const float w = expf(__ldcg(ml + 2 * s) - mx);
      l += w * __ldcg(ml + 2 * s + 1);
      o += w * __ldcg(p.part_o + ((base_rh + h) * p.max_splits + s) * D + d);
    }
    out[row * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d] = Elem<T>::from_f32(o * p.out_scale / l);
  }
  if (tid == 0) *ticket = 0;  // ready for the next launch on this workspace
}

}  // namespace

int launch_attn_generic(const GenericParams& p, int dtype, int splits, cudaStream_t st, int kv_dtype) {
  if (p.D > kMaxD || p.D <= 0) return PA_ERR_UNSUPPORTED;
  if (p.split_tokens % kChunk != 0 && splits > 1) return PA_ERR_INVALID;
  const int head_tiles = (p.group + kHeadTile - 1) / kHeadTile;
  if (p.num_rows <= 0) return PA_OK;
  if (p.num_rows > 0x7fffffffLL || (int64_t)p.Hkv * head_tiles > 65535 || splits > 65535) return PA_ERR_INVALID;
  dim3 grid(static_cast<unsigned>(p.num_rows), p.Hkv * head_tiles, splits);
  const bool fp8 = kv_dtype == PA_DTYPE_FP8_E4M3;
  if (!fp8 && kv_dtype != -1 && kv_dtype != dtype) return PA_ERR_UNSUPPORTED;
  switch (dtype) {
    case PA_DTYPE_F32:
      if (fp8) attn_generic_kernel<float, Fp8E4M3><<<grid, kThreads, 0, st>>>(p);
      else attn_generic_kernel<float, float><<<grid, kThreads, 0, st>>>(p);
      break;
    case PA_DTYPE_F16:
      if (fp8) attn_generic_kernel<__half, Fp8E4M3><<<grid, kThreads, 0, st>>>(p);
      else attn_generic_kernel<__half, __half><<<grid, kThreads, 0, st>>>(p);
      break;
    case PA_DTYPE_BF16:
      if (fp8) attn_generic_kernel<__nv_bfloat16, Fp8E4M3><<<grid, kThreads, 0, st>>>(p);
      else attn_generic_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
      break;
    default: return PA_ERR_UNSUPPORTED;
  }
  PA_CHECK_LAUNCH();
  return PA_OK;
}

int generic_chunk_tokens() { return kChunk; }

}  // namespace pa
