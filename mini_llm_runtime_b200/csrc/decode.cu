// Batched single-token paged decode, split-KV with a log-sum-exp merge.
//
// Replaces paged_attention_decode_batch_parallel
// (kernels/reference/paged_attention.py:178-254) and generalises the Triton
// split-KV pair (kernels/triton/paged_attention.py:528-700 stage 1,
// :1530-1618 merge) to a ragged batch.
//
// Fast path (F16/BF16, head_dim 64 or 128, block_size % 16 == 0) — HBM-bound:
//  * One CTA per (sequence, KV head, split of the context); the whole GQA
//    group of that KV head (up to 16 query heads) rides on every K/V tile, so
//    each K/V byte is read from HBM once per layer.
//  * Each warp streams 16-token sub-blocks of the split (sub-block j of warp w
//    is the split's sub-block w + j*NW).  Lane 0 looks the physical block up
//    in the block table and issues two 3-D TMA boxes {64 dims, 1 head,
//    16 tokens} (K and V, 128-byte swizzle) into the warp's ring of STAGES
//    shared-memory stages, completing an mbarrier — one table load per
//    sub-block, no per-token gathers.
//  * Scores S = Q K^T and O += P V use mma.sync m16n8k16 with FP32
//    accumulators: rows are the group's query heads (padded to 16), so the
//    per-token math costs ~1% of the CUDA-core budget and the kernel stays on
//    the memory roofline.  Online softmax runs in FP32 in the log2 domain
//    (scores pre-multiplied by scale*log2(e), exp2f).
//  * Warps of a CTA are merged through shared memory; splits of a sequence
//    are merged by the CTA that draws the last ticket (atomicAdd on a
//    per-(seq, head-tile) counter, reset by that CTA).  No CTA ever waits for
//    another one.
// Tokens past context_len inside the last block are masked (-inf scores) and
// their V fragments zeroed, so stale or NaN-poisoned slots cannot leak in.
//
// Everything else (F32, other head dims / block sizes) goes to the CUDA-core
// kernel in attn_generic.cu.
#include "attn_generic.cuh"

namespace pa {
namespace {

struct FastParams {
  const void* q;
  int64_t q_s0, q_s1;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  const int64_t* context_lens;
  void* out;
  int64_t o_s0, o_s1;
  int Hq, Hkv, group, bs;
  float scale_log2;
  int split_sub;  // 16-token sub-blocks per split
  int max_splits;
  float* part_ml;
  float* part_o;
  int* tickets;
  int* status;
};

constexpr int kSub = 16;         // tokens per sub-block
constexpr int kTileRowBytes = 128;  // one 64-wide column tile row (SW128 span)
constexpr int kTileBytes = kSub * kTileRowBytes;  // 2 KB

template <int D, int NW, int STAGES>
struct Cfg {
  static constexpr int kColTiles = D / 64;
  static constexpr int kStageBytes = 2 * kColTiles * kTileBytes;  // K + V
  static constexpr int kWarpBytes = STAGES * kStageBytes;
  static constexpr int kKK = D / 16;  // k-steps of S = Q K^T
  static constexpr int kDT = D / 8;   // n-tiles of O = P V
  static constexpr int kMergeFloats = 16 * (D + 2);
  static_assert(kWarpBytes >= kMergeFloats * 4, "merge area must fit in a warp's ring");
  static constexpr size_t kSmem = 1024 + (size_t)NW * kWarpBytes + (size_t)NW * STAGES * 8 + 64;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset inside a 64-col SW128 tile
  return static_cast<uint32_t>(row * kTileRowBytes + ((chunk ^ (row & 7)) << 4));
}

template <typename T, int D, int NW, int STAGES>
__global__ void __launch_bounds__(NW * 32) decode_fast_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                             const __grid_constant__ CUtensorMap tmap_v,
                                                             FastParams p) {
  using C = Cfg<D, NW, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NW * C::kWarpBytes);
  __shared__ int last_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z;
  const int split = blockIdx.x;
  const int head_tiles = (p.group + 15) >> 4;
  const int kvh = blockIdx.y / head_tiles;
  const int ht = blockIdx.y - kvh * head_tiles;
  const int h0 = kvh * p.group + ht * 16;
  const int hn = min(16, p.group - ht * 16);

  int64_t ctx = p.context_lens[b];
  const int64_t cap = p.bt_width * (int64_t)p.bs;
  if (ctx > cap) ctx = cap;
  if (ctx <= 0) return;
  const int nsub = static_cast<int>((ctx + kSub - 1) / kSub);
  const int s0 = split * p.split_sub;
  if (s0 >= nsub) return;
  const int s1 = min(nsub, s0 + p.split_sub);
  const int nsplits = (nsub + p.split_sub - 1) / p.split_sub;
  const int nj = (s1 - s0 > warp) ? (s1 - s0 - warp + NW - 1) / NW : 0;  // sub-blocks of this warp

  uint8_t* ring = smem + warp * C::kWarpBytes;
  uint64_t* wbar = bars + warp * STAGES;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  __syncwarp();

  const int64_t* bt_row = p.bt + (int64_t)b * p.bt_stride;
  auto issue = [&](int j, int stage) {
    const int sb = s0 + warp + j * NW;
    const int64_t tok0 = (int64_t)sb * kSub;
    const int64_t pb = bt_row[tok0 / p.bs];
    const int y = static_cast<int>(pb * p.bs + tok0 % p.bs);
    uint8_t* st = ring + stage * C::kStageBytes;
    mbar_arrive_expect_tx(&wbar[stage], C::kStageBytes);
#pragma unroll
    for (int ct = 0; ct < C::kColTiles; ++ct) {
      tma_load_3d(st + ct * kTileBytes, &tmap_k, &wbar[stage], ct * 64, kvh, y);
      tma_load_3d(st + (C::kColTiles + ct) * kTileBytes, &tmap_v, &wbar[stage], ct * 64, kvh, y);
    }
  };
  if (lane == 0) {
    for (int j = 0; j < STAGES && j < nj; ++j) issue(j, j);
  }

  // Q fragments (A operand, rows = query heads of this tile, padded to 16).
  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_s0;
  const int r0 = lane >> 2, r1 = r0 + 8, cq = 2 * (lane & 3);
  uint32_t qa[C::kKK][4];
#pragma unroll
  for (int kk = 0; kk < C::kKK; ++kk) {
    const int c = kk * 16 + cq;
    qa[kk][0] = r0 < hn ? load_pair_u32(qb + (int64_t)(h0 + r0) * p.q_s1 + c) : 0u;
    qa[kk][1] = r1 < hn ? load_pair_u32(qb + (int64_t)(h0 + r1) * p.q_s1 + c) : 0u;
    qa[kk][2] = r0 < hn ? load_pair_u32(qb + (int64_t)(h0 + r0) * p.q_s1 + c + 8) : 0u;
    qa[kk][3] = r1 < hn ? load_pair_u32(qb + (int64_t)(h0 + r1) * p.q_s1 + c + 8) : 0u;
  }

  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[C::kDT][4];
#pragma unroll
  for (int i = 0; i < C::kDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  const int mi = lane >> 3, mr = lane & 7;  // ldmatrix: matrix index / row inside matrix
  bool ok = true;
  for (int j = 0; j < nj; ++j) {
    const int stage = j % STAGES;
    if (ok) ok = mbar_wait(&wbar[stage], (j / STAGES) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
    const uint32_t kbase = smem_u32(ring + stage * C::kStageBytes);
    const uint32_t vbase = kbase + C::kColTiles * kTileBytes;

    // S = Q K^T for 16 tokens: two n-tiles of 8 tokens.
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < C::kKK; ++kk) {
      const int ct = kk >> 2, kin = kk & 3;
      const int row = (mi >> 1) * 8 + mr;
      const int chunk = 2 * kin + (mi & 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(kbase + ct * kTileBytes + swz(row, chunk), b00, b01, b10, b11);
      MmaOp<T>::run(s[0], qa[kk], b00, b01);
      MmaOp<T>::run(s[1], qa[kk], b10, b11);
    }
    const int valid = static_cast<int>(min((int64_t)kSub, ctx - (int64_t)(s0 + warp + j * NW) * kSub));
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = nt * 8 + cq + (e & 1);
        s[nt][e] = tok < valid ? s[nt][e] * p.scale_log2 : -INFINITY;
      }
    float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - mn0);
      s[nt][1] = exp2f(s[nt][1] - mn0);
      s[nt][2] = exp2f(s[nt][2] - mn1);
      s[nt][3] = exp2f(s[nt][3] - mn1);
    }
    l0 = l0 * a0 + (s[0][0] + s[0][1] + s[1][0] + s[1][1]);
    l1 = l1 * a1 + (s[0][2] + s[0][3] + s[1][2] + s[1][3]);
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < C::kDT; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }
    uint32_t pa[4];
    pa[0] = MmaOp<T>::pack(s[0][0], s[0][1]);
    pa[1] = MmaOp<T>::pack(s[0][2], s[0][3]);
    pa[2] = MmaOp<T>::pack(s[1][0], s[1][1]);
    pa[3] = MmaOp<T>::pack(s[1][2], s[1][3]);

    // O += P V: V fragments via ldmatrix.trans, two head-dim n-tiles per load.
    const bool partial = valid < kSub;
#pragma unroll
    for (int dt = 0; dt < C::kDT; dt += 2) {
      const int dtt = dt + (mi >> 1);
      const int row = (mi & 1) * 8 + mr;
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(vbase + (dtt >> 3) * kTileBytes + swz(row, dtt & 7), v0, v1, v2, v3);
      if (partial) {
        // v0/v2 hold tokens cq, cq+1; v1/v3 hold tokens 8+cq, 9+cq.
        const uint32_t mlo = (cq < valid ? 0x0000ffffu : 0u) | (cq + 1 < valid ? 0xffff0000u : 0u);
        const uint32_t mhi = (cq + 8 < valid ? 0x0000ffffu : 0u) | (cq + 9 < valid ? 0xffff0000u : 0u);
        v0 &= mlo;
        v2 &= mlo;
        v1 &= mhi;
        v3 &= mhi;
      }
      MmaOp<T>::run(o[dt], pa, v0, v1);
      MmaOp<T>::run(o[dt + 1], pa, v2, v3);
    }
    __syncwarp();
    if (lane == 0 && j + STAGES < nj) issue(j + STAGES, stage);
  }

  // Row sums live in 4 lanes each.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // Per-warp (m, l, O) into the warp's own (now idle) ring.
  float* wm = reinterpret_cast<float*>(ring);
  float* wl = wm + 16;
  float* wo = wl + 16;  // [16][D]
  __syncwarp();
  if ((lane & 3) == 0) {
    wm[r0] = m0;
    wl[r0] = l0;
    wm[r1] = m1;
    wl[r1] = l1;
  }
#pragma unroll
  for (int dt = 0; dt < C::kDT; ++dt) {
    const int c = dt * 8 + cq;
    wo[r0 * D + c] = o[dt][0];
    wo[r0 * D + c + 1] = o[dt][1];
    wo[r1 * D + c] = o[dt][2];
    wo[r1 * D + c + 1] = o[dt][3];
  }
  __syncthreads();

  T* out = reinterpret_cast<T*>(p.out);
  const int64_t base_rh = (int64_t)b * p.Hq + h0;
  const bool single = nsplits == 1;
  for (int i = tid; i < hn * D; i += NW * 32) {
    const int h = i / D, d = i - h * D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, reinterpret_cast<float*>(smem + w * C::kWarpBytes)[h]);
    float l = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float* fw = reinterpret_cast<float*>(smem + w * C::kWarpBytes);
      const float mw = fw[h];
      if (mw == -INFINITY) continue;  // warp had no sub-block
      const float sc = exp2f(mw - mx);
      l += sc * fw[16 + h];
      acc += sc * fw[32 + h * D + d];
    }
    if (single) {
      out[(int64_t)b * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d] = Elem<T>::from_f32(acc / l);
    } else {
      p.part_o[((base_rh + h) * p.max_splits + split) * D + d] = acc;
      if (d == 0) {
        p.part_ml[((base_rh + h) * p.max_splits + split) * 2 + 0] = mx;
        p.part_ml[((base_rh + h) * p.max_splits + split) * 2 + 1] = l;
      }
    }
  }
  if (single) return;

  __threadfence();
  __syncthreads();
  int* ticket = p.tickets + (int64_t)b * (p.Hkv * head_tiles) + blockIdx.y;
  if (tid == 0) last_s = (atomicAdd(ticket, 1) == nsplits - 1);
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  for (int i = tid; i < hn * D; i += NW * 32) {
    const int h = i / D, d = i - h * D;
    const float* ml = p.part_ml + (base_rh + h) * p.max_splits * 2;
    float mx = -INFINITY;
    for (int s = 0; s < nsplits; ++s) mx = fmaxf(mx, __ldcg(ml + 2 * s));
    float l = 0.f, acc = 0.f;
    for (int s = 0; s < nsplits; ++s) {
      const float w = exp2f(__ldcg(ml + 2 * s) - mx);
      l += w * __ldcg(ml + 2 * s + 1);
      acc += w * __ldcg(p.part_o + ((base_rh + h) * p.max_splits + s) * D + d);
    }
    out[(int64_t)b * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d] = Elem<T>::from_f32(acc / l);
  }
  if (tid == 0) *ticket = 0;
}

int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

constexpr int kNW = 4;
constexpr int kStages = 4;

template <typename T, int D>
int launch_fast(const FastParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int batch, int splits,
                cudaStream_t st) {
  using C = Cfg<D, kNW, kStages>;
  auto kern = decode_fast_kernel<T, D, kNW, kStages>;
  static bool attr_done[64] = {};  // per instantiation and device
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return PA_ERR_CUDA;
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::kSmem) != cudaSuccess)
      return PA_ERR_CUDA;
    attr_done[dev] = true;
  }
  const int head_tiles = (p.group + 15) / 16;
  dim3 grid(splits, p.Hkv * head_tiles, batch);
  kern<<<grid, kNW * 32, C::kSmem, st>>>(tk, tv, p);
  PA_CHECK_LAUNCH();
  return PA_OK;
}

bool fast_path_ok(int dtype, int D, int bs, int64_t num_blocks, const void* q, int64_t q_s0, int64_t q_s1,
                  const void* kp, const void* vp) {
  if (dtype != PA_DTYPE_BF16 && dtype != PA_DTYPE_F16) return false;
  if (D != 64 && D != 128) return false;
  if (bs % kSub != 0 || bs > 256) return false;
  if (num_blocks * (int64_t)bs >= (int64_t(1) << 31)) return false;
  if ((q_s0 & 1) || (q_s1 & 1) || (reinterpret_cast<uintptr_t>(q) & 3)) return false;
  if ((reinterpret_cast<uintptr_t>(kp) & 15) || (reinterpret_cast<uintptr_t>(vp) & 15)) return false;
  return true;
}

int fast_split_sub(int batch, int hkv, int head_tiles, int64_t bt_width, int bs, int partition_tokens, int sms) {
  const int64_t max_sub = (bt_width * bs + kSub - 1) / kSub;
  int64_t split;
  if (partition_tokens > 0) {
    split = (partition_tokens + kSub - 1) / kSub;
  } else {
    // Size splits so the upper bound of CTAs is ~4 per SM; real ragged
    // batches then land near two resident waves.
    const int64_t units = (int64_t)batch * hkv * head_tiles * max_sub;
    const int64_t target = (int64_t)sms * 4;
    split = (units + target - 1) / target;
    split = (split + kNW - 1) / kNW * kNW;
    if (split < 2 * kNW) split = 2 * kNW;
  }
  if (split > max_sub) split = max_sub;
  if (split < 1) split = 1;
  return static_cast<int>(split);
}

int generic_split_tokens(int batch, int hkv, int head_tiles, int64_t bt_width, int bs, int partition_tokens,
                         int sms) {
  const int chunk = generic_chunk_tokens();
  const int64_t max_tok = bt_width * bs;
  int64_t split;
  if (partition_tokens > 0) {
    split = partition_tokens;
  } else {
    const int64_t ctas = (int64_t)batch * hkv * head_tiles;
    split = ctas >= 2 * sms ? max_tok : 2 * chunk;
  }
  split = (split + chunk - 1) / chunk * chunk;
  if (split > (max_tok + chunk - 1) / chunk * chunk) split = (max_tok + chunk - 1) / chunk * chunk;
  if (split < chunk) split = chunk;
  return static_cast<int>(split);
}

}  // namespace
}  // namespace pa

extern "C" size_t pa_decode_workspace_size(int batch, int num_q_heads, int head_dim, int max_splits) {
  if (batch <= 0 || num_q_heads <= 0 || head_dim <= 0 || max_splits <= 0) return 0;
  return pa::workspace_layout(batch, num_q_heads, head_dim, max_splits).total;
}

extern "C" int pa_decode_num_splits(int batch, int num_kv_heads, int num_q_heads, int head_dim, int block_size,
                                    int64_t bt_width, int partition_tokens, int dtype) {
  using namespace pa;
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || block_size <= 0 || bt_width <= 0)
    return PA_ERR_INVALID;
  const int group = num_q_heads / num_kv_heads;
  const int sms = num_sms(current_device());
  const int64_t max_tok = bt_width * block_size;
  if ((dtype == PA_DTYPE_BF16 || dtype == PA_DTYPE_F16) && (head_dim == 64 || head_dim == 128) &&
      block_size % 16 == 0 && block_size <= 256) {
    const int ht = (group + 15) / 16;
    const int split = fast_split_sub(batch, num_kv_heads, ht, bt_width, block_size, partition_tokens, sms);
    const int64_t max_sub = (max_tok + 15) / 16;
    return static_cast<int>((max_sub + split - 1) / split);
  }
  const int ht = (group + 7) / 8;
  const int split = generic_split_tokens(batch, num_kv_heads, ht, bt_width, block_size, partition_tokens, sms);
  return static_cast<int>((max_tok + split - 1) / split);
}

extern "C" int pa_paged_decode(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer,
                               const void* v_pool_layer, int64_t num_blocks, int block_size, int num_kv_heads,
                               int head_dim, const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                               const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                               int num_q_heads, float scale, int dtype, int partition_tokens, void* workspace,
                               size_t workspace_bytes, void* stream) {
  using namespace pa;
  if (batch < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks <= 0 || bt_width <= 0 || partition_tokens < 0)
    return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  if (q == nullptr || k_pool_layer == nullptr || v_pool_layer == nullptr || block_tables == nullptr ||
      context_lens == nullptr || out == nullptr)
    return PA_ERR_INVALID;
  if (dtype != PA_DTYPE_F32 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16) return PA_ERR_UNSUPPORTED;
  if (batch > 65535) return PA_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int group = num_q_heads / num_kv_heads;
  const int sms = num_sms(current_device());
  const int splits =
      pa_decode_num_splits(batch, num_kv_heads, num_q_heads, head_dim, block_size, bt_width, partition_tokens, dtype);
  if (splits <= 0) return PA_ERR_INVALID;
  if (splits > 65535) return PA_ERR_INVALID;
  const WorkspaceLayout wl = workspace_layout(batch, num_q_heads, head_dim, splits);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  if (splits > 1 && (ws == nullptr || workspace_bytes < wl.total)) return PA_ERR_WORKSPACE;
  if (ws != nullptr && (reinterpret_cast<uintptr_t>(ws) & 255)) return PA_ERR_WORKSPACE;
  int* status = (ws != nullptr && workspace_bytes >= 256) ? reinterpret_cast<int*>(ws) : nullptr;

  if (fast_path_ok(dtype, head_dim, block_size, num_blocks, q, q_s0, q_s1, k_pool_layer, v_pool_layer)) {
    FastParams p;
    p.q = q;
    p.q_s0 = q_s0;
    p.q_s1 = q_s1;
    p.bt = block_tables;
    p.bt_stride = bt_stride;
    p.bt_width = bt_width;
    p.context_lens = context_lens;
    p.out = out;
    p.o_s0 = o_s0;
    p.o_s1 = o_s1;
    p.Hq = num_q_heads;
    p.Hkv = num_kv_heads;
    p.group = group;
    p.bs = block_size;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.split_sub = fast_split_sub(batch, num_kv_heads, (group + 15) / 16, bt_width, block_size, partition_tokens, sms);
    p.max_splits = splits;
    p.part_ml = splits > 1 ? reinterpret_cast<float*>(ws + wl.part_ml) : nullptr;
    p.part_o = splits > 1 ? reinterpret_cast<float*>(ws + wl.part_o) : nullptr;
    p.tickets = splits > 1 ? reinterpret_cast<int*>(ws + wl.tickets) : nullptr;
    p.status = status;
    CUtensorMap tk, tv;
    const uint64_t slots = static_cast<uint64_t>(num_blocks) * block_size;
    const uint64_t s1b = static_cast<uint64_t>(head_dim) * 2;
    const uint64_t s2b = s1b * num_kv_heads;
    if (make_map_3d(&tk, dtype, k_pool_layer, head_dim, num_kv_heads, slots, s1b, s2b, 64, 1, 16,
                    CU_TENSOR_MAP_SWIZZLE_128B) != PA_OK ||
        make_map_3d(&tv, dtype, v_pool_layer, head_dim, num_kv_heads, slots, s1b, s2b, 64, 1, 16,
                    CU_TENSOR_MAP_SWIZZLE_128B) != PA_OK)
      return PA_ERR_CUDA;
    if (dtype == PA_DTYPE_BF16) {
      return head_dim == 64 ? launch_fast<__nv_bfloat16, 64>(p, tk, tv, batch, splits, st)
                            : launch_fast<__nv_bfloat16, 128>(p, tk, tv, batch, splits, st);
    }
    return head_dim == 64 ? launch_fast<__half, 64>(p, tk, tv, batch, splits, st)
                          : launch_fast<__half, 128>(p, tk, tv, batch, splits, st);
  }

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
  g.cu_q = nullptr;
  g.num_seqs = batch;
  g.num_blocks = num_blocks;
  g.num_rows = batch;
  g.Hq = num_q_heads;
  g.Hkv = num_kv_heads;
  g.D = head_dim;
  g.bs = block_size;
  g.group = group;
  g.scale = scale;
  g.split_tokens =
      generic_split_tokens(batch, num_kv_heads, (group + 7) / 8, bt_width, block_size, partition_tokens, sms);
  g.max_splits = splits;
  g.part_ml = splits > 1 ? reinterpret_cast<float*>(ws + wl.part_ml) : nullptr;
  g.part_o = splits > 1 ? reinterpret_cast<float*>(ws + wl.part_o) : nullptr;
  g.tickets = splits > 1 ? reinterpret_cast<int*>(ws + wl.tickets) : nullptr;
  g.status = status;
  return launch_attn_generic(g, dtype, splits, st);
}
