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

constexpr int kSub = 16;            // tokens per sub-block
constexpr int kTileRowBytes = 128;  // one 64-wide column tile row (SW128 span)
constexpr int kTileBytes = kSub * kTileRowBytes;  // 2 KB

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset inside a 64-col SW128 tile
  return static_cast<uint32_t>(row * kTileRowBytes + ((chunk ^ (row & 7)) << 4));
}

// Online-softmax state of one warp for one (sequence, KV head, head tile):
// rows = up to 16 query heads of the GQA group (mma M dimension), FP32
// (m, l) per row in the log2 domain and the FP32 O accumulator fragments.
template <typename T, int D>
struct WarpState {
  static constexpr int kKK = D / 16;  // k-steps of S = Q K^T
  static constexpr int kDT = D / 8;   // n-tiles of O = P V
  uint32_t qa[kKK][4];
  float m0, m1, l0, l1;
  float o[kDT][4];

  __device__ __forceinline__ void reset() {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int i = 0; i < kDT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }

  // A fragments of Q: rows h0 .. h0+hn-1 of q row qb (padded with zeros).
  __device__ __forceinline__ void load_q(const T* qb, int64_t q_s1, int h0, int hn, int lane) {
    const int r0 = lane >> 2, r1 = r0 + 8, cq = 2 * (lane & 3);
#pragma unroll
    for (int kk = 0; kk < kKK; ++kk) {
      const int c = kk * 16 + cq;
      qa[kk][0] = r0 < hn ? load_pair_u32(qb + (int64_t)(h0 + r0) * q_s1 + c) : 0u;
      qa[kk][1] = r1 < hn ? load_pair_u32(qb + (int64_t)(h0 + r1) * q_s1 + c) : 0u;
      qa[kk][2] = r0 < hn ? load_pair_u32(qb + (int64_t)(h0 + r0) * q_s1 + c + 8) : 0u;
      qa[kk][3] = r1 < hn ? load_pair_u32(qb + (int64_t)(h0 + r1) * q_s1 + c + 8) : 0u;
    }
  }

  // NSUB 16-token sub-blocks staged at kb[u] / vb[u] (SW128 tiles); the
  // first valid[u] tokens of sub-block u belong to the context.  Two
  // sub-blocks per call give two independent MMA chains and one online-
  // softmax rescale per 32 tokens.
  template <int NSUB>
  __device__ __forceinline__ void consume(const uint32_t* kb, const uint32_t* vb, const int* valid, float scale_log2,
                                          int lane) {
    const int mi = lane >> 3, mr = lane & 7, cq = 2 * (lane & 3);
    float s[2 * NSUB][4];
#pragma unroll
    for (int i = 0; i < 2 * NSUB; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kKK; ++kk) {
      const int ct = kk >> 2, kin = kk & 3;
      const int row = (mi >> 1) * 8 + mr;
      const int chunk = 2 * kin + (mi & 1);
#pragma unroll
      for (int u = 0; u < NSUB; ++u) {
        uint32_t b00, b01, b10, b11;
        ldsm_x4(kb[u] + ct * kTileBytes + swz(row, chunk), b00, b01, b10, b11);
        MmaOp<T>::run(s[2 * u], qa[kk], b00, b01);
        MmaOp<T>::run(s[2 * u + 1], qa[kk], b10, b11);
      }
    }
#pragma unroll
    for (int u = 0; u < NSUB; ++u)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = nt * 8 + cq + (e & 1);
          s[2 * u + nt][e] = tok < valid[u] ? s[2 * u + nt][e] * scale_log2 : -INFINITY;
        }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int i = 0; i < 2 * NSUB; ++i) {
      mx0 = fmaxf(mx0, fmaxf(s[i][0], s[i][1]));
      mx1 = fmaxf(mx1, fmaxf(s[i][2], s[i][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float a0 = exp2f(m0 - mn0), a1 = exp2f(m1 - mn1);
    float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
    for (int i = 0; i < 2 * NSUB; ++i) {
      s[i][0] = exp2f(s[i][0] - mn0);
      s[i][1] = exp2f(s[i][1] - mn0);
      s[i][2] = exp2f(s[i][2] - mn1);
      s[i][3] = exp2f(s[i][3] - mn1);
      sum0 += s[i][0] + s[i][1];
      sum1 += s[i][2] + s[i][3];
    }
    l0 = l0 * a0 + sum0;
    l1 = l1 * a1 + sum1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < kDT; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }
#pragma unroll
    for (int u = 0; u < NSUB; ++u) {
      uint32_t pa[4];
      pa[0] = MmaOp<T>::pack(s[2 * u][0], s[2 * u][1]);
      pa[1] = MmaOp<T>::pack(s[2 * u][2], s[2 * u][3]);
      pa[2] = MmaOp<T>::pack(s[2 * u + 1][0], s[2 * u + 1][1]);
      pa[3] = MmaOp<T>::pack(s[2 * u + 1][2], s[2 * u + 1][3]);
      const int vu = valid[u];
      const bool partial = vu < kSub;
      // v0/v2 hold tokens cq, cq+1; v1/v3 hold tokens 8+cq, 9+cq.  Tokens past
      // the context are zeroed so stale / NaN slots cannot reach the sum.
      const uint32_t mlo = (cq < vu ? 0x0000ffffu : 0u) | (cq + 1 < vu ? 0xffff0000u : 0u);
      const uint32_t mhi = (cq + 8 < vu ? 0x0000ffffu : 0u) | (cq + 9 < vu ? 0xffff0000u : 0u);
#pragma unroll
      for (int dt = 0; dt < kDT; dt += 2) {
        const int dtt = dt + (mi >> 1);
        const int row = (mi & 1) * 8 + mr;
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vb[u] + (dtt >> 3) * kTileBytes + swz(row, dtt & 7), v0, v1, v2, v3);
        if (partial) {
          v0 &= mlo;
          v2 &= mlo;
          v1 &= mhi;
          v3 &= mhi;
        }
        MmaOp<T>::run(o[dt], pa, v0, v1);
        MmaOp<T>::run(o[dt + 1], pa, v2, v3);
      }
    }
  }

  // Row sums are spread over the 4 lanes of a quad; gather them, then write
  // rows [0, 16) as records of kRec floats: {m, l, -, -, O[0..D)} (O starts
  // 16-byte aligned so merges read it with float4 loads).
  static constexpr int kRec = D + 4;
  __device__ __forceinline__ void store(float* area, int lane) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const int r0 = lane >> 2, r1 = r0 + 8, cq = 2 * (lane & 3);
    float* a0 = area + r0 * kRec;
    float* a1 = area + r1 * kRec;
    if ((lane & 3) == 0) {
      a0[0] = m0;
      a0[1] = l0;
      a1[0] = m1;
      a1[1] = l1;
    }
#pragma unroll
    for (int dt = 0; dt < kDT; ++dt) {
      const int c = 4 + dt * 8 + cq;
      *reinterpret_cast<float2*>(a0 + c) = make_float2(o[dt][0], o[dt][1]);
      *reinterpret_cast<float2*>(a1 + c) = make_float2(o[dt][2], o[dt][3]);
    }
  }
};

// Merge `nw` warp records (m, l, O) of row h, column d (log2 domain).
template <int D>
__device__ __forceinline__ void merge_records(const float* area, int nw, int h, int d, float& m, float& l,
                                              float& acc) {
  constexpr int kRec = D + 4;
  m = -INFINITY;
  for (int w = 0; w < nw; ++w) m = fmaxf(m, area[(w * 16 + h) * kRec]);
  l = 0.f;
  acc = 0.f;
  for (int w = 0; w < nw; ++w) {
    const float* r = area + (w * 16 + h) * kRec;
    if (r[0] == -INFINITY) continue;  // warp saw no token of this piece
    const float sc = exp2f(r[0] - m);
    l += sc * r[1];
    acc += sc * r[4 + d];
  }
}

// Eight outputs of one row as a single 16-byte store.
template <typename T>
__device__ __forceinline__ void store8(T* dst, const float* v, float scale) {
  int4 pk;
  pk.x = static_cast<int>(MmaOp<T>::pack(v[0] * scale, v[1] * scale));
  pk.y = static_cast<int>(MmaOp<T>::pack(v[2] * scale, v[3] * scale));
  pk.z = static_cast<int>(MmaOp<T>::pack(v[4] * scale, v[5] * scale));
  pk.w = static_cast<int>(MmaOp<T>::pack(v[6] * scale, v[7] * scale));
  *reinterpret_cast<int4*>(dst) = pk;
}

// ===========================================================================
// Balanced ("flattened") decode.  The batch's KV sub-blocks, ordered by
// (sequence, KV head, head tile, position), form one index space of `total`
// sub-blocks; warp g of the grid (W warps in all) owns the slice
// [g*total/W, (g+1)*total/W).  A slice covers pieces of one or more
// segments (segment = one sequence x KV head x head tile).  A segment inside
// one slice is finished by its warp, which writes the output directly; the
// segments cut by a slice's ends (at most its first and last piece) are
// written as (m, l, O) partial records and merged by decode_combine_kernel.
// Warps never wait for one another: no block barrier after the start-up
// scan, no fences, no atomics — under a saturated memory system every such
// round trip costs microseconds.
// ===========================================================================
constexpr int kFlatMaxBatch = 1024;

struct FlatParams {
  const void* q;
  int64_t q_s0, q_s1;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  const int64_t* context_lens;
  void* out;
  int64_t o_s0, o_s1;
  int B, Hq, Hkv, group, HT, SPS, bs;
  float scale_log2;
  int W;           // warps in the grid = slices
  float* part_ml;  // [W][2][16][2]   (m, l) of a slice's first / last cut piece
  float* part_o;   // [W][2][16][D]   unnormalised O of the same
  int* status;
  // Fused KV write (all null when the new token is already in the pools):
  // the new token's K/V rows [B, Hkv, D] (contiguous, pool dtype) replace the
  // pool rows in the staged sub-block and are stored to slots[b] of the pools.
  const void* new_k;
  const void* new_v;
  const int64_t* slots;
  void* k_pool;
  void* v_pool;
  int64_t num_slots;
};

// Segment cursor over the flattened sub-block index space.
struct SegCursor {
  int b, segx;
  int64_t start, end;
  __device__ __forceinline__ void seek(const int* pre, int B, int SPS, int64_t x) {
    int lo = 0, hi = B - 1;  // largest b with pre[b] * SPS <= x
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if ((int64_t)pre[mid] * SPS <= x) lo = mid; else hi = mid - 1;
    }
    b = lo;
    const int64_t base = (int64_t)pre[b] * SPS;
    const int nsub = pre[b + 1] - pre[b];
    segx = static_cast<int>((x - base) / nsub);
    start = base + (int64_t)segx * nsub;
    end = start + nsub;
  }
};

template <int D, int NW, int STAGES>
struct FlatCfg {
  static constexpr int kColTiles = D / 64;
  static constexpr int kStageBytes = 2 * kColTiles * kTileBytes;  // K + V
  static constexpr int kRingBytes = NW * STAGES * kStageBytes;
  static constexpr int kRec = D + 4;                             // record floats per row
  static constexpr int kStagingBytes = NW * 16 * kRec * 4;        // one 16-row record per warp
  static constexpr int kPrefixBytes = (kFlatMaxBatch + 1) * 4;
  static constexpr int kOffStaging = kRingBytes;
  static constexpr int kOffPrefix = kOffStaging + kStagingBytes;
  static constexpr int kOffBars = kOffPrefix + ((kPrefixBytes + 15) & ~15);
  static constexpr size_t kSmem = 1024 + kOffBars + NW * STAGES * 8 + 64;
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

template <typename T, int D, int NW, int STAGES, int CTAS>
__global__ void __launch_bounds__(NW * 32, CTAS) decode_flat_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                                   const __grid_constant__ CUtensorMap tmap_v,
                                                                   FlatParams p) {
  using C = FlatCfg<D, NW, STAGES>;
  static_assert(STAGES >= 2, "pairs of sub-blocks are consumed together");
  constexpr int NT = NW * 32;
  constexpr int kRec = C::kRec;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int* pre = reinterpret_cast<int*>(smem + C::kOffPrefix);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  __shared__ int warp_sums[NW];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t cap = p.bt_width * (int64_t)p.bs;
  // Launched with PDL: wait for the previous kernel before touching global
  // memory; let the combine kernel (and the next PDL kernel) launch early.
  grid_dep_wait();
  grid_dep_launch();

  // ---- prefix sums of per-sequence sub-block counts (block-wide scan) ----
  {
    const int per = (p.B + NT - 1) / NT;
    const int b0 = tid * per;
    static_assert(kFlatMaxBatch <= 16 * NT, "scan chunk");
    int cnt[16];  // per <= kFlatMaxBatch / NT <= 16
    int local = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int b = b0 + i;
      cnt[i] = 0;
      if (i < per && b < p.B) {
        int64_t ctx = p.context_lens[b];
        ctx = ctx > cap ? cap : ctx;
        cnt[i] = ctx > 0 ? static_cast<int>((ctx + kSub - 1) / kSub) : 0;
      }
      local += cnt[i];
    }
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    int run = incl - local;
    for (int w = 0; w < warp; ++w) run += warp_sums[w];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int b = b0 + i;
      if (i < per && b < p.B) {
        pre[b] = run;
        run += cnt[i];
      }
    }
    if (b0 < p.B && b0 + per >= p.B) pre[p.B] = run;
  }
  __syncthreads();
  const int64_t total = (int64_t)pre[p.B] * p.SPS;
  const int g = blockIdx.x * NW + warp;
  const int64_t lo = (int64_t)g * total / p.W, hi = (int64_t)(g + 1) * total / p.W;
  if (lo >= hi) return;  // empty slice (only when total < W); no block barrier follows
  const int nj = static_cast<int>(hi - lo);  // this warp's sub-blocks, contiguous

  uint8_t* ring = smem + warp * STAGES * C::kStageBytes;
  float* staging = reinterpret_cast<float*>(smem + C::kOffStaging) + warp * 16 * kRec;
  uint64_t* wbar = bars + warp * STAGES;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  __syncwarp();

  // Lane i caches the TMA row coordinate and KV head of sub-block tb + i of
  // the slice, so a TMA issue never waits on a block-table load.
  int tb = -32, my_y = 0, my_kvh = 0;
  auto refill = [&](int j) {  // warp-uniform
    tb = j & ~31;
    const int jj = tb + lane;
    if (jj < nj) {
      const int64_t xx = lo + jj;
      SegCursor cur;
      cur.seek(pre, p.B, p.SPS, xx);
      const int64_t tok0 = (xx - cur.start) * kSub;
      const int64_t pb = p.bt[(int64_t)cur.b * p.bt_stride + tok0 / p.bs];
      my_y = static_cast<int>(pb * p.bs + tok0 % p.bs);
      my_kvh = cur.segx / p.HT;
    }
  };
  auto issue = [&](int j) {  // warp-uniform call, lane 0 issues
    if (j >= tb + 32) refill(j);
    const int y = __shfl_sync(0xffffffffu, my_y, j & 31);
    const int kvh = __shfl_sync(0xffffffffu, my_kvh, j & 31);
    if (lane == 0) {
      const int stage = j % STAGES;
      uint8_t* st = ring + stage * C::kStageBytes;
      mbar_arrive_expect_tx(&wbar[stage], C::kStageBytes);
#pragma unroll
      for (int ct = 0; ct < C::kColTiles; ++ct) {
        tma_load_3d(st + ct * kTileBytes, &tmap_k, &wbar[stage], ct * 64, kvh, y);
        tma_load_3d(st + (C::kColTiles + ct) * kTileBytes, &tmap_v, &wbar[stage], ct * 64, kvh, y);
      }
    }
  };
  for (int j = 0; j < STAGES && j < nj; ++j) issue(j);

  const T* qbase = reinterpret_cast<const T*>(p.q);
  T* out = reinterpret_cast<T*>(p.out);
  WarpState<T, D> ws;
  int jc = 0;  // sub-blocks of this slice consumed so far
  bool ok = true;
  SegCursor pc;
  pc.seek(pre, p.B, p.SPS, lo);
  {
    const int kvh = pc.segx / p.HT, ht = pc.segx - kvh * p.HT;
    ws.load_q(qbase + (int64_t)pc.b * p.q_s0, p.q_s1, kvh * p.group + ht * 16, min(16, p.group - ht * 16), lane);
  }
  int64_t x = lo;
  while (x < hi) {
    const int b = pc.b, segx = pc.segx;
    const int kvh = segx / p.HT, ht = segx - kvh * p.HT;
    const int h0 = kvh * p.group + ht * 16, hn = min(16, p.group - ht * 16);
    const int64_t pend = min(pc.end, hi);
    const bool whole = pc.start >= lo && pc.end <= hi;
    const int slot = (x == lo) ? 0 : 1;
    int64_t ctx = p.context_lens[b];
    ctx = ctx > cap ? cap : ctx;
    // The next piece's Q fragments load while this piece streams.
    SegCursor nc = pc;
    uint32_t qn[WarpState<T, D>::kKK][4];
    if (pend < hi) {
      nc.seek(pre, p.B, p.SPS, pend);
      const int kvn = nc.segx / p.HT, htn = nc.segx - kvn * p.HT;
      const int h0n = kvn * p.group + htn * 16, hnn = min(16, p.group - htn * 16);
      const T* qb = qbase + (int64_t)nc.b * p.q_s0;
      const int r0 = lane >> 2, r1 = r0 + 8, cq = 2 * (lane & 3);
#pragma unroll
      for (int kk = 0; kk < WarpState<T, D>::kKK; ++kk) {
        const int cc = kk * 16 + cq;
        qn[kk][0] = r0 < hnn ? load_pair_u32(qb + (int64_t)(h0n + r0) * p.q_s1 + cc) : 0u;
        qn[kk][1] = r1 < hnn ? load_pair_u32(qb + (int64_t)(h0n + r1) * p.q_s1 + cc) : 0u;
        qn[kk][2] = r0 < hnn ? load_pair_u32(qb + (int64_t)(h0n + r0) * p.q_s1 + cc + 8) : 0u;
        qn[kk][3] = r1 < hnn ? load_pair_u32(qb + (int64_t)(h0n + r1) * p.q_s1 + cc + 8) : 0u;
      }
    }
    ws.reset();
    const int jend = static_cast<int>(pend - lo);
    while (jc < jend) {
      const int n = (jend - jc >= 2) ? 2 : 1;
      uint32_t kb[2], vb[2];
      int valid[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (u < n) {
          const int j = jc + u;
          const int stage = j % STAGES;
          if (ok) ok = mbar_wait(&wbar[stage], (j / STAGES) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
          kb[u] = smem_u32(ring + stage * C::kStageBytes);
          vb[u] = kb[u] + C::kColTiles * kTileBytes;
          const int64_t sub = lo + j - pc.start;
          valid[u] = static_cast<int>(min((int64_t)kSub, ctx - sub * kSub));
          if (p.new_k != nullptr && (sub + 1) * kSub >= ctx) {
            // Fused KV write: the sub-block holding the new token (position
            // ctx - 1) gets its K/V rows from new_k / new_v in place of the
            // pool's, and the head-tile-0 warp stores them to the pools.
            // Lane i moves one 16-byte chunk: K then V, 64-column tiles,
            // 8 chunks per 128-byte row (the TMA's 128-byte swizzle).
            const int r = static_cast<int>(ctx - 1 - sub * kSub);
            constexpr int kChunks = 2 * C::kColTiles * 8;
            if (lane < kChunks) {
              const int kv = lane / (C::kColTiles * 8), rem = lane - kv * (C::kColTiles * 8);
              const int ct = rem >> 3, c = rem & 7;
              const int64_t src = ((int64_t)b * p.Hkv + kvh) * D + ct * 64 + c * 8;
              const int4 val = __ldg(reinterpret_cast<const int4*>(
                  reinterpret_cast<const T*>(kv ? p.new_v : p.new_k) + src));
              uint8_t* dst = ring + stage * C::kStageBytes + (kv * C::kColTiles + ct) * kTileBytes + r * 128 +
                             ((c ^ (r & 7)) << 4);
              *reinterpret_cast<int4*>(dst) = val;
              const int64_t slot = p.slots[b];
              if (ht == 0 && slot >= 0 && slot < p.num_slots)
                *reinterpret_cast<int4*>(reinterpret_cast<T*>(kv ? p.v_pool : p.k_pool) +
                                         (slot * p.Hkv + kvh) * D + ct * 64 + c * 8) = val;
              fence_proxy_async_smem();  // before the stage is refilled by TMA
            }
            __syncwarp();
          }
        }
      }
      if (n == 2) ws.template consume<2>(kb, vb, valid, p.scale_log2, lane);
      else ws.template consume<1>(kb, vb, valid, p.scale_log2, lane);
      __syncwarp();
      for (int u = 0; u < n; ++u)
        if (jc + u + STAGES < nj) issue(jc + u + STAGES);
      jc += n;
    }
    // Finish the piece: stage the record in this warp's shared memory, then
    // write it with 16-byte stores (final output, or a partial record).
    ws.store(staging, lane);
    __syncwarp();
    float* pml = p.part_ml + ((int64_t)(g * 2 + slot) * 16) * 2;
    float* po = p.part_o + ((int64_t)(g * 2 + slot) * 16) * D;
    for (int i = lane; i < hn * (D / 8); i += 32) {
      const int h = i / (D / 8), d = 8 * (i - h * (D / 8));
      const float* r = staging + h * kRec;
      const float4 v0 = *reinterpret_cast<const float4*>(r + 4 + d);
      const float4 v1 = *reinterpret_cast<const float4*>(r + 8 + d);
      if (whole) {
        const float vals[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        store8<T>(out + (int64_t)b * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d, vals, 1.f / r[1]);
      } else {
        *reinterpret_cast<float4*>(po + h * D + d) = v0;
        *reinterpret_cast<float4*>(po + h * D + d + 4) = v1;
      }
    }
    if (!whole && lane < hn) *reinterpret_cast<float2*>(pml + lane * 2) = make_float2(staging[lane * kRec], staging[lane * kRec + 1]);
    __syncwarp();
    x = pend;
    if (x < hi) {
      pc = nc;
#pragma unroll
      for (int kk = 0; kk < WarpState<T, D>::kKK; ++kk)
#pragma unroll
        for (int e = 0; e < 4; ++e) ws.qa[kk][e] = qn[kk][e];
    }
  }
}

// Second stage of the balanced decode: every segment (sequence x KV head x
// head tile) cut by slice ends is merged (log-sum-exp) from the partial
// records of the warps g0..g1 owning its first / last sub-block; warps with
// an empty slice (only when the batch has fewer sub-blocks than warps) hold
// none.  One CTA of 256 threads per segment; segments finished inside one
// slice return at once.  Launched with PDL right behind the main kernel; the
// loads of one stage are issued together so a merge costs a few round trips.
constexpr int kCombineThreads = 256;
// At most 64 registers (4 CTAs' worth per SM): a combine CTA then fits beside
// the two main-kernel CTAs of an SM (2 x 128 threads x 188 registers), so the
// PDL launch makes it resident early and only the record loads remain after
// the main kernel ends.

template <typename T, int D>
__global__ void __launch_bounds__(kCombineThreads, 4) decode_combine_kernel(FlatParams p) {
  __shared__ float sm_m[kCombineThreads], sm_l[kCombineThreads];
  __shared__ float red[kCombineThreads * 8];
  __shared__ int wsum[2][kCombineThreads / 32];
  const int seg = blockIdx.x;
  const int b = seg / p.SPS, segx = seg - b * p.SPS;
  // The slice boundaries follow from the context lengths alone, an input
  // the main kernel does not write: recompute this sequence's sub-block
  // offset and the batch total before waiting for the main kernel (PDL), so
  // only the record loads remain after the wait.
  int pb0, nsub, ptot;
  {
    const int64_t cap = p.bt_width * (int64_t)p.bs;
    int before = 0, all = 0;
    for (int i = threadIdx.x; i < p.B; i += kCombineThreads) {
      int64_t ctx = p.context_lens[i];
      ctx = ctx > cap ? cap : ctx;
      const int c = ctx > 0 ? static_cast<int>((ctx + kSub - 1) / kSub) : 0;
      all += c;
      before += i < b ? c : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      all += __shfl_xor_sync(0xffffffffu, all, o);
    }
    if ((threadIdx.x & 31) == 0) {
      wsum[0][threadIdx.x >> 5] = before;
      wsum[1][threadIdx.x >> 5] = all;
    }
    __syncthreads();
    pb0 = 0;
    ptot = 0;
#pragma unroll
    for (int w = 0; w < kCombineThreads / 32; ++w) {
      pb0 += wsum[0][w];
      ptot += wsum[1][w];
    }
    int64_t ctx = p.context_lens[b];
    ctx = ctx > cap ? cap : ctx;
    nsub = ctx > 0 ? static_cast<int>((ctx + kSub - 1) / kSub) : 0;
  }
  if (nsub <= 0) return;
  const int W = p.W;
  const int64_t total = (int64_t)ptot * p.SPS;
  const int64_t sstart = (int64_t)pb0 * p.SPS + (int64_t)segx * nsub, send = sstart + nsub;
  const int g0 = static_cast<int>(((sstart + 1) * W - 1) / total);
  const int g1 = static_cast<int>((send * W - 1) / total);
  if (g0 == g1) return;  // finished inside one slice
  const int nrec = g1 - g0 + 1;
  grid_dep_wait();  // the main kernel's records are complete and visible
  const int kvh = segx / p.HT, ht = segx - kvh * p.HT;
  const int h0 = kvh * p.group + ht * 16, hn = min(16, p.group - ht * 16);
  const bool g0_first = (int64_t)g0 * total / W == sstart;
  const int tid = threadIdx.x;
  auto rec = [&](int r) -> int64_t {  // record row base (h = 0), or -1 for an empty slice
    const int gg = g0 + r;
    if ((int64_t)gg * total / W == (int64_t)(gg + 1) * total / W) return -1;
    const int sl = (r == 0 && !g0_first) ? 1 : 0;
    return (int64_t)(gg * 2 + sl) * 16;
  };
  // One pass: thread (item, stripe) merges the records stripe, stripe +
  // stripes, ... of one (row, 8 columns) item online (running max in the
  // log2 domain, rescaled l and O), four records' loads in flight at a
  // time; then the stripes of each item are merged by log-sum-exp through
  // shared memory.  One dependent round of global loads per four records.
  const int items = hn * (D / 8);
  const int stripes = kCombineThreads / items;
  const int item = tid % items, stripe = tid / items;
  float mrun = -INFINITY, lrun = 0.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (stripe < stripes) {
    const int h = item / (D / 8), d = 8 * (item - h * (D / 8));
    for (int r0 = stripe; r0 < nrec; r0 += 4 * stripes) {
      float2 ml[4];
      float4 v0[4], v1[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int r = r0 + u * stripes;
        const int64_t base = r < nrec ? rec(r) : -1;
        ml[u] = make_float2(-INFINITY, 0.f);
        v0[u] = v1[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (base >= 0) {
          ml[u] = __ldcg(reinterpret_cast<const float2*>(p.part_ml + (base + h) * 2));
          const float4* src = reinterpret_cast<const float4*>(p.part_o + (base + h) * D + d);
          v0[u] = __ldcg(src);
          v1[u] = __ldcg(src + 1);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (ml[u].x == -INFINITY) continue;
        const float mnew = fmaxf(mrun, ml[u].x);
        const float a = exp2f(mrun - mnew), wt = exp2f(ml[u].x - mnew);  // a = 0 on the first record
        lrun = lrun * a + ml[u].y * wt;
        acc[0] = fmaf(wt, v0[u].x, acc[0] * a);
        acc[1] = fmaf(wt, v0[u].y, acc[1] * a);
        acc[2] = fmaf(wt, v0[u].z, acc[2] * a);
        acc[3] = fmaf(wt, v0[u].w, acc[3] * a);
        acc[4] = fmaf(wt, v1[u].x, acc[4] * a);
        acc[5] = fmaf(wt, v1[u].y, acc[5] * a);
        acc[6] = fmaf(wt, v1[u].z, acc[6] * a);
        acc[7] = fmaf(wt, v1[u].w, acc[7] * a);
        mrun = mnew;
      }
    }
  }
  sm_m[tid] = mrun;
  sm_l[tid] = lrun;
#pragma unroll
  for (int e = 0; e < 8; ++e) red[tid * 8 + e] = acc[e];
  __syncthreads();
  if (tid < items) {
    const int h = tid / (D / 8), d = 8 * (tid - h * (D / 8));
    float mx = -INFINITY;
    for (int s2 = 0; s2 < stripes; ++s2) mx = fmaxf(mx, sm_m[s2 * items + tid]);
    float lt = 0.f, sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s2 = 0; s2 < stripes; ++s2) {
      const int t2 = s2 * items + tid;
      const float ms = sm_m[t2];
      if (ms == -INFINITY) continue;
      const float wt = exp2f(ms - mx);
      lt = fmaf(sm_l[t2], wt, lt);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum[e] = fmaf(red[t2 * 8 + e], wt, sum[e]);
    }
    T* out = reinterpret_cast<T*>(p.out);
    store8<T>(out + (int64_t)b * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d, sum, 1.f / lt);
  }
}

// ===========================================================================
// Explicit-partition split-KV decode: one CTA per (sequence, KV head x head
// tile, partition of `split_sub` sub-blocks); warps of a CTA interleave over
// its sub-blocks; partitions are merged by the CTA drawing the last ticket.
// Used when the caller fixes the partition size (the reference's split-KV
// API takes partition_size, kernels/triton/paged_attention.py:24-37).
// ===========================================================================
struct SplitParams {
  const void* q;
  int64_t q_s0, q_s1;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  const int64_t* context_lens;
  void* out;
  int64_t o_s0, o_s1;
  int Hq, Hkv, group, bs;
  float scale_log2;
  int split_sub;  // 16-token sub-blocks per partition
  int max_splits;
  float* part_ml;  // [B, Hq, max_splits, 2]
  float* part_o;   // [B, Hq, max_splits, D]
  int* tickets;
  int* status;
};

template <int D, int NW, int STAGES>
struct SplitCfg {
  static constexpr int kColTiles = D / 64;
  static constexpr int kStageBytes = 2 * kColTiles * kTileBytes;
  static constexpr int kRingBytes = NW * STAGES * kStageBytes;
  static constexpr int kMergeBytes = NW * 16 * (D + 4) * 4;
  static constexpr size_t kSmem = 1024 + kRingBytes + kMergeBytes + NW * STAGES * 8 + 64;
};

template <typename T, int D, int NW, int STAGES>
__global__ void __launch_bounds__(NW * 32) decode_split_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                              const __grid_constant__ CUtensorMap tmap_v,
                                                              SplitParams p) {
  using C = SplitCfg<D, NW, STAGES>;
  constexpr int NT = NW * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* merge = reinterpret_cast<float*>(smem + C::kRingBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kRingBytes + C::kMergeBytes);
  __shared__ int last_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.z, split = blockIdx.x;
  const int head_tiles = (p.group + 15) >> 4;
  const int kvh = blockIdx.y / head_tiles, ht = blockIdx.y - kvh * head_tiles;
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
  const int nj = (s1 - s0 > warp) ? (s1 - s0 - warp + NW - 1) / NW : 0;

  uint8_t* ring = smem + warp * STAGES * C::kStageBytes;
  uint64_t* wbar = bars + warp * STAGES;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const int64_t* bt_row = p.bt + (int64_t)b * p.bt_stride;
  auto issue = [&](int j) {
    const int64_t tok0 = (int64_t)(s0 + warp + j * NW) * kSub;
    const int64_t pb = bt_row[tok0 / p.bs];
    const int y = static_cast<int>(pb * p.bs + tok0 % p.bs);
    const int stage = j % STAGES;
    uint8_t* st = ring + stage * C::kStageBytes;
    mbar_arrive_expect_tx(&wbar[stage], C::kStageBytes);
#pragma unroll
    for (int ct = 0; ct < C::kColTiles; ++ct) {
      tma_load_3d(st + ct * kTileBytes, &tmap_k, &wbar[stage], ct * 64, kvh, y);
      tma_load_3d(st + (C::kColTiles + ct) * kTileBytes, &tmap_v, &wbar[stage], ct * 64, kvh, y);
    }
  };
  if (lane == 0) {
    for (int j = 0; j < STAGES && j < nj; ++j) issue(j);
  }
  WarpState<T, D> ws;
  ws.reset();
  ws.load_q(reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_s0, p.q_s1, h0, hn, lane);
  bool ok = true;
  for (int j = 0; j < nj; ++j) {
    const int stage = j % STAGES;
    if (ok) ok = mbar_wait(&wbar[stage], (j / STAGES) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
    const uint32_t kbase = smem_u32(ring + stage * C::kStageBytes);
    const int valid = static_cast<int>(min((int64_t)kSub, ctx - (int64_t)(s0 + warp + j * NW) * kSub));
    const uint32_t vbase = kbase + C::kColTiles * kTileBytes;
    ws.template consume<1>(&kbase, &vbase, &valid, p.scale_log2, lane);
    __syncwarp();
    if (lane == 0 && j + STAGES < nj) issue(j + STAGES);
  }
  ws.store(merge + warp * 16 * (D + 4), lane);
  __syncthreads();

  T* out = reinterpret_cast<T*>(p.out);
  const int64_t base_rh = (int64_t)b * p.Hq + h0;
  const bool single = nsplits == 1;
  for (int i = tid; i < hn * D; i += NT) {
    const int h = i / D, d = i - h * D;
    float m, l, acc;
    merge_records<D>(merge, NW, h, d, m, l, acc);
    if (single) {
      out[(int64_t)b * p.o_s0 + (int64_t)(h0 + h) * p.o_s1 + d] = Elem<T>::from_f32(acc / l);
    } else {
      p.part_o[((base_rh + h) * p.max_splits + split) * D + d] = acc;
      if (d == 0) {
        p.part_ml[((base_rh + h) * p.max_splits + split) * 2 + 0] = m;
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
  for (int i = tid; i < hn * D; i += NT) {
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

// Kernel shapes: (warps per CTA, ring stages per warp).
// Two CTAs per SM (about 107 KB of shared memory each), so a CTA's start-up
// and merge tail overlap the other CTA's streaming — and, with PDL, the next
// kernel's CTAs.
#ifndef PA_FLAT_NW64
#define PA_FLAT_NW64 4
#endif
#ifndef PA_FLAT_ST64
#define PA_FLAT_ST64 4
#endif
constexpr int kFlatNW64 = PA_FLAT_NW64, kFlatST64 = PA_FLAT_ST64;
constexpr int kFlatNW128 = 2, kFlatST128 = 4;
#ifndef PA_FLAT_CTAS
#define PA_FLAT_CTAS 2
#endif
constexpr int kFlatCtasPerSm = PA_FLAT_CTAS;
constexpr int flat_nw(int D) { return D == 64 ? kFlatNW64 : kFlatNW128; }
constexpr int kSplitNW = 4, kSplitST = 4;

template <typename K>
bool set_smem_attr(K kern, size_t bytes, bool* done) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return false;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
      return false;
    done[dev] = true;
  }
  return true;
}

template <typename T, int D, int NW, int ST, int CTAS>
int launch_flat(const FlatParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int grid, cudaStream_t st) {
  using C = FlatCfg<D, NW, ST>;
  auto kern = decode_flat_kernel<T, D, NW, ST, CTAS>;
  static bool done[64] = {};
  if (!set_smem_attr(kern, C::kSmem, done)) return PA_ERR_CUDA;
  const int r = launch_pdl(kern, dim3(grid), dim3(NW * 32), C::kSmem, st, tk, tv, p);
  if (r != PA_OK) return r;
  return launch_pdl(decode_combine_kernel<T, D>, dim3(p.B * p.SPS), dim3(kCombineThreads), 0, st, p);
}

template <typename T, int D>
int launch_split(const SplitParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int batch, int splits,
                 cudaStream_t st) {
  using C = SplitCfg<D, kSplitNW, kSplitST>;
  auto kern = decode_split_kernel<T, D, kSplitNW, kSplitST>;
  static bool done[64] = {};
  if (!set_smem_attr(kern, C::kSmem, done)) return PA_ERR_CUDA;
  const int head_tiles = (p.group + 15) / 16;
  dim3 grid(splits, p.Hkv * head_tiles, batch);
  kern<<<grid, kSplitNW * 32, C::kSmem, st>>>(tk, tv, p);
  PA_CHECK_LAUNCH();
  return PA_OK;
}

bool tc_shape_ok(int dtype, int D, int bs) {
  return (dtype == PA_DTYPE_BF16 || dtype == PA_DTYPE_F16) && (D == 64 || D == 128) && bs % kSub == 0 && bs <= 256;
}

bool fast_path_ok(int dtype, int D, int bs, int64_t num_blocks, const void* q, int64_t q_s0, int64_t q_s1,
                  const void* kp, const void* vp, const void* out, int64_t o_s0, int64_t o_s1) {
  if (!tc_shape_ok(dtype, D, bs)) return false;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (o_s0 & 7) || (o_s1 & 7)) return false;
  if (num_blocks * (int64_t)bs >= (int64_t(1) << 31)) return false;
  if ((q_s0 & 1) || (q_s1 & 1) || (reinterpret_cast<uintptr_t>(q) & 3)) return false;
  if ((reinterpret_cast<uintptr_t>(kp) & 15) || (reinterpret_cast<uintptr_t>(vp) & 15)) return false;
  return true;
}

// Which kernel a call uses and how many partials it may write.
struct DecodePlan {
  enum Kind { kFlat, kSplit, kGeneric } kind;
  int grid;         // flat: CTAs
  int split_sub;    // split: sub-blocks per partition
  int split_tokens; // generic: tokens per partition
  int splits;       // split / generic: partitions per sequence (max)
  size_t ws_bytes;
};

DecodePlan plan_decode(int batch, int hkv, int hq, int D, int bs, int64_t bt_width, int partition_tokens,
                       int dtype) {
  DecodePlan pl{};
  const int group = hq / hkv;
  const int sms = num_sms(current_device());
  const int64_t max_tok = bt_width * bs;
  const size_t tickets = align256(sizeof(int) * (size_t)batch * hq);
  if (tc_shape_ok(dtype, D, bs) && partition_tokens == 0 && batch <= kFlatMaxBatch) {
    pl.kind = DecodePlan::kFlat;
    pl.grid = sms * kFlatCtasPerSm;
    const size_t W = (size_t)pl.grid * flat_nw(D);
    const size_t ml = align256(sizeof(float) * 2 * 16 * 2 * W);
    const size_t po = align256(sizeof(float) * 2 * 16 * (size_t)D * W);
    pl.ws_bytes = 256 + tickets + ml + po;
    return pl;
  }
  if (tc_shape_ok(dtype, D, bs)) {
    pl.kind = DecodePlan::kSplit;
    const int64_t max_sub = (max_tok + kSub - 1) / kSub;
    int64_t split;
    if (partition_tokens > 0) {
      split = (partition_tokens + kSub - 1) / kSub;
    } else {  // batch too large for the flat kernel's prefix table
      split = max_sub;
    }
    split = split > max_sub ? max_sub : (split < 1 ? 1 : split);
    pl.split_sub = static_cast<int>(split);
    pl.splits = static_cast<int>((max_sub + split - 1) / split);
    pl.ws_bytes = workspace_layout(batch, hq, D, pl.splits).total;
    return pl;
  }
  pl.kind = DecodePlan::kGeneric;
  const int chunk = generic_chunk_tokens();
  const int ht = (group + 7) / 8;
  int64_t split;
  if (partition_tokens > 0) {
    split = partition_tokens;
  } else {
    const int64_t ctas = (int64_t)batch * hkv * ht;
    split = ctas >= 2 * sms ? max_tok : 2 * chunk;
  }
  const int64_t max_round = (max_tok + chunk - 1) / chunk * chunk;
  split = (split + chunk - 1) / chunk * chunk;
  split = split > max_round ? max_round : (split < chunk ? chunk : split);
  pl.split_tokens = static_cast<int>(split);
  pl.splits = static_cast<int>((max_tok + split - 1) / split);
  pl.ws_bytes = workspace_layout(batch, hq, D, pl.splits).total;
  return pl;
}

}  // namespace
}  // namespace pa

extern "C" size_t pa_decode_workspace_bytes(int batch, int num_kv_heads, int num_q_heads, int head_dim,
                                            int block_size, int64_t bt_width, int partition_tokens, int dtype) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0 || head_dim <= 0 ||
      block_size <= 0 || bt_width <= 0 || partition_tokens < 0)
    return 0;
  return pa::plan_decode(batch, num_kv_heads, num_q_heads, head_dim, block_size, bt_width, partition_tokens, dtype)
      .ws_bytes;
}

namespace pa {
namespace {

// The new token's K/V for a fused write (see pa_paged_decode_write).
struct FusedWrite {
  const void* new_k;
  const void* new_v;
  const int64_t* slots;
};

int decode_impl(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer, const void* v_pool_layer,
                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                int64_t bt_stride, int64_t bt_width, const int64_t* context_lens, void* out, int64_t o_s0,
                int64_t o_s1, int batch, int num_q_heads, float scale, int dtype, int partition_tokens,
                void* workspace, size_t workspace_bytes, void* stream, const FusedWrite* fw, bool* fused);

}  // namespace
}  // namespace pa

extern "C" int pa_paged_decode(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer,
                               const void* v_pool_layer, int64_t num_blocks, int block_size, int num_kv_heads,
                               int head_dim, const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                               const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                               int num_q_heads, float scale, int dtype, int partition_tokens, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return pa::decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim,
                         block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch, num_q_heads, scale,
                         dtype, partition_tokens, workspace, workspace_bytes, stream, nullptr, nullptr);
}

extern "C" int pa_paged_decode_write(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k,
                                     const void* new_v, const int64_t* slot_mapping, void* k_pool_layer,
                                     void* v_pool_layer, int64_t num_blocks, int block_size, int num_kv_heads,
                                     int head_dim, const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                                     const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                                     int num_q_heads, float scale, int dtype, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  using namespace pa;
  if (batch < 0) return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  if (new_k == nullptr || new_v == nullptr || slot_mapping == nullptr) return PA_ERR_INVALID;
  const bool aligned = !((reinterpret_cast<uintptr_t>(new_k) | reinterpret_cast<uintptr_t>(new_v)) & 15);
  FusedWrite fw{new_k, new_v, slot_mapping};
  bool fused = false;
  if (aligned) {
    const int r = decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads,
                              head_dim, block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch,
                              num_q_heads, scale, dtype, 0, workspace, workspace_bytes, stream, &fw, &fused);
    if (r != PA_OK || fused) return r;
  }
  // Not fusable here (other kernel, odd alignment): the scatter, then decode.
  const int64_t s1 = head_dim, s0 = (int64_t)num_kv_heads * head_dim;
  const int r = pa_kv_scatter(new_k, s0, s1, 1, new_v, s0, s1, 1, dtype, slot_mapping, 1, batch, k_pool_layer,
                              v_pool_layer, num_blocks * (int64_t)block_size, num_kv_heads, head_dim, dtype, stream);
  if (r != PA_OK) return r;
  return pa_paged_decode(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim,
                         block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch, num_q_heads, scale,
                         dtype, 0, workspace, workspace_bytes, stream);
}

namespace pa {
namespace {

int decode_impl(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer, const void* v_pool_layer,
                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                int64_t bt_stride, int64_t bt_width, const int64_t* context_lens, void* out, int64_t o_s0,
                int64_t o_s1, int batch, int num_q_heads, float scale, int dtype, int partition_tokens,
                void* workspace, size_t workspace_bytes, void* stream, const FusedWrite* fw, bool* fused) {
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
  DecodePlan pl =
      plan_decode(batch, num_kv_heads, num_q_heads, head_dim, block_size, bt_width, partition_tokens, dtype);
  const bool fast = fast_path_ok(dtype, head_dim, block_size, num_blocks, q, q_s0, q_s1, k_pool_layer, v_pool_layer,
                                 out, o_s0, o_s1);
  if (!fast && pl.kind != DecodePlan::kGeneric) {
    // Unaligned views: same math on the CUDA-core kernel.
    const int chunk = generic_chunk_tokens();
    const int64_t max_tok = bt_width * block_size;
    pl.kind = DecodePlan::kGeneric;
    pl.split_tokens = static_cast<int>((max_tok + chunk - 1) / chunk * chunk);
    pl.splits = 1;
  }
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  if (ws == nullptr || workspace_bytes < pl.ws_bytes || (reinterpret_cast<uintptr_t>(ws) & 255))
    return PA_ERR_WORKSPACE;
  int* status = reinterpret_cast<int*>(ws);
  const size_t off_ml = 256 + align256(sizeof(int) * (size_t)batch * num_q_heads);

  if (pl.kind == DecodePlan::kFlat || pl.kind == DecodePlan::kSplit) {
    CUtensorMap tk, tv;
    const uint64_t slots = static_cast<uint64_t>(num_blocks) * block_size;
    const uint64_t s1b = static_cast<uint64_t>(head_dim) * 2;
    const uint64_t s2b = s1b * num_kv_heads;
#ifndef PA_DECODE_L2_PROMOTION
#define PA_DECODE_L2_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_128B
#endif
    // Rows of one KV head are 128 B with a Hkv*128 B stride; a wider L2
    // promotion would drag the other heads' rows in ahead of their readers.
    if (make_map_3d(&tk, dtype, k_pool_layer, head_dim, num_kv_heads, slots, s1b, s2b, 64, 1, 16,
                    CU_TENSOR_MAP_SWIZZLE_128B, PA_DECODE_L2_PROMOTION) != PA_OK ||
        make_map_3d(&tv, dtype, v_pool_layer, head_dim, num_kv_heads, slots, s1b, s2b, 64, 1, 16,
                    CU_TENSOR_MAP_SWIZZLE_128B, PA_DECODE_L2_PROMOTION) != PA_OK)
      return PA_ERR_CUDA;
    const float scale_log2 = scale * 1.4426950408889634f;
    if (pl.kind == DecodePlan::kFlat) {
      FlatParams p;
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
      p.B = batch;
      p.Hq = num_q_heads;
      p.Hkv = num_kv_heads;
      p.group = group;
      p.HT = (group + 15) / 16;
      p.SPS = num_kv_heads * p.HT;
      p.bs = block_size;
      p.scale_log2 = scale_log2;
      p.W = pl.grid * flat_nw(head_dim);
      const size_t ml_bytes = align256(sizeof(float) * 2 * 16 * 2 * (size_t)p.W);
      const size_t po_bytes = align256(sizeof(float) * 2 * 16 * (size_t)head_dim * p.W);
      p.part_ml = reinterpret_cast<float*>(ws + off_ml);
      p.part_o = reinterpret_cast<float*>(ws + off_ml + ml_bytes);
      p.status = status;
      p.new_k = fw ? fw->new_k : nullptr;
      p.new_v = fw ? fw->new_v : nullptr;
      p.slots = fw ? fw->slots : nullptr;
      p.k_pool = const_cast<void*>(k_pool_layer);
      p.v_pool = const_cast<void*>(v_pool_layer);
      p.num_slots = static_cast<int64_t>(num_blocks) * block_size;
      if (fused != nullptr) *fused = fw != nullptr;
      constexpr int CT = kFlatCtasPerSm;
      if (dtype == PA_DTYPE_BF16)
        return head_dim == 64 ? launch_flat<__nv_bfloat16, 64, kFlatNW64, kFlatST64, CT>(p, tk, tv, pl.grid, st)
                              : launch_flat<__nv_bfloat16, 128, kFlatNW128, kFlatST128, CT>(p, tk, tv, pl.grid, st);
      return head_dim == 64 ? launch_flat<__half, 64, kFlatNW64, kFlatST64, CT>(p, tk, tv, pl.grid, st)
                            : launch_flat<__half, 128, kFlatNW128, kFlatST128, CT>(p, tk, tv, pl.grid, st);
    }
    if (pl.splits > 65535) return PA_ERR_INVALID;
    const WorkspaceLayout wl = workspace_layout(batch, num_q_heads, head_dim, pl.splits);
    SplitParams p;
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
    p.scale_log2 = scale_log2;
    p.split_sub = pl.split_sub;
    p.max_splits = pl.splits;
    p.part_ml = reinterpret_cast<float*>(ws + wl.part_ml);
    p.part_o = reinterpret_cast<float*>(ws + wl.part_o);
    p.tickets = reinterpret_cast<int*>(ws + wl.tickets);
    p.status = status;
    if (dtype == PA_DTYPE_BF16)
      return head_dim == 64 ? launch_split<__nv_bfloat16, 64>(p, tk, tv, batch, pl.splits, st)
                            : launch_split<__nv_bfloat16, 128>(p, tk, tv, batch, pl.splits, st);
    return head_dim == 64 ? launch_split<__half, 64>(p, tk, tv, batch, pl.splits, st)
                          : launch_split<__half, 128>(p, tk, tv, batch, pl.splits, st);
  }

  if (pl.splits > 65535) return PA_ERR_INVALID;
  const WorkspaceLayout wl = workspace_layout(batch, num_q_heads, head_dim, pl.splits);
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
  g.split_tokens = pl.split_tokens;
  g.max_splits = pl.splits;
  g.part_ml = pl.splits > 1 ? reinterpret_cast<float*>(ws + wl.part_ml) : nullptr;
  g.part_o = pl.splits > 1 ? reinterpret_cast<float*>(ws + wl.part_o) : nullptr;
  g.tickets = pl.splits > 1 ? reinterpret_cast<int*>(ws + wl.tickets) : nullptr;
  g.status = status;
  return launch_attn_generic(g, dtype, pl.splits, st);
}

}  // namespace
}  // namespace pa
