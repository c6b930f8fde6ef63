// tcgen05 causal chunk-prefill over a paged KV cache (BF16/F16, head_dim 64
// or 128).
//
// Math: for every query row of a chunk, softmax(scale * q K^T) V over the
// keys at absolute positions <= prefix + i (reference:
// kernels/reference/paged_attention.py:346-434 — the tiled online softmax
// of :398-431 — and its dense twin :282-343).
//
// Work item: (sequence, KV head, pair of M-tiles).  An M-tile packs the GQA
// group into the 128 MMA rows: row r = (query position r / G, query head
// r % G), P = floor(128 / G) positions per tile (18 for a group of 7 -> 126
// live rows), so every K/V tile staged from the paged pool feeds all G query
// heads of both M-tiles.  The kernel is persistent (one CTA per SM).  Items
// are handed out longest first (by KV tile count; a counting sort of the
// work units built in shared memory at start, or descending query position
// past its capacity) and dynamically: the producer warp claims the next
// index from a global counter (self-rewinding: the last CTA to finish zeroes
// it) and publishes it through a small ring in shared memory to the other
// roles.  Without a control block the CTAs take every gridDim.x-th claim.
//
// Warp roles (384 threads; setmaxnreg moves registers to the softmax):
//   warp 8      TMA producer: the item's two Q tiles (3-D boxes {64, G, P}
//               straight from the packed [T, Hq, D] tensor, double-buffered
//               across items when shared memory allows), then per KV tile
//               of N tokens the K and V boxes {64, 1, 16} addressed through
//               the block table into rings of stages (128-byte swizzle =
//               canonical UMMA layout).  Tokens at or past the context use an
//               out-of-range coordinate: TMA fills zeros.
//   warps 9-10  MMA issuers, one per M-tile w (warp 9 also owns TMEM): per
//               KV tile j, S_w(j) = Q_w K(j)^T (both operands from shared
//               memory) and O_w += P_w(j-1) V(j-1) (P from tensor memory, V
//               from shared memory, half the shared-memory traffic of an SS
//               MMA).  Head dim 64 gives S, P and O columns of their own, so
//               S_w(j+1) is issued as soon as the softmax has copied S_w(j)
//               into registers.  Head dim 128 fills an M-tile's 256 columns
//               with O and a 128-key S, writes P over S, and issues
//               P_w(j-1) V(j-1) before S_w(j) (one thread's MMAs run in
//               order).  Each issuer does its own mbarrier waits: the
//               stall such a wait costs right after a thread's MMAs is
//               covered by the other issuer's MMAs, and one M-tile's chain
//               never waits for the other's.
//   warps 0-3   softmax of M-tile 0, warps 4-7 softmax of M-tile 1 (one row
//               per thread, FP32 statistics in the log2 domain).  While one
//               group exponentiates, the tensor core works for the other.
//               O stays in TMEM for the whole item; it is rescaled only when
//               a row's running maximum grows by more than 2^8 (the
//               unnormalised P then stays below 256, exact enough in FP32 and
//               BF16), and read once at the end for 1/l and the store.
//   warp 11     idle.
// Every mbarrier wait is bounded; a failed wait records a status code, sets
// a CTA-wide abort flag, and every role winds down (in-flight copies and
// MMAs are drained, TMEM is freed) without further waiting.
#include <algorithm>
#include <type_traits>

#include "prefill_tc.cuh"
#include "tcgen05.cuh"

namespace pa {
namespace {

constexpr int kM = 128;                      // MMA rows per M-tile
constexpr int kThreads = 384;                // 3 warpgroups
constexpr int kProducerWarp = 8, kMmaWarp0 = 9, kMmaWarp1 = 10;
constexpr int kConsumerWarps = 10;           // 2 MMA warps + 8 softmax warps read each item index
// setmaxnreg budgets (per thread): launch gives 168 x 384; the control
// warpgroup drops to 56 so the two softmax warpgroups can hold a 128-float
// S row next to a 32-column O slice: 4*32*56 + 8*32*224 = 384*168.
constexpr int kCtrlRegs = 56, kSoftmaxRegs = 224;
static_assert(4 * 32 * kCtrlRegs + 8 * 32 * kSoftmaxRegs <= kThreads * 168, "register split");
constexpr float kRescaleLog2 = 8.f;          // lazy-rescale threshold (log2 units)
constexpr int kBoxTokens = 16;               // tokens per K/V TMA box
// Of every 8 column pairs of a score row, how many take the FMA-pipe exp2
// (the rest the MUFU one).  Measured best: a quarter at head_dim 64, where
// the softmax is a larger share of each tile, none at head_dim 128 (twice
// the tensor work per score).
#ifndef PA_PREFILL_POLY64
#define PA_PREFILL_POLY64 2
#endif
#ifndef PA_PREFILL_POLY128
#define PA_PREFILL_POLY128 0
#endif
// Waits of the MMA issuers and of the softmax on its scores: 1 polls
// (test_wait; the waiter is on the critical path and wakes sooner), 0
// suspends in try_wait (its issue slots stay with the other warps of its
// SMSP).  Head dim 128 keeps the softmax wait suspended: there the other
// group's exponentials run beside it.
#ifndef PA_PREFILL_SPIN_ISSUER
#define PA_PREFILL_SPIN_ISSUER 1
#endif
#ifndef PA_PREFILL_SPIN_SOFTMAX64
#define PA_PREFILL_SPIN_SOFTMAX64 1
#endif
#ifndef PA_PREFILL_SPIN_SOFTMAX128
#define PA_PREFILL_SPIN_SOFTMAX128 0
#endif

// head_dim 128 takes 128-token KV tiles with P written over S's TMEM
// columns (O 128 + S 128 fill an M-tile's 256); 0 selects 64-token tiles
// with P in columns of its own.
#ifndef PA_PREFILL_D128_ALIAS
#define PA_PREFILL_D128_ALIAS 1
#endif

template <int D> struct Shape;
// N = KV tokens per tile, ST = K/V ring stages, QB = Q buffers (items in
// flight), kAliasP = P overwrites S in TMEM.
template <> struct Shape<64> {
  static constexpr int N = 128, ST = 4, QB = 2;
  static constexpr bool kAliasP = false;
};
#if PA_PREFILL_D128_ALIAS
template <> struct Shape<128> {
  static constexpr int N = 128, ST = 2, QB = 1;
  static constexpr bool kAliasP = true;
};
#else
template <> struct Shape<128> {
  static constexpr int N = 64, ST = 3, QB = 2;
  static constexpr bool kAliasP = false;
};
#endif

template <int D>
struct Lay {
  static constexpr int N = Shape<D>::N, ST = Shape<D>::ST, QB = Shape<D>::QB;
  static constexpr bool kAliasP = Shape<D>::kAliasP;
  // With P over S, K and V have rings of their own (K(g) is free once the
  // last S that reads it is done, a tile before V(g)), which doubles how far
  // ahead of use the loads can start; otherwise one ring holds both.
  static constexpr bool kSplitKV = kAliasP;
  static constexpr int kDH = D / 64;           // 128-byte column slabs per row
  static constexpr int kSlab = kM * 128;       // one 128-row slab (16 KB)
  static constexpr int kQTile = kDH * kSlab;   // Q tile: [kDH][128 rows][128 B]
  static constexpr int kKVTile = kDH * N * 128;  // K or V tile: [kDH][N rows][128 B]
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + QB * 2 * kQTile;
  static constexpr int kOffV = kOffK + ST * kKVTile;
  static constexpr int kOffBar = kOffV + ST * kKVTile;
  static constexpr int kRing = 4;             // claimed item indices in flight
  static constexpr int kNumBars = 2 * QB + 5 * ST + 10 + 2 + 2 * kRing;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;  // tmem slot, abort flag, item ring
  // Longest-first order of the work units (sequence x pair of M-tiles):
  // unit codes sorted by KV tile count, the per-count offsets, and each
  // sequence's chunk length and prefix.
  static constexpr int kLptUnits = 2048, kLptLevels = 512, kLptSeqs = 512;
  static constexpr int kOffLpt = kOffMisc + 16 + 4 * kRing;
  static constexpr size_t kSmem = 1024 + kOffLpt + 4 * (kLptUnits + kLptLevels + 2 * kLptSeqs);
  // TMEM: 256 columns per M-tile w: S (N FP32 columns), P (N/2 columns of
  // packed 16-bit values) and O, each aligned to its width:
  //   D=64,  N=128: S [0,128)  P [128,192)  O [192,256)
  //   D=128, N=128: O [0,128)  S [128,256), P over S [128,192)
  //   D=128, N=64:  O [0,128)  S [128,192)  P [192,224)
  static constexpr uint32_t kWgCols = 256;
  static constexpr uint32_t kTmemS = D == 64 ? 0 : 128;
  static constexpr uint32_t kTmemP = kAliasP ? kTmemS : kTmemS + N;
  static constexpr uint32_t kTmemO = D == 64 ? 192 : 0;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr int kBoxes = (N / kBoxTokens) * kDH;  // per K (and per V) tile
  static_assert(kBoxes <= 32, "one TMA box per producer lane");
  static constexpr uint32_t kSPEnd = kAliasP ? kTmemS + N : kTmemP + N / 2;
  static_assert(kSPEnd <= kWgCols && kTmemO + D <= kWgCols && (kTmemO + D <= kTmemS || kTmemO >= kSPEnd),
                "TMEM layout");
  static_assert(kSmem <= 227 * 1024, "shared memory");
  static_assert(N % 32 == 0 && N <= 128, "S row loads in 32-column pieces");
};

struct TcParams {
  const int64_t* cu_q;
  const int64_t* context_lens;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  int64_t num_blocks, num_slots;
  void* out;
  int64_t o_s0, o_s1;
  int64_t ctx_cap;  // min(bt_width * bs, 2^31 - 1)
  int64_t total_q;
  int G, P, bs, Hkv, num_seqs, pairs, num_items;
  float scale_log2;
  int* status;   // control[0]; null: no status, static schedule
  int* claim;    // control[1]: next item to hand out (dynamic schedule)
  int* finish;   // control[2]: CTAs done; the last one zeroes claim and finish
};

// Positions fit in 32 bits: total_q and the pool's slot count are checked
// below 2^31 on the host, and ctx is clamped to the table's reach.
struct Item {
  int seq, kvh, ntiles;
  int q0, C, ctx, prefix, p0;
};

// Item idx of the schedule: pair index descending (largest query positions,
// hence longest key ranges, first), then sequence, then KV head.  False for
// items with no query rows.
__device__ __forceinline__ bool item_at(const TcParams& p, int idx, int N, Item& it) {
  const int per_pair = p.num_seqs * p.Hkv;
  const int pair = p.pairs - 1 - idx / per_pair;
  const int rem = idx - (idx / per_pair) * per_pair;
  it.seq = rem / p.Hkv;
  it.kvh = rem - it.seq * p.Hkv;
  const int64_t q0 = __ldg(p.cu_q + it.seq);
  const int64_t C = __ldg(p.cu_q + it.seq + 1) - q0;
  int64_t ctx = __ldg(p.context_lens + it.seq);
  if (ctx > p.ctx_cap) ctx = p.ctx_cap;
  if (C <= 0 || C > ctx || q0 < 0 || q0 + C > p.total_q) return false;
  it.q0 = static_cast<int>(q0);
  it.C = static_cast<int>(C);
  it.ctx = static_cast<int>(ctx);
  it.prefix = it.ctx - it.C;
  it.p0 = pair * 2 * p.P;
  if (it.p0 >= it.C) return false;
  const int last = it.prefix + min(it.C, it.p0 + 2 * p.P) - 1;
  it.ntiles = last / N + 1;
  return true;
}

// 2^x on the MUFU (XU) pipe.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float y;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
  return y;
}

// 2^x for two values on the FMA pipe (the MUFU pipe runs exp2 at a
// sixteenth of the FMA rate, so moving part of the softmax's exponentials
// here balances the two).  Method: Cody-Waite range reduction
// x = n + f, n = round(x) (adding 1.5 * 2^23 rounds to an integer in the
// low mantissa bits), |f| <= 1/2, then 2^f by a degree-3 polynomial whose
// coefficients were fitted for minimum relative error on [-1/2, 1/2]
// (max relative error 1.0e-4, far below the 2^-9 of the BF16/F16 P it
// feeds), and 2^n applied by adding n to the exponent field.  Inputs are
// clamped to >= -127 (-inf -> exactly 0); they never exceed +8 here.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kShift = 12582912.f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -127.f);
  x.y = fmaxf(x.y, -127.f);
  const float2 t = __fadd2_rn(x, make_float2(kShift, kShift));
  const float2 n = __fadd2_rn(t, make_float2(-kShift, -kShift));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 q = __ffma2_rn(make_float2(0.0550089068f, 0.0550089068f), f, make_float2(0.242210984f, 0.242210984f));
  q = __ffma2_rn(q, f, make_float2(0.693282962f, 0.693282962f));
  q = __ffma2_rn(q, f, make_float2(1.f, 1.f));
  return make_float2(__uint_as_float(__float_as_uint(q.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(q.y) + (__float_as_uint(t.y) << 23)));
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b) { return MmaOp<T>::pack(a, b); }

// KV tiles of the pair `pi` of a chunk (item_at's ntiles).
__device__ __forceinline__ int pair_tiles(int prefix, int C, int pi, int P, int N) {
  const int p0 = pi * 2 * P;
  return (prefix + min(C, p0 + 2 * P) - 1) / N + 1;
}

// Warp-collective: sorts the units (sequence, pair) with query rows by KV
// tile count, descending, into lpt[] (unit code pair * num_seqs + seq).
// Each sequence's metadata is read from global memory once (one round of
// loads) into seq_c / seq_pre; lvl[] holds the counts.  Returns the number
// of claims (units x Hkv), or -1 (keep the query-position order) when the
// batch exceeds the tables or has fewer than kLptMinSeqs sequences: with
// few sequences the costliest units all belong to one of them, and the
// CTAs starting on them together stream the same K/V lines in step, which
// measured slower than the query-position order's mix of sequences.
constexpr int kLptMinSeqs = 8;
__device__ int build_lpt(const TcParams& p, int N, int max_units, int max_levels, int max_seqs, int* lpt, int* lvl,
                         int* seq_c, int* seq_pre, int lane) {
  if (p.num_seqs > max_seqs || p.num_seqs < kLptMinSeqs) return -1;
  const int P2 = 2 * p.P;
  int units = 0, top = 0;
  for (int s = lane; s < p.num_seqs; s += 32) {
    // item_at's checks: a sequence without query rows has no units.
    const int64_t q0 = __ldg(p.cu_q + s);
    const int64_t c = __ldg(p.cu_q + s + 1) - q0;
    int64_t ctx = __ldg(p.context_lens + s);
    if (ctx > p.ctx_cap) ctx = p.ctx_cap;
    int C = 0, prefix = 0;
    if (!(c <= 0 || c > ctx || q0 < 0 || q0 + c > p.total_q)) {
      C = static_cast<int>(c);
      prefix = static_cast<int>(ctx - c);
      const int np = min((C + P2 - 1) / P2, p.pairs);  // the schedule covers p.pairs pairs
      units += np;
      top = max(top, pair_tiles(prefix, C, np - 1, p.P, N));
    }
    seq_c[s] = C;
    seq_pre[s] = prefix;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    units += __shfl_xor_sync(0xffffffffu, units, o);
    top = max(top, __shfl_xor_sync(0xffffffffu, top, o));
  }
  if (units > max_units || top >= max_levels || (int64_t)units * p.Hkv >= (int64_t(1) << 31)) return -1;
  for (int l = lane; l <= top; l += 32) lvl[l] = 0;
  __syncwarp();
  // Counting sort: count per tile count, offsets (highest count first),
  // then place.  Lanes take sequences and step through their pairs
  // together, so units of equal count alternate between sequences (as in
  // the query-position order): CTAs running at the same time then read
  // different sequences' K/V.
  auto for_units = [&](auto&& fn) {
    for (int s = lane; s < p.num_seqs; s += 32) {
      const int C = seq_c[s];
      if (C == 0) continue;
      const int np = min((C + P2 - 1) / P2, p.pairs);
      for (int pi = 0; pi < np; ++pi) fn(s, pi, pair_tiles(seq_pre[s], C, pi, p.P, N));
    }
  };
  for_units([&](int, int, int cost) { atomicAdd(&lvl[cost], 1); });
  __syncwarp();
  int carry = 0;  // lvl[l] := units costing more than l
  for (int base = top; base >= 0; base -= 32) {
    const int l = base - lane;
    const int v = l >= 0 ? lvl[l] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (l >= 0) lvl[l] = carry + incl - v;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  __syncwarp();
  for_units([&](int s, int pi, int cost) { lpt[atomicAdd(&lvl[cost], 1)] = pi * p.num_seqs + s; });
  __syncwarp();
  return units * p.Hkv;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                                                const __grid_constant__ CUtensorMap tmap_k,
                                                                const __grid_constant__ CUtensorMap tmap_v,
                                                                TcParams p) {
  using L = Lay<D>;
  constexpr int N = L::N, ST = L::ST, QB = L::QB;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + QB;
  uint64_t* kv_full = q_empty + QB;   // [ST], K and V of a tile (K only with split rings)
  uint64_t* kv_empty = kv_full + ST;
  uint64_t* v_full = kv_empty + ST;   // [ST], split rings: V of a tile
  uint64_t* v_empty = v_full + ST;
  uint64_t* s_full = v_empty + ST;    // [2], MMA commit after S_w
  uint64_t* s_free = s_full + 2;      // [2], 128 arrivals: S_w read into registers
  uint64_t* p_full = s_free + 2;      // [2], 128 arrivals: P_w in TMEM (and O_w rescaled)
  uint64_t* pv_done = p_full + 2;     // [2], MMA commit after P_w V
  uint64_t* o_empty = pv_done + 2;    // [2], 128 arrivals once an item's O is read out
  uint64_t* mma_done = o_empty + 2;  // [2], per issuer
  uint64_t* turn = mma_done + 2;     // [ST], issuer 0 has issued its MMAs of a tile
  uint64_t* item_full = turn + ST;             // [kRing], producer publishes an index
  uint64_t* item_empty = item_full + L::kRing;  // [kRing], 9 consumer warps took it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  volatile int* ring = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < QB; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);  // a commit from each issuer
    }
    for (int i = 0; i < ST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 2);
      mbar_init(&turn[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&pv_done[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    mbar_init(&mma_done[0], 1);
    mbar_init(&mma_done[1], 1);
    for (int i = 0; i < L::kRing; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp0) {
    tc::tmem_alloc(tmem_slot, L::kTmemCols);
    tc::tmem_relinquish();
  }
  if (warp == kProducerWarp) {
    // Q rows past G*P are never written by TMA: zero them once.
    const int live = p.G * p.P;
    const int dead_chunks = (kM - live) * 8;  // 16-byte chunks per slab
    for (int t = 0; t < QB * 2 * L::kDH; ++t)
      for (int c = lane; c < dead_chunks; c += 32)
        *reinterpret_cast<int4*>(smem + L::kOffQ + t * L::kSlab + live * 128 + c * 16) = make_int4(0, 0, 0, 0);
    fence_proxy_async_smem();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kCtrlRegs));
  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tmap_q);
      prefetch_tensormap(&tmap_k);
      prefetch_tensormap(&tmap_v);
    }
    uint32_t li = 0, g = 0;  // Q loads issued (one per item), K/V tiles issued
    bool k_pending = false;  // split rings: K(g) issued, V(g) not yet
    uint32_t pub = 0;        // item indices published to the ring
    int next_static = blockIdx.x;
    bool ok = true;
    // Longest first: items are claimed in order of descending KV tile count
    // (cost), so the last claims of the grid are the cheapest and the CTAs
    // finish together.  A counting sort of the units (sequence, pair of
    // M-tiles) by cost, in shared memory; claim c is unit lpt[c / Hkv],
    // KV head c % Hkv.  Shapes past the table's capacity keep the schedule
    // order (descending query position).
    int* lpt = reinterpret_cast<int*>(smem + L::kOffLpt);
    int* lvl = lpt + L::kLptUnits;
    int* seq_c = lvl + L::kLptLevels;
    int* seq_pre = seq_c + L::kLptSeqs;
    const int n_claims =
        build_lpt(p, N, L::kLptUnits, L::kLptLevels, L::kLptSeqs, lpt, lvl, seq_c, seq_pre, lane);
    for (;;) {
      // Claim the next item with query rows (dynamic: global counter;
      // static: every gridDim.x-th) and publish its index to the consumers.
      int idx = -1;
      if (lane == 0) {
        for (;;) {
          int c;
          if (p.claim != nullptr) {
            c = atomicAdd(p.claim, 1);
          } else {
            c = next_static;
            next_static += gridDim.x;
          }
          if (n_claims >= 0) {
            if (c >= n_claims) break;
            const int unit = lpt[c / p.Hkv];
            const int pair = unit / p.num_seqs, seq = unit - pair * p.num_seqs;
            idx = (p.pairs - 1 - pair) * (p.num_seqs * p.Hkv) + seq * p.Hkv + (c - (c / p.Hkv) * p.Hkv);
            break;
          }
          if (c >= p.num_items) break;
          Item probe;
          if (item_at(p, c, N, probe)) {
            idx = c;
            break;
          }
        }
        const int rs = pub % L::kRing;
        if (pub >= (uint32_t)L::kRing)
          ok = mbar_wait(&item_empty[rs], ((pub / L::kRing) - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
        if (ok) {
          ring[rs] = idx;
          mbar_arrive(&item_full[rs]);
          ++pub;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      idx = __shfl_sync(0xffffffffu, idx, 0);
      if (!ok || idx < 0) break;
      Item it;
      item_at(p, idx, N, it);
      const int qb = li % QB;
      if (lane == 0) {
        if (*abort_flag) ok = false;
        if (ok && li >= (uint32_t)QB)
          ok = mbar_wait(&q_empty[qb], ((li / QB) - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
        if (ok) {
          mbar_arrive_expect_tx(&q_full[qb], 2 * L::kDH * p.G * p.P * 128);
          for (int w = 0; w < 2; ++w)
            for (int dh = 0; dh < L::kDH; ++dh)
              tma_load_3d(smem + L::kOffQ + (qb * 2 + w) * L::kQTile + dh * L::kSlab, &tmap_q, &q_full[qb],
                          dh * 64, it.kvh * p.G, it.q0 + it.p0 + w * p.P);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ++li;
      const int64_t* bt_row = p.bt + (int64_t)it.seq * p.bt_stride;
      for (int j = 0; j < it.ntiles && ok; ++j, ++g) {
        const int st = g % ST;
        if (lane == 0) {
          if (*abort_flag) ok = false;
          if (ok && g >= (uint32_t)ST)
            ok = mbar_wait(&kv_empty[st], ((g / ST) - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
          if (ok) mbar_arrive_expect_tx(&kv_full[st], (L::kSplitKV ? 1 : 2) * L::kKVTile);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        int y = static_cast<int>(p.num_slots);  // out of range -> zero fill
        int off = 0;
        if (lane < L::kBoxes) {
          const int grp = lane % (N / kBoxTokens), dh = lane / (N / kBoxTokens);
          const int tok = j * N + grp * kBoxTokens;
          if (tok < it.ctx) {
            const int64_t pb = __ldg(bt_row + tok / p.bs);
            if (pb >= 0 && pb < p.num_blocks) y = static_cast<int>(pb) * p.bs + tok % p.bs;
          }
          off = st * L::kKVTile + dh * N * 128 + grp * kBoxTokens * 128;
          tma_load_3d(smem + L::kOffK + off, &tmap_k, &kv_full[st], dh * 64, it.kvh, y);
          if (!L::kSplitKV) tma_load_3d(smem + L::kOffV + off, &tmap_v, &kv_full[st], dh * 64, it.kvh, y);
        }
        __syncwarp();
        if constexpr (L::kSplitKV) {
          k_pending = true;
          if (lane == 0) {
            if (*abort_flag) ok = false;
            if (ok && g >= (uint32_t)ST)
              ok = mbar_wait(&v_empty[st], ((g / ST) - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
            if (ok) mbar_arrive_expect_tx(&v_full[st], L::kKVTile);
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          if (lane < L::kBoxes)
            tma_load_3d(smem + L::kOffV + off, &tmap_v, &v_full[st], (lane / (N / kBoxTokens)) * 64, it.kvh, y);
          __syncwarp();
          k_pending = false;
        }
      }
      if (!ok) break;
    }
    if (!ok && lane == 0) *abort_flag = 1;
    // Copies still in flight (only after an abort) land before exit: the
    // last phase of every stage / Q buffer that was used.
    if (lane == 0) {
      const uint32_t gk = g + (k_pending ? 1u : 0u);  // K tiles issued
      for (uint32_t x = (gk > (uint32_t)ST ? gk - ST : 0); x < gk; ++x)
        mbar_wait(&kv_full[x % ST], (x / ST) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
      if (L::kSplitKV)
        for (uint32_t x = (g > (uint32_t)ST ? g - ST : 0); x < g; ++x)
          mbar_wait(&v_full[x % ST], (x / ST) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
      for (uint32_t x = (li > (uint32_t)QB ? li - QB : 0); x < li; ++x)
        mbar_wait(&q_full[x % QB], (x / QB) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
    }
  } else if (warp == kMmaWarp0 || warp == kMmaWarp1) {
    // ------------------------------------------------------------ MMA issuers
    // Warp 9 issues every MMA of M-tile 0, warp 10 every MMA of M-tile 1,
    // each from its lane 0 and each doing its own waits.  A wait (or any
    // synchronisation) right after a thread's MMAs stalls that thread for
    // some hundred cycles; with one issuer per M-tile the other issuer's
    // MMAs keep the tensor core busy meanwhile, and one M-tile's chain
    // (softmax -> P V, S -> softmax) never waits for the other's.  Shared
    // stages (Q, K, V) are released by a commit from each issuer.
    const int w = warp - kMmaWarp0;
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idesc_s = tc::instr_desc_f16(kBf16, kM, N, false, false);
      constexpr uint32_t idesc_o = tc::instr_desc_f16(kBf16, kM, D, false, true);
      const uint32_t sbase = smem_u32(smem);
      // Descriptor words of the first buffer of each operand (SW128, SBO
      // 1024; V is MN-major with its 64-column halves N*128 bytes apart).
      constexpr uint32_t kHi = tc::desc_hi_sw128(1024);
      const uint32_t q_lo = tc::desc_lo(sbase + L::kOffQ, 16);
      const uint32_t k_lo = tc::desc_lo(sbase + L::kOffK, 16);
      const uint32_t v_lo = tc::desc_lo(sbase + L::kOffV, N * 128);
      const uint32_t s_tmem = tmem + w * L::kWgCols + L::kTmemS;
      const uint32_t p_tmem = tmem + w * L::kWgCols + L::kTmemP;
      const uint32_t o_tmem = tmem + w * L::kWgCols + L::kTmemO;
      // O_w (+)= P_w V(stage): P_w from TMEM (8 columns per K=16 step), V
      // from shared memory; one add per MMA (compile-time offsets).
      // K steps [k0, k1) of the tile (keys 16*k0 .. 16*k1-1).
      auto issue_pv_steps = [&](int stage, bool accumulate, int k0, int k1) {
        tc::fence_after_sync();
        const uint32_t b0 = v_lo + stage * (L::kKVTile >> 4);
#pragma unroll
        for (int kk = 0; kk < N / 16; ++kk)
          if (kk >= k0 && kk < k1)
            tc::mma_ts_words(o_tmem, p_tmem + kk * 8, b0 + ((kk * 2048) >> 4), kHi, idesc_o,
                             (accumulate || kk > 0) ? 1u : 0u);
      };
      // S_w = Q_w K(stage)^T, both from shared memory.
      auto issue_s = [&](int qb, int stage) {
        tc::fence_after_sync();
        const uint32_t a0 = q_lo + (qb * 2 + w) * (L::kQTile >> 4);
        const uint32_t b0 = k_lo + stage * (L::kKVTile >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_ss_words(s_tmem, a0 + (((kk >> 2) * L::kSlab + (kk & 3) * 32) >> 4),
                           b0 + (((kk >> 2) * N * 128 + (kk & 3) * 32) >> 4), kHi, idesc_s, kk > 0 ? 1u : 0u);
        tc::commit(&s_full[w]);
      };
      bool ok = true;
      auto wait = [&](uint64_t* bar, uint32_t parity, int code) {
#if PA_PREFILL_SPIN_ISSUER
        ok = ok && mbar_wait_spin(bar, parity, p.status, code) && !*abort_flag;
#else
        ok = ok && mbar_wait(bar, parity, p.status, code) && !*abort_flag;
#endif
        return ok;
      };
      uint32_t li = 0, g = 0;
      // P_w(t) V(t) once P_w(t) is in TMEM (and O_w read out, for an item's
      // first P V).
      auto pv_when_ready = [&](uint32_t t, bool accumulate, bool first_of_item) {
        wait(&p_full[w], t & 1, PA_DEVICE_TIMEOUT_MMA);
        if (first_of_item && li > 0) wait(&o_empty[w], (li - 1) & 1, PA_DEVICE_TIMEOUT_MMA);
        if (!ok) return false;
        issue_pv_steps(t % ST, accumulate, 0, N / 16);
        return true;
      };
      for (uint32_t cons = 0; ok; ++cons) {
        const int rs = cons % L::kRing;
        if (!wait(&item_full[rs], (cons / L::kRing) & 1, PA_DEVICE_TIMEOUT_TMA)) break;
        const int idx = ring[rs];
        mbar_arrive(&item_empty[rs]);
        Item it;
        if (idx < 0 || !item_at(p, idx, N, it)) break;
        const int ntiles = it.ntiles;
        const int qb = li % QB;
        for (int j = 0; j < ntiles && ok; ++j, ++g) {
          const int st = g % ST;
          if (j == 0) wait(&q_full[qb], (li / QB) & 1, PA_DEVICE_TIMEOUT_TMA);
          wait(&kv_full[st], (g / ST) & 1, PA_DEVICE_TIMEOUT_TMA);
          // Issuer 1 queues its MMAs of tile g behind issuer 0's, so the
          // tensor core finishes M-tile 0's work first and the two softmax
          // groups stay an MMA group apart instead of exponentiating at the
          // same time.  (turn[st] completes once per use of stage st; issuer
          // 0 cannot reuse the stage before issuer 1 has released it.)
          if (w == 1) wait(&turn[st], (g / ST) & 1, PA_DEVICE_TIMEOUT_MMA);
          if constexpr (L::kAliasP) {
            // P_w(g-1) sits in S_w's columns: its P V goes first, then
            // S_w(g) overwrites them (one thread's MMAs run in issue order),
            // and the commit after S_w(g) also tells the softmax that O_w
            // holds the P V of tile g-1.
            if (j > 0) {
              wait(&v_full[(g - 1) % ST], ((g - 1) / ST) & 1, PA_DEVICE_TIMEOUT_TMA);
              if (!pv_when_ready(g - 1, j > 1, j == 1)) break;
              tc::commit(&v_empty[(g - 1) % ST]);
            }
            if (!ok) break;
            issue_s(qb, st);
            tc::commit(&kv_empty[st]);  // K(g)
            if (j == ntiles - 1) tc::commit(&q_empty[qb]);  // the item's last read of Q_w
            if (w == 0) mbar_arrive(&turn[st]);
          } else {
            // S_w(g) once K(g) is in and the softmax has read S_w(g-1), then
            // P_w(g-1) V(g-1) once P_w(g-1) is in TMEM.
            if (g > 0) wait(&s_free[w], (g - 1) & 1, PA_DEVICE_TIMEOUT_MMA);
            if (!ok) break;
            issue_s(qb, st);
            if (j == ntiles - 1) tc::commit(&q_empty[qb]);  // the item's last read of Q_w
            if (w == 0) mbar_arrive(&turn[st]);
            if (j > 0) {
              if (!pv_when_ready(g - 1, j > 1, j == 1)) break;
              tc::commit(&pv_done[w]);
              tc::commit(&kv_empty[(g - 1) % ST]);
            }
          }
        }
        if (!ok) break;
        // Last P V of the item, then release its K/V stage (its Q buffer
        // went with the last S).
        if (L::kSplitKV) wait(&v_full[(g - 1) % ST], ((g - 1) / ST) & 1, PA_DEVICE_TIMEOUT_TMA);
        if (!ok || !pv_when_ready(g - 1, ntiles > 1, ntiles == 1)) break;
        tc::commit(&pv_done[w]);
        tc::commit(L::kSplitKV ? &v_empty[(g - 1) % ST] : &kv_empty[(g - 1) % ST]);
        ++li;
      }
      if (!ok) *abort_flag = 1;
      // Every MMA this thread issued has retired before TMEM is released.
      tc::commit(&mma_done[w]);
      mbar_wait(&mma_done[w], 0, p.status, PA_DEVICE_TIMEOUT_MMA);
    }
    __syncwarp();
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------ softmax
    const int w = warp >> 2;                 // M-tile of this group
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int r = quarter * 32 + lane;       // row of the M-tile = TMEM lane
    const uint32_t wg_addr = tmem + ((uint32_t)(quarter * 32) << 16) + w * L::kWgCols;
    const int pl = r / p.G, hj = r - (r / p.G) * p.G;
    const bool row_in_tile = r < p.G * p.P;
    uint32_t li = 0, t = 0;
    bool ok = true;
    for (uint32_t cons = 0; ok; ++cons) {
      const int rs = cons % L::kRing;
      ok = mbar_wait(&item_full[rs], (cons / L::kRing) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
      ok = __all_sync(0xffffffffu, ok);
      const int idx = ring[rs];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[rs]);
      if (!ok || idx < 0) break;
      Item it;
      item_at(p, idx, N, it);
      const int p0w = it.p0 + w * p.P;
      const int npw = max(0, min(p.P, it.C - p0w));
      const bool live = row_in_tile && pl < npw;
      const int Lr = it.prefix + p0w + min(pl, max(npw - 1, 0));
      const int nfull = (it.prefix + p0w + 1) / N;
      float m_run = -INFINITY, l = 0.f;
      for (int j = 0; j < it.ntiles; ++j, ++t) {
        constexpr bool kSpin = D == 64 ? PA_PREFILL_SPIN_SOFTMAX64 : PA_PREFILL_SPIN_SOFTMAX128;
        ok = (kSpin ? mbar_wait_spin(&s_full[w], t & 1, p.status, PA_DEVICE_TIMEOUT_MMA)
                    : mbar_wait(&s_full[w], t & 1, p.status, PA_DEVICE_TIMEOUT_MMA)) &&
             !*abort_flag;
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc::fence_after_sync();
        uint32_t su[N];  // S row as raw bits
#pragma unroll
        for (int c = 0; c < N / 32; ++c) tc::tmem_ld32(wg_addr + L::kTmemS + c * 32, su + c * 32);
        tc::tmem_wait_ld();
        if constexpr (!L::kAliasP) {
          tc::fence_before_sync();
          mbar_arrive(&s_free[w]);  // S_w may now be overwritten by the next tile's S
        }
        if (j >= nfull) {
          const int lim = Lr - j * N;  // keep keys k <= lim
#pragma unroll
          for (int k = 0; k < N; ++k) su[k] = (k <= lim) ? su[k] : 0xff800000u;  // -inf
        }
#define SV(k) __uint_as_float(su[k])
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int q = 0; q < N / 2; ++q) mx4[q & 3] = fmax3(mx4[q & 3], SV(2 * q), SV(2 * q + 1));
        const float mx = fmax3(fmax3(mx4[0], mx4[1], mx4[2]), mx4[3], mx4[3]) * p.scale_log2;
        // The P V of the previous tile must finish before O_w is rescaled or
        // P_w overwritten; wait for it only where needed, so the exponentials
        // below overlap it.  (Waiting before every P store also keeps this
        // group at most one p_full phase ahead of the MMA warp.)
        // (With P over S, the S_w(t) commit waited for above already covers
        // the P V of tile t-1.)
        bool pv_waited = t == 0 || L::kAliasP;
        auto wait_pv = [&]() {
          if (pv_waited) return true;
          pv_waited = true;
          bool w_ok = mbar_wait(&pv_done[w], (t - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
          w_ok = __all_sync(0xffffffffu, w_ok);
          if (w_ok) tc::fence_after_sync();
          return w_ok;
        };
        if (j == 0) {
          m_run = mx;  // key 0 is always visible: finite
        } else {
          const float m_new = fmaxf(m_run, mx);
          const bool need = m_new > m_run + kRescaleLog2;
          if (__any_sync(0xffffffffu, need)) {
            // O_w holds P V up to tile j-1: scale the rows that need it.
            ok = wait_pv();
            if (!ok) break;
            const float alpha = need ? fast_exp2(m_run - m_new) : 1.f;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t ov[32];
              tc::tmem_ld32(wg_addr + L::kTmemO + c * 32, ov);
              tc::tmem_wait_ld();
#pragma unroll
              for (int d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
              tc::tmem_st32(wg_addr + L::kTmemO + c * 32, ov);
            }
            tc::tmem_wait_st();
            if (need) {
              l *= alpha;
              m_run = m_new;
            }
          }
        }
        if (j == it.ntiles - 1 && r < N) {
          // V rows past the context (stale or poisoned slots of the last
          // block) are zeroed so 0-probability columns contribute exactly 0.
          // Both groups zero them before their P is published: each M-tile's
          // P V is issued by its own thread after its own group's zeroing,
          // and the other group's stores write the same zero bytes.
          const int tok = j * N + r;
          if (tok >= it.ctx) {
            const int st = t % ST;
            if (mbar_wait(L::kSplitKV ? &v_full[st] : &kv_full[st], (t / ST) & 1, p.status, PA_DEVICE_TIMEOUT_TMA)) {
#pragma unroll
              for (int dh = 0; dh < L::kDH; ++dh) {
                uint8_t* vrow = smem + L::kOffV + st * L::kKVTile + dh * N * 128 + r * 128;
#pragma unroll
                for (int c = 0; c < 8; ++c) *reinterpret_cast<int4*>(vrow + c * 16) = make_int4(0, 0, 0, 0);
              }
            }
          }
        }
        // P = 2^(s * scale_log2 - m_run), two columns per packed FP32 op;
        // kPoly of every 8 column pairs use the FMA-pipe exp2, the
        // rest the MUFU one, so the two pipes share the load.
        constexpr int kPoly = D == 64 ? PA_PREFILL_POLY64 : PA_PREFILL_POLY128;
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
        const float2 negm2 = make_float2(-m_run, -m_run);
        float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        uint32_t pk[N / 2];  // P row, two 16-bit values per 32-bit TMEM column
        const uint32_t p_addr = wg_addr + L::kTmemP;
#pragma unroll
        for (int c = 0; c < N / 8; ++c) {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const int q = c * 4 + h;
            const float2 x = __ffma2_rn(make_float2(SV(2 * q), SV(2 * q + 1)), sc2, negm2);
            float2 e;
            if ((q & 7) < kPoly) {
              e = exp2_poly2(x);
            } else {
              e.x = fast_exp2(x.x);
              e.y = fast_exp2(x.y);
            }
            sum2[h] = __fadd2_rn(sum2[h], e);
            pk[q] = pack2<T>(e.x, e.y);
          }
        }
        ok = wait_pv();
        if (!ok) break;
#pragma unroll
        for (int c = 0; c + 32 <= N / 2; c += 32) tc::tmem_st32(p_addr + c, pk + c);
        if ((N / 2) % 32) tc::tmem_st16(p_addr + (N / 2) / 32 * 32, pk + (N / 2) / 32 * 32);
        tc::tmem_wait_st();
#undef SV
        const float2 s01 = __fadd2_rn(sum2[0], sum2[1]), s23 = __fadd2_rn(sum2[2], sum2[3]);
        const float2 s0123 = __fadd2_rn(s01, s23);
        l += s0123.x + s0123.y;
        fence_proxy_async_smem();  // V rows zeroed above (generic proxy) -> MMA reads
        tc::fence_before_sync();
        mbar_arrive(&p_full[w]);
      }
      if (!ok) break;
      // Epilogue: the item's last P V has landed in O_w (pv_done completes
      // once per tile, or once per item with P over S).
      const uint32_t pv_phase = L::kAliasP ? li : t - 1;
      ok = mbar_wait(&pv_done[w], pv_phase & 1, p.status, PA_DEVICE_TIMEOUT_MMA) && !*abort_flag;
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc::fence_after_sync();
      const float inv = 1.f / l;
      T* out = reinterpret_cast<T*>(p.out) + (int64_t)(it.q0 + p0w + pl) * p.o_s0 +
               (int64_t)(it.kvh * p.G + hj) * p.o_s1;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        tc::tmem_ld32(wg_addr + L::kTmemO + c * 32, ov);
        tc::tmem_wait_ld();
        if (live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            int4 v;
            v.x = static_cast<int>(pack2<T>(__uint_as_float(ov[q * 8 + 0]) * inv, __uint_as_float(ov[q * 8 + 1]) * inv));
            v.y = static_cast<int>(pack2<T>(__uint_as_float(ov[q * 8 + 2]) * inv, __uint_as_float(ov[q * 8 + 3]) * inv));
            v.z = static_cast<int>(pack2<T>(__uint_as_float(ov[q * 8 + 4]) * inv, __uint_as_float(ov[q * 8 + 5]) * inv));
            v.w = static_cast<int>(pack2<T>(__uint_as_float(ov[q * 8 + 6]) * inv, __uint_as_float(ov[q * 8 + 7]) * inv));
            *reinterpret_cast<int4*>(out + c * 32 + q * 8) = v;
          }
        }
      }
      tc::fence_before_sync();
      mbar_arrive(&o_empty[w]);
      ++li;
    }
    if (!ok) *abort_flag = 1;
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, L::kTmemCols);
  }
  if (threadIdx.x == 0 && p.claim != nullptr) {
    // Every claim of this CTA precedes this point; the last CTA through
    // rewinds the counters for the next launch.
    __threadfence();
    if (atomicAdd(p.finish, 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(p.claim, 0);
      atomicExch(p.finish, 0);
    }
  }
}

int current_device_id() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

template <typename T, int D>
int launch_typed(const PrefillTcArgs& a, const TcParams& p, cudaStream_t st) {
  using L = Lay<D>;
  CUtensorMap tq, tk, tv;
  const int es = 2;
  if (make_map_3d(&tq, a.dtype, a.q, D, a.Hq, a.total_q, (uint64_t)a.q_s1 * es, (uint64_t)a.q_s0 * es, 64, a.group,
                  p.P, CU_TENSOR_MAP_SWIZZLE_128B) != PA_OK)
    return PA_ERR_CUDA;
  const uint64_t s1b = (uint64_t)D * es, s2b = s1b * a.Hkv;
  if (make_map_3d(&tk, a.dtype, a.kp, D, a.Hkv, p.num_slots, s1b, s2b, 64, 1, kBoxTokens,
                  CU_TENSOR_MAP_SWIZZLE_128B) != PA_OK ||
      make_map_3d(&tv, a.dtype, a.vp, D, a.Hkv, p.num_slots, s1b, s2b, 64, 1, kBoxTokens,
                  CU_TENSOR_MAP_SWIZZLE_128B) != PA_OK)
    return PA_ERR_CUDA;
  static bool attr_done[64] = {};
  const int dev = current_device_id();
  if (dev < 0 || dev >= 64) return PA_ERR_CUDA;
  auto kern = prefill_tc_kernel<T, D>;
  if (!attr_done[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmem) != cudaSuccess)
      return PA_ERR_CUDA;
    attr_done[dev] = true;
  }
  const int grid = std::min(p.num_items, num_sms(dev));
  kern<<<grid, kThreads, L::kSmem, st>>>(tq, tk, tv, p);
  PA_CHECK_LAUNCH();
  return PA_OK;
}

}  // namespace

bool prefill_tc_supported(const PrefillTcArgs& a) {
  if (a.dtype != PA_DTYPE_BF16 && a.dtype != PA_DTYPE_F16) return false;
  if (a.D != 64 && a.D != 128) return false;
  if (a.bs % kBoxTokens != 0) return false;
  if (a.group < 1 || a.group > kM) return false;
  if (a.num_blocks * (int64_t)a.bs >= (int64_t(1) << 31) || a.total_q >= (int64_t(1) << 31)) return false;
  if (a.max_q_len <= 0) return false;
  const auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!al16(a.q) || !al16(a.out) || !al16(a.kp) || !al16(a.vp)) return false;
  if ((a.q_s0 % 8) || (a.q_s1 % 8) || (a.o_s0 % 8) || (a.o_s1 % 8)) return false;
  return true;
}

int launch_prefill_tc(const PrefillTcArgs& a, cudaStream_t st) {
  TcParams p;
  p.cu_q = a.cu_q;
  p.context_lens = a.context_lens;
  p.bt = a.bt;
  p.bt_stride = a.bt_stride;
  p.bt_width = a.bt_width;
  p.num_blocks = a.num_blocks;
  p.num_slots = a.num_blocks * (int64_t)a.bs;
  p.ctx_cap = std::min<int64_t>(a.bt_width * (int64_t)a.bs, (int64_t(1) << 31) - 1);
  p.total_q = a.total_q;
  p.out = a.out;
  p.o_s0 = a.o_s0;
  p.o_s1 = a.o_s1;
  p.G = a.group;
  p.P = kM / a.group;
  p.bs = a.bs;
  p.Hkv = a.Hkv;
  p.num_seqs = a.num_seqs;
  p.pairs = (a.max_q_len + 2 * p.P - 1) / (2 * p.P);
  const int64_t items = (int64_t)p.pairs * a.num_seqs * a.Hkv;
  if (items <= 0) return PA_OK;
  if (items >= (int64_t(1) << 31)) return PA_ERR_INVALID;
  p.num_items = static_cast<int>(items);
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.status = a.control;
  p.claim = a.control != nullptr ? a.control + 1 : nullptr;
  p.finish = a.control != nullptr ? a.control + 2 : nullptr;
  const bool bf16 = a.dtype == PA_DTYPE_BF16;
  if (a.D == 64) return bf16 ? launch_typed<__nv_bfloat16, 64>(a, p, st) : launch_typed<__half, 64>(a, p, st);
  return bf16 ? launch_typed<__nv_bfloat16, 128>(a, p, st) : launch_typed<__half, 128>(a, p, st);
}

}  // namespace pa
