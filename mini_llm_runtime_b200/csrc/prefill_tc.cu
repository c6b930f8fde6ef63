// tcgen05 causal chunk-prefill over a paged KV cache (BF16/F16, head_dim 64).
//
// Math: for every query row of a chunk, softmax(scale * q K^T) V over the
// keys at absolute positions <= prefix + i (reference:
// kernels/reference/paged_attention.py:346-434 — the tiled online softmax
// of :398-431 — and its dense twin :282-343).
//
// Work unit (one CTA): (sequence, KV head, M-tile).  The M-tile packs the
// whole GQA group into the 128 MMA rows: row r = (query position r / G,
// query head r % G), P = floor(128 / G) positions per tile (18 for Qwen2.5's
// group of 7 -> 126 live rows), so every K/V tile loaded from the paged pool
// feeds all G query heads at once.  Tiles with the largest query positions
// (most KV tiles) launch first.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: Q tile once (3-D box {64, G, P} straight from
//               the packed [T, Hq, D] tensor), then per 128-token KV tile 8+8
//               boxes {64, 1, 16} addressed through the block table into a
//               2-stage ring (128-byte swizzle, canonical UMMA K-major
//               layout).  Blocks past the context use an out-of-range
//               coordinate, which TMA fills with zeros.
//   warp 1      TMEM owner + single-thread MMA issuer:
//                 S_j = Q K_j^T   (M128 N128 K64, both K-major)  -> TMEM S[j%2]
//                 O_j = P_j V_j   (M128 N64 K128, V as MN-major B) -> TMEM O[j%2]
//               S_{j+1} is issued before O_j so QK^T of the next tile overlaps
//               the softmax of this one.
//   warps 2..5  softmax: one thread per row (TMEM lane), FP32 online softmax
//               in the log2 domain, causal mask only on diagonal tiles,
//               P written to shared memory as BF16/F16 (SW128 K-major),
//               O tile read back from TMEM and accumulated in registers with
//               the running rescale, final 1/l and store.
// Every mbarrier wait is bounded (status word + early exit); TMEM is freed
// on every path.
#include <type_traits>

#include "prefill_tc.cuh"
#include "tcgen05.cuh"

namespace pa {
namespace {

constexpr int kM = 128;      // MMA rows (packed query positions x heads)
constexpr int kN = 128;      // KV tokens per tile
constexpr int kD = 64;       // head_dim
constexpr int kStages = 2;   // K/V ring depth
constexpr int kThreads = 192;
constexpr int kTileBytes = kN * kD * 2;  // 16 KB: one K, V or Q tile
constexpr int kPBytes = kM * kN * 2;     // 32 KB: one P tile
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;
constexpr int kOffV = kOffK + kStages * kTileBytes;
constexpr int kOffP = kOffV + kStages * kTileBytes;
constexpr int kOffBar = kOffP + 2 * kPBytes;
constexpr int kNumBars = 1 + 2 * kStages + 8 + 1;
constexpr int kOffTmem = kOffBar + kNumBars * 8;
constexpr size_t kSmem = 1024 + kOffTmem + 16;
constexpr uint32_t kTmemCols = 512;  // S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384)
constexpr uint32_t kTmemS = 0, kTmemO = 256;

struct TcParams {
  const int64_t* cu_q;
  const int64_t* context_lens;
  const int64_t* bt;
  int64_t bt_stride, bt_width;
  int64_t num_slots;
  void* out;
  int64_t o_s0, o_s1;
  int G, P, bs, mtiles;
  float scale_log2;
  int* status;
};

template <typename T> struct Pack2;
template <> struct Pack2<__nv_bfloat16> {
  __device__ __forceinline__ static uint32_t run(float a, float b) { return MmaOp<__nv_bfloat16>::pack(a, b); }
};
template <> struct Pack2<__half> {
  __device__ __forceinline__ static uint32_t run(float a, float b) { return MmaOp<__half>::pack(a, b); }
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                                                                const __grid_constant__ CUtensorMap tmap_k,
                                                                const __grid_constant__ CUtensorMap tmap_v,
                                                                TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kStages;
  uint64_t* s_full = kv_empty + kStages;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_free = o_full + 2;
  uint64_t* mma_done = o_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = blockIdx.z, kvh = blockIdx.y;
  const int mt = p.mtiles - 1 - static_cast<int>(blockIdx.x);
  const int64_t q0 = p.cu_q[seq];
  const int64_t C = p.cu_q[seq + 1] - q0;
  int64_t ctx = p.context_lens[seq];
  const int64_t cap = p.bt_width * (int64_t)p.bs;
  if (ctx > cap) ctx = cap;
  const int64_t prefix = ctx - C;
  const int64_t p0 = (int64_t)mt * p.P;
  if (C <= 0 || prefix < 0 || p0 >= C) return;  // uniform for the CTA
  const int np = static_cast<int>(min((int64_t)p.P, C - p0));
  const int64_t Lmin = prefix + p0;
  const int64_t Lmax = prefix + p0 + np - 1;
  const int ntiles = static_cast<int>(Lmax / kN) + 1;
  const int nfull = static_cast<int>((Lmin + 1) / kN);  // tiles below need no mask

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&tmap_q);
      prefetch_tensormap(&tmap_k);
      prefetch_tensormap(&tmap_v);
      const int qrows = p.G * p.P;
      for (int r = qrows; r < kM; ++r)
        for (int c = 0; c < 8; ++c) *reinterpret_cast<int4*>(smem + kOffQ + r * 128 + c * 16) = make_int4(0, 0, 0, 0);
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(q_full, qrows * 128);
      tma_load_3d(smem + kOffQ, &tmap_q, q_full, 0, kvh * p.G, static_cast<int>(q0 + p0));
      const int64_t* bt_row = p.bt + (int64_t)seq * p.bt_stride;
      bool ok = true;
      int issued = 0;
      for (int j = 0; j < ntiles && ok; ++j) {
        const int st = j % kStages;
        if (j >= kStages) ok = mbar_wait(&kv_empty[st], ((j / kStages) - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
        if (!ok) break;
        ++issued;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kTileBytes);
        for (int i = 0; i < kN / 16; ++i) {
          const int64_t tok = (int64_t)j * kN + i * 16;
          int y = static_cast<int>(p.num_slots);  // out of range -> zero fill
          if (tok < ctx) {
            const int64_t pb = bt_row[tok / p.bs];
            y = static_cast<int>(pb * p.bs + tok % p.bs);
          }
          tma_load_3d(smem + kOffK + st * kTileBytes + i * 2048, &tmap_k, &kv_full[st], 0, kvh, y);
          tma_load_3d(smem + kOffV + st * kTileBytes + i * 2048, &tmap_v, &kv_full[st], 0, kvh, y);
        }
      }
      // Copies still in flight (only on an aborted run) must land before exit.
      for (int j = max(0, issued - kStages); j < issued; ++j)
        mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      constexpr uint32_t idesc_s = tc::instr_desc_f16(kBf16, kM, kN, false, false);
      constexpr uint32_t idesc_o = tc::instr_desc_f16(kBf16, kM, kD, false, true);
      bool ok = mbar_wait(q_full, 0, p.status, PA_DEVICE_TIMEOUT_TMA);
      tc::fence_after_sync();
      const uint32_t qaddr = smem_u32(smem + kOffQ);
      for (int j = 0; j <= ntiles && ok; ++j) {
        if (j < ntiles) {
          const int st = j % kStages;
          ok = mbar_wait(&kv_full[st], (j / kStages) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
          if (!ok) break;
          tc::fence_after_sync();
          const uint32_t kaddr = smem_u32(smem + kOffK + st * kTileBytes);
          const uint32_t d_s = tmem + kTmemS + (j & 1) * kN;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            tc::mma_ss(d_s, tc::smem_desc_sw128(qaddr + kk * 32, 16, 1024),
                       tc::smem_desc_sw128(kaddr + kk * 32, 16, 1024), idesc_s, kk > 0);
          }
          tc::commit(&s_full[j & 1]);
        }
        if (j >= 1) {
          const int jp = j - 1, b = jp & 1, stp = jp % kStages;
          ok = mbar_wait(&p_full[b], (jp >> 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
          if (ok && jp >= 2) ok = mbar_wait(&o_free[b], ((jp >> 1) - 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
          if (!ok) break;
          tc::fence_after_sync();
          const uint32_t paddr = smem_u32(smem + kOffP + b * kPBytes);
          const uint32_t vaddr = smem_u32(smem + kOffV + stp * kTileBytes);
          const uint32_t d_o = tmem + kTmemO + b * kD;
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk) {
            const uint64_t a = tc::smem_desc_sw128(paddr + (kk >> 2) * (kM * 128) + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = tc::smem_desc_sw128(vaddr + kk * 2048, 16, 1024);
            tc::mma_ss(d_o, a, bd, idesc_o, kk > 0);
          }
          tc::commit(&o_full[b]);
          tc::commit(&kv_empty[stp]);
        }
      }
      // Every MMA this thread issued has retired before TMEM is released
      // (immediate on the normal path; bounded on an aborted one).
      tc::commit(mma_done);
      mbar_wait(mma_done, 0, p.status, PA_DEVICE_TIMEOUT_MMA);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int pl = r / p.G, hj = r - pl * p.G;
    const bool row_live = (r < p.G * p.P) && (pl < np);
    const int64_t Lr = prefix + p0 + min(pl, np - 1);
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    float oacc[kD];
#pragma unroll
    for (int d = 0; d < kD; ++d) oacc[d] = 0.f;
    bool ok = true;
    // Iteration j: softmax of tile j (j < ntiles), then fold O_{j-1} into
    // the register accumulator while the tensor core computes O_j / S_{j+1}.
    for (int j = 0; j <= ntiles; ++j) {
      float alpha = 1.f;
      if (j < ntiles) {
        const int b = j & 1;
        if (ok) ok = mbar_wait(&s_full[b], (j >> 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
        tc::fence_after_sync();
        uint32_t su[kN];
#pragma unroll
        for (int c = 0; c < kN / 32; ++c) tc::tmem_ld32(lane_addr + kTmemS + b * kN + c * 32, su + c * 32);
        tc::tmem_wait_ld();
        float sv[kN];
#pragma unroll
        for (int k = 0; k < kN; ++k) sv[k] = __uint_as_float(su[k]);
        if (j >= nfull) {
          const int64_t lim64 = Lr - (int64_t)j * kN;  // keep tokens k <= lim
          const int lim = static_cast<int>(lim64 > kN ? kN : lim64);
#pragma unroll
          for (int k = 0; k < kN; ++k) sv[k] = (k <= lim) ? sv[k] : -INFINITY;
        }
        float mx = sv[0];
#pragma unroll
        for (int k = 1; k < kN; ++k) mx = fmaxf(mx, sv[k]);
        const float m_new = fmaxf(m, mx * p.scale_log2);
        alpha = exp2f(m - m_new);
        if (j == ntiles - 1) {
          // V rows past the context (stale or NaN-poisoned slots of the last
          // block) are zeroed so that 0-probability columns stay exactly 0.
          const int64_t tok = (int64_t)j * kN + r;
          if (tok >= ctx) {
            if (ok) ok = mbar_wait(&kv_full[j % kStages], (j / kStages) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
            uint8_t* vrow = smem + kOffV + (j % kStages) * kTileBytes + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) *reinterpret_cast<int4*>(vrow + c * 16) = make_int4(0, 0, 0, 0);
          }
        }
        float sum = 0.f;
        uint8_t* prow = smem + kOffP + b * kPBytes + r * 128;
#pragma unroll
        for (int c = 0; c < kN / 8; ++c) {
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            e[i] = exp2f(fmaf(sv[c * 8 + i], p.scale_log2, -m_new));
            sum += e[i];
          }
          int4 v;
          v.x = static_cast<int>(Pack2<T>::run(e[0], e[1]));
          v.y = static_cast<int>(Pack2<T>::run(e[2], e[3]));
          v.z = static_cast<int>(Pack2<T>::run(e[4], e[5]));
          v.w = static_cast<int>(Pack2<T>::run(e[6], e[7]));
          const int chunk = c & 7;
          *reinterpret_cast<int4*>(prow + (c >> 3) * (kM * 128) + ((chunk ^ (r & 7)) << 4)) = v;
        }
        l = l * alpha + sum;
        m = m_new;
        fence_proxy_async_smem();
        tc::fence_before_sync();
        mbar_arrive(&p_full[b]);
      }
      if (j >= 1) {
        const int jt = j - 1, bo = jt & 1;
        if (ok) ok = mbar_wait(&o_full[bo], (jt >> 1) & 1, p.status, PA_DEVICE_TIMEOUT_MMA);
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t ov[32];
          tc::tmem_ld32(lane_addr + kTmemO + bo * kD + c * 32, ov);
          tc::tmem_wait_ld();
#pragma unroll
          for (int d = 0; d < 32; ++d)
            oacc[c * 32 + d] = fmaf(oacc[c * 32 + d], alpha_prev, __uint_as_float(ov[d]));
        }
        tc::fence_before_sync();
        mbar_arrive(&o_free[bo]);
      }
      alpha_prev = alpha;
    }

    if (row_live) {
      const float inv = 1.f / l;
      T* out = reinterpret_cast<T*>(p.out) + (q0 + p0 + pl) * p.o_s0 + (int64_t)(kvh * p.G + hj) * p.o_s1;
#pragma unroll
      for (int c = 0; c < kD / 8; ++c) {
        int4 v;
        v.x = static_cast<int>(Pack2<T>::run(oacc[c * 8 + 0] * inv, oacc[c * 8 + 1] * inv));
        v.y = static_cast<int>(Pack2<T>::run(oacc[c * 8 + 2] * inv, oacc[c * 8 + 3] * inv));
        v.z = static_cast<int>(Pack2<T>::run(oacc[c * 8 + 4] * inv, oacc[c * 8 + 5] * inv));
        v.w = static_cast<int>(Pack2<T>::run(oacc[c * 8 + 6] * inv, oacc[c * 8 + 7] * inv));
        *reinterpret_cast<int4*>(out + c * 8) = v;
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

int current_device_id() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

bool prefill_tc_supported(const PrefillTcArgs& a) {
  if (a.dtype != PA_DTYPE_BF16 && a.dtype != PA_DTYPE_F16) return false;
  if (a.D != kD) return false;
  if (a.bs % 16 != 0 || a.bs > 256) return false;
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
  p.num_slots = a.num_blocks * (int64_t)a.bs;
  p.out = a.out;
  p.o_s0 = a.o_s0;
  p.o_s1 = a.o_s1;
  p.G = a.group;
  p.P = kM / a.group;
  p.bs = a.bs;
  p.mtiles = (a.max_q_len + p.P - 1) / p.P;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.status = a.status;

  CUtensorMap tq, tk, tv;
  const int es = 2;
  if (make_map_3d(&tq, a.dtype, a.q, kD, a.Hq, a.total_q, (uint64_t)a.q_s1 * es, (uint64_t)a.q_s0 * es, kD,
                  a.group, p.P, CU_TENSOR_MAP_SWIZZLE_128B) != PA_OK)
    return PA_ERR_CUDA;
  const uint64_t s1b = (uint64_t)kD * es, s2b = s1b * a.Hkv;
  if (make_map_3d(&tk, a.dtype, a.kp, kD, a.Hkv, p.num_slots, s1b, s2b, kD, 1, 16, CU_TENSOR_MAP_SWIZZLE_128B) !=
          PA_OK ||
      make_map_3d(&tv, a.dtype, a.vp, kD, a.Hkv, p.num_slots, s1b, s2b, kD, 1, 16, CU_TENSOR_MAP_SWIZZLE_128B) !=
          PA_OK)
    return PA_ERR_CUDA;

  static bool attr_done[2][64] = {};
  const int dev = current_device_id();
  if (dev < 0 || dev >= 64) return PA_ERR_CUDA;
  const int ti = a.dtype == PA_DTYPE_BF16 ? 0 : 1;
  auto kern = a.dtype == PA_DTYPE_BF16 ? prefill_tc_kernel<__nv_bfloat16> : prefill_tc_kernel<__half>;
  if (!attr_done[ti][dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess)
      return PA_ERR_CUDA;
    attr_done[ti][dev] = true;
  }
  if (a.num_seqs > 65535 || a.Hkv > 65535) return PA_ERR_INVALID;
  dim3 grid(p.mtiles, a.Hkv, a.num_seqs);
  kern<<<grid, kThreads, kSmem, st>>>(tq, tk, tv, p);
  PA_CHECK_LAUNCH();
  return PA_OK;
}

}  // namespace pa
