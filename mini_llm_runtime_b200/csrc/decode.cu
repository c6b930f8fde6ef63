// Batched single-token paged decode, split-KV with a log-sum-exp merge.
//
// Replaces paged_attention_decode_batch_parallel
// (kernels/reference/paged_attention.py:178-254) and generalises the Triton
// split-KV pair (kernels/triton/paged_attention.py:528-700 stage 1,
// :1530-1618 merge) to a ragged batch.
//
// Fast path (F16/BF16 queries over F16/BF16 or FP8 e4m3 pools, head_dim 64
// or 128, block_size % 16 == 0, batch <= 1024) — HBM-bound:
// decode_flat_kernel, then decode_combine_kernel.
//  * The batch's KV is one index space of 16-token sub-blocks ordered by
//    (sequence, KV-head pack, position).  Each CTA owns an equal contiguous
//    range of it and each warp an equal part of its CTA's range, so every SM
//    streams the same number of bytes whatever the context lengths.
//  * A warp streams its sub-blocks through its own TMA ring (3-D boxes
//    {64 dims, 1 head, 16 tokens}, 128-byte swizzle — 64-byte for FP8 —
//    mbarrier completion), looking the physical block of each sub-block up
//    in a lane-cached slice of the block table.
//  * S^T = K Q^T and O^T += V^T P^T use mma.sync m16n8k16 with FP32
//    accumulators, tokens / head dims as M and 8 query heads as N.  When a
//    GQA group has at most 8 query heads and the KV heads pair up, one warp
//    serves two KV heads at once, one 8-column tile each, so a group of 7
//    fills 7 of 8 columns of every MMA.  FP8 tiles feed the MMAs through
//    in-register e4m3 -> f16 conversion of the ldmatrix fragments.
//  * Online softmax in FP32, log2 domain (scores pre-multiplied by
//    scale * log2(e), exp2f).
//  * A segment (one sequence x one KV-head pack) that lies inside one warp's
//    range is finished by that warp.  Pieces of a segment cut by warp
//    boundaries are merged by log-sum-exp in shared memory at the end of the
//    CTA; a segment cut by CTA boundaries leaves one FP32 (m, l, O) record
//    per CTA, merged by decode_combine_kernel, a second PDL launch.  No CTA
//    waits for another one and nothing needs a memory fence: the kernel
//    boundary orders the records before the combine reads them.
// Tokens past context_len inside the last block are masked (-inf scores) and
// their V fragments zeroed, so stale or NaN-poisoned slots cannot leak in.
//
// decode_split_kernel serves batches above 1024 sequences (one CTA per
// (sequence, KV head, partition), last-ticket merge).  Everything else (F32,
// other head dims / block sizes) goes to the CUDA-core kernel in
// attn_generic.cu.
#include <type_traits>

#include "attn_generic.cuh"

// The decode kernels' K/V copies carry an L2 evict-first policy (1) or none
// (0): the pools are read once per call.
#ifndef PA_DECODE_KV_EVICT_FIRST
#define PA_DECODE_KV_EVICT_FIRST 1
#endif
// Early-inputs launches warm L2 with the first piece's query rows before the
// wait for the previous kernel (1) or not (0).
#ifndef PA_DECODE_Q_PREFETCH
#define PA_DECODE_Q_PREFETCH 1
#endif

namespace pa {
namespace {

constexpr int kSub = 16;            // tokens per sub-block
constexpr int kTileRowBytes = 128;  // one 64-wide column tile row (SW128 span)
constexpr int kTileBytes = kSub * kTileRowBytes;  // 2 KB: 16 tokens x 64 dims of one head

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset inside a 64-col SW128 tile
  return static_cast<uint32_t>(row * kTileRowBytes + ((chunk ^ (row & 7)) << 4));
}

// Query head (relative to the piece's first head) of record row r (column r
// % 8 of column tile r / 8), or -1 for padding.  PK = 2: rows 0-7 serve the
// first KV head's group, rows 8-15 the second's (group <= 8).  PK = 1: rows
// 0..hn-1 are consecutive heads.
template <int PK>
__device__ __forceinline__ int row_head(int r, int group, int hn) {
  if (PK == 2) {
    const int i = r & 7;
    return i < group ? (r < 8 ? i : group + i) : -1;
  }
  return r < hn ? r : -1;
}

// Four e4m3 values (bytes 0..3) as two f16x2 MMA registers (exact): lo =
// bytes 0, 1 and hi = bytes 2, 3, low byte in the low half.  The 32-bit
// register is split into its 16-bit halves in place, so no mask or shift
// precedes the conversions.
__device__ __forceinline__ void e4m3x4_to_f16x2(uint32_t v, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a 16 x 64-byte tile
// written by TMA with 64-byte swizzle (chunk bits 4-5 ^= address bits 7-8).
__device__ __forceinline__ uint32_t swz64(int row, int chunk) {
  return static_cast<uint32_t>(row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
}

// Two adjacent query elements as one MMA register (converted when the MMA
// type differs from the query type: FP8 pools run the MMAs in f16).
template <typename T, typename TQ>
__device__ __forceinline__ uint32_t q_pair(const TQ* p) {
  if constexpr (std::is_same<T, TQ>::value) {
    return load_pair_u32(p);
  } else {
    return MmaOp<T>::pack(Elem<TQ>::to_f32(p[0]), Elem<TQ>::to_f32(p[1]));
  }
}

// Online-softmax state of one warp for one piece of a segment, in the
// transposed orientation S^T = K Q^T, O^T = V^T P^T: 16 tokens (S^T) or 16
// head dims (O^T) are the MMA's M and 8 query heads its N.  A warp serves two
// column tiles j of 8 query heads: PK = 2, the GQA group of KV head j of the
// pack (<= 8 heads); PK = 1, heads 8j .. 8j + 7 of a <= 16-head tile (both
// read the same K/V, so one set of fragments serves both tiles).  A group of
// 7 heads then fills 7 of 8 columns of every MMA.  Column n of tile j is
// record row 8j + n.  FP32 (m, l) per column in the log2 domain.
//
// Shared-memory stage layout: tile t = (kv * kColTiles + ct) * PK + h holds
// 16 tokens x 64 dims of KV head h of the pack — 16-bit elements with
// 128-byte swizzle, or (P8) e4m3 bytes with 64-byte swizzle.
//  * S^T: A fragments are K rows straight from ldmatrix, B fragments Q^T.
//    P8: an ldmatrix lane receives 4 consecutive bytes (dims 4t .. 4t+3 of a
//    16-dim k-step) of one token; the k-step's dims are taken in the order
//    that makes those its A fragment (k-positions 2t, 2t+1, 2t+8, 2t+9 hold
//    dims 4t .. 4t+3), and the Q^T fragments use the same order, which leaves
//    every dot product unchanged.  The bytes are converted to f16 (exact) in
//    registers; no dequantized copy is written.
//  * P^T: the exponentiated S^T fragments, packed to 16 bits, become B
//    fragments (tokens 2t, 2t+1 of column g) by one movmatrix per 8x8 block.
//  * O^T: A fragments are V^T from ldmatrix.trans.  16-bit pools: rows g /
//    g + 8 of an m-tile are its dims g / g + 8.  P8: a lane receives bytes
//    (token 2t: dims 2g, 2g+1; token 2t+1: dims 2g, 2g+1); one byte permute
//    splits them into dim 2g (row g) and dim 2g + 1 (row g + 8).
// Per lane, accumulator element e of m-tile c of tile j holds column
// 2t + (e & 1) and dim 16c + (P8 ? 2g + (e >> 1) : g + 8 (e >> 1)).
template <typename T, int D, int PK, bool P8 = false>
struct WarpState {
  static constexpr int kKK = D / 16;  // k-steps of S^T; m-tiles of O^T
  static constexpr int kColTiles = D / 64;
  uint32_t qa[kKK][4];  // [kk][2j + i]: B fragment i of Q^T, column tile j
  float m[2][2], l[2][2];  // [j][column 2t + c]
  float o[2][kKK][4];

  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      m[j][0] = m[j][1] = -INFINITY;
      l[j][0] = l[j][1] = 0.f;
#pragma unroll
      for (int c = 0; c < kKK; ++c) o[j][c][0] = o[j][c][1] = o[j][c][2] = o[j][c][3] = 0.f;
    }
  }

  template <typename TQ>
  __device__ __forceinline__ static void load_q(uint32_t (&qa_out)[kKK][4], const TQ* qb, int64_t q_s1, int h0,
                                                int group, int hn, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int e = row_head<PK>(8 * j + g, group, hn);
      const TQ* p = qb + (int64_t)(h0 + (e < 0 ? 0 : e)) * q_s1;
#pragma unroll
      for (int kk = 0; kk < kKK; ++kk) {
        // P8: k-positions 2t, 2t+1 / 2t+8, 2t+9 take dims 4t, 4t+1 / 4t+2, 4t+3.
        const int c = kk * 16 + (P8 ? 4 * t : 2 * t), c2 = c + (P8 ? 2 : 8);
        qa_out[kk][2 * j] = e >= 0 ? q_pair<T, TQ>(p + c) : 0u;
        qa_out[kk][2 * j + 1] = e >= 0 ? q_pair<T, TQ>(p + c2) : 0u;
      }
    }
  }

  // Column tiles served by KV head h of the pack: PK = 2, tile h; PK = 1, both.
  static constexpr int kTilesPerHead = PK == 2 ? 1 : 2;

  template <int NSUB>
  __device__ __forceinline__ void consume(const uint32_t* stage, const int* valid, float scale_log2, int lane) {
    constexpr uint32_t kTile = P8 ? kSub * 64 : kTileBytes;
    constexpr uint32_t kVOff = kColTiles * PK * kTile;
    const int mi = lane >> 3, mr = lane & 7, g = lane >> 2, cq = 2 * (lane & 3);
    float s[NSUB][2][4];
#pragma unroll
    for (int u = 0; u < NSUB; ++u)
#pragma unroll
      for (int j = 0; j < 2; ++j) s[u][j][0] = s[u][j][1] = s[u][j][2] = s[u][j][3] = 0.f;
    // ---- S^T = K Q^T ----
#pragma unroll
    for (int u = 0; u < NSUB; ++u)
#pragma unroll
      for (int h = 0; h < PK; ++h) {
        if constexpr (P8) {
          // Matrices 0 / 1: tokens 0-7 / 8-15 of 16-byte chunk 2k'; 2 / 3: of chunk 2k' + 1.
          const int tok = (mi & 1) * 8 + mr;
#pragma unroll
          for (int kp = 0; kp < kKK / 2; ++kp) {
            uint32_t r0, r1, r2, r3;
            ldsm_x4(stage[u] + ((kp >> 1) * PK + h) * kTile + swz64(tok, 2 * (kp & 1) + (mi >> 1)), r0, r1, r2, r3);
            uint32_t a[4], b[4];
            e4m3x4_to_f16x2(r0, a[0], a[2]);
            e4m3x4_to_f16x2(r1, a[1], a[3]);
            e4m3x4_to_f16x2(r2, b[0], b[2]);
            e4m3x4_to_f16x2(r3, b[1], b[3]);
#pragma unroll
            for (int jj = 0; jj < kTilesPerHead; ++jj) {
              const int j = PK == 2 ? h : jj;
              MmaOp<T>::run(s[u][j], a, qa[2 * kp][2 * j], qa[2 * kp][2 * j + 1]);
              MmaOp<T>::run(s[u][j], b, qa[2 * kp + 1][2 * j], qa[2 * kp + 1][2 * j + 1]);
            }
          }
        } else {
          // Matrices: (tokens 0-7, dims 0-7), (8-15, 0-7), (0-7, 8-15), (8-15, 8-15) of the k-step.
          const int tok = (mi & 1) * 8 + mr;
#pragma unroll
          for (int kk = 0; kk < kKK; ++kk) {
            uint32_t a[4];
            ldsm_x4(stage[u] + ((kk >> 2) * PK + h) * kTile + swz(tok, 2 * (kk & 3) + (mi >> 1)), a[0], a[1], a[2],
                    a[3]);
#pragma unroll
            for (int jj = 0; jj < kTilesPerHead; ++jj) {
              const int j = PK == 2 ? h : jj;
              MmaOp<T>::run(s[u][j], a, qa[kk][2 * j], qa[kk][2 * j + 1]);
            }
          }
        }
      }
    // ---- online softmax over the columns (query heads) ----
    // Elements 0, 1: token g, columns cq, cq+1; elements 2, 3: token g + 8.
#pragma unroll
    for (int u = 0; u < NSUB; ++u)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = g + 8 * (e >> 1);
          s[u][j][e] = tok < valid[u] ? s[u][j][e] * scale_log2 : -INFINITY;
        }
    float mn[2][2], al[2][2];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < NSUB; ++u) mx = fmaxf(mx, fmaxf(s[u][j][c], s[u][j][c + 2]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        mn[j][c] = fmaxf(m[j][c], mx);
        al[j][c] = exp2f(m[j][c] - mn[j][c]);
        m[j][c] = mn[j][c];
      }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int u = 0; u < NSUB; ++u) {
        s[u][j][0] = exp2f(s[u][j][0] - mn[j][0]);
        s[u][j][1] = exp2f(s[u][j][1] - mn[j][1]);
        s[u][j][2] = exp2f(s[u][j][2] - mn[j][0]);
        s[u][j][3] = exp2f(s[u][j][3] - mn[j][1]);
        sum0 += s[u][j][0] + s[u][j][2];
        sum1 += s[u][j][1] + s[u][j][3];
      }
      l[j][0] = l[j][0] * al[j][0] + sum0;
      l[j][1] = l[j][1] * al[j][1] + sum1;
#pragma unroll
      for (int c = 0; c < kKK; ++c) {
        o[j][c][0] *= al[j][0];
        o[j][c][1] *= al[j][1];
        o[j][c][2] *= al[j][0];
        o[j][c][3] *= al[j][1];
      }
    }
    // ---- O^T += V^T P^T ----
#pragma unroll
    for (int u = 0; u < NSUB; ++u) {
      uint32_t pb[2][2];  // B fragments of P^T: tokens 2t, 2t+1 (0) / 2t+8, 2t+9 (1) of column g
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        pb[j][0] = movmatrix_t(MmaOp<T>::pack(s[u][j][0], s[u][j][1]));
        pb[j][1] = movmatrix_t(MmaOp<T>::pack(s[u][j][2], s[u][j][3]));
      }
      const int vu = valid[u];
      const bool partial = vu < kSub;
      // A registers of tokens cq, cq+1 (low / high half) and 8+cq, 9+cq:
      // tokens past the context are zeroed so stale / NaN slots cannot
      // reach the sum.
      const uint32_t mlo = (cq < vu ? 0x0000ffffu : 0u) | (cq + 1 < vu ? 0xffff0000u : 0u);
      const uint32_t mhi = (cq + 8 < vu ? 0x0000ffffu : 0u) | (cq + 9 < vu ? 0xffff0000u : 0u);
#pragma unroll
      for (int h = 0; h < PK; ++h) {
        if constexpr (P8) {
          const int tok = (mi & 1) * 8 + mr;
#pragma unroll
          for (int jp = 0; jp < kKK / 2; ++jp) {
            uint32_t r0, r1, r2, r3;
            ldsm_x4_t(stage[u] + kVOff + ((jp >> 1) * PK + h) * kTile + swz64(tok, 2 * (jp & 1) + (mi >> 1)), r0, r1,
                      r2, r3);
            if (partial) {  // r0 / r2: tokens cq, cq+1; r1 / r3: 8+cq, 9+cq
              r0 &= mlo;
              r2 &= mlo;
              r1 &= mhi;
              r3 &= mhi;
            }
            // Low half: dim 2g of both tokens (row g); high half: dim 2g+1 (row g+8).
            const uint32_t e0 = __byte_perm(r0, 0u, 0x3120), e1 = __byte_perm(r1, 0u, 0x3120);
            const uint32_t e2 = __byte_perm(r2, 0u, 0x3120), e3 = __byte_perm(r3, 0u, 0x3120);
            uint32_t a[4], b[4];
            e4m3x4_to_f16x2(e0, a[0], a[1]);
            e4m3x4_to_f16x2(e1, a[2], a[3]);
            e4m3x4_to_f16x2(e2, b[0], b[1]);
            e4m3x4_to_f16x2(e3, b[2], b[3]);
#pragma unroll
            for (int jj = 0; jj < kTilesPerHead; ++jj) {
              const int j = PK == 2 ? h : jj;
              MmaOp<T>::run(o[j][2 * jp], a, pb[j][0], pb[j][1]);
              MmaOp<T>::run(o[j][2 * jp + 1], b, pb[j][0], pb[j][1]);
            }
          }
        } else {
          // Matrices: (tokens 0-7, dims 0-7), (0-7, 8-15), (8-15, 0-7), (8-15, 8-15) of the m-tile.
          const int tok = (mi >> 1) * 8 + mr;
#pragma unroll
          for (int c = 0; c < kKK; ++c) {
            uint32_t a[4];
            ldsm_x4_t(stage[u] + kVOff + ((c >> 2) * PK + h) * kTile + swz(tok, 2 * (c & 3) + (mi & 1)), a[0], a[1],
                      a[2], a[3]);
            if (partial) {
              a[0] &= mlo;
              a[1] &= mlo;
              a[2] &= mhi;
              a[3] &= mhi;
            }
#pragma unroll
            for (int jj = 0; jj < kTilesPerHead; ++jj) {
              const int j = PK == 2 ? h : jj;
              MmaOp<T>::run(o[j][c], a, pb[j][0], pb[j][1]);
            }
          }
        }
      }
    }
  }

  // Sum the column sums over the 8 lanes of a column (tokens are spread that way).
  __device__ __forceinline__ void reduce_l() {
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        l[j][c] += __shfl_xor_sync(0xffffffffu, l[j][c], 4);
        l[j][c] += __shfl_xor_sync(0xffffffffu, l[j][c], 8);
        l[j][c] += __shfl_xor_sync(0xffffffffu, l[j][c], 16);
      }
  }

  // Columns as records of kRec floats: {m, l, -, -, O[0..D)} at row 8j + n.
  // Call reduce_l first.
  static constexpr int kRec = D + 4;
  __device__ __forceinline__ void store(float* area, int lane) const {
    const int g = lane >> 2, cq = 2 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float* r0 = area + (8 * j + cq) * kRec;
      float* r1 = r0 + kRec;
      if (g == 0) {
        r0[0] = m[j][0];
        r0[1] = l[j][0];
        r1[0] = m[j][1];
        r1[1] = l[j][1];
      }
#pragma unroll
      for (int c = 0; c < kKK; ++c) {
        if constexpr (P8) {
          *reinterpret_cast<float2*>(r0 + 4 + 16 * c + 2 * g) = make_float2(o[j][c][0], o[j][c][2]);
          *reinterpret_cast<float2*>(r1 + 4 + 16 * c + 2 * g) = make_float2(o[j][c][1], o[j][c][3]);
        } else {
          r0[4 + 16 * c + g] = o[j][c][0];
          r1[4 + 16 * c + g] = o[j][c][1];
          r0[4 + 16 * c + 8 + g] = o[j][c][2];
          r1[4 + 16 * c + 8 + g] = o[j][c][3];
        }
      }
    }
  }

  // Final output of a piece that is a whole segment, times out_scale.  Call
  // reduce_l first.
  template <typename TO>
  __device__ __forceinline__ void store_out(TO* ob, int64_t o_s1, int h0, int group, int hn, int lane,
                                            float out_scale) const {
    const int g = lane >> 2, cq = 2 * (lane & 3);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float i0 = out_scale / l[j][0], i1 = out_scale / l[j][1];
      if constexpr (P8) {
        // Lane: dims 16c + 2g, +1 of columns cq and cq + 1.
        const int e0 = row_head<PK>(8 * j + cq, group, hn), e1 = row_head<PK>(8 * j + cq + 1, group, hn);
#pragma unroll
        for (int c = 0; c < kKK; ++c) {
          if (e0 >= 0)
            *reinterpret_cast<uint32_t*>(ob + (int64_t)(h0 + e0) * o_s1 + 16 * c + 2 * g) =
                MmaOp<TO>::pack(o[j][c][0] * i0, o[j][c][2] * i0);
          if (e1 >= 0)
            *reinterpret_cast<uint32_t*>(ob + (int64_t)(h0 + e1) * o_s1 + 16 * c + 2 * g) =
                MmaOp<TO>::pack(o[j][c][1] * i1, o[j][c][3] * i1);
        }
      } else {
        // Lane: dims 16c + g and 16c + 8 + g of columns cq, cq + 1; one
        // movmatrix per 8x8 block gives it dims 16c (+8) + cq, +1 of column g.
        const int e = row_head<PK>(8 * j + g, group, hn);
        TO* dst = ob + (int64_t)(h0 + (e < 0 ? 0 : e)) * o_s1 + cq;
#pragma unroll
        for (int c = 0; c < kKK; ++c) {
          const uint32_t lo = movmatrix_t(MmaOp<TO>::pack(o[j][c][0] * i0, o[j][c][1] * i1));
          const uint32_t hi = movmatrix_t(MmaOp<TO>::pack(o[j][c][2] * i0, o[j][c][3] * i1));
          if (e >= 0) {
            *reinterpret_cast<uint32_t*>(dst + 16 * c) = lo;
            *reinterpret_cast<uint32_t*>(dst + 16 * c + 8) = hi;
          }
        }
      }
    }
  }
};

// Eight outputs of one row as a single 16-byte store.
template <typename T>
__device__ __forceinline__ int4 pack8(const float* v, float scale) {
  int4 pk;
  pk.x = static_cast<int>(MmaOp<T>::pack(v[0] * scale, v[1] * scale));
  pk.y = static_cast<int>(MmaOp<T>::pack(v[2] * scale, v[3] * scale));
  pk.z = static_cast<int>(MmaOp<T>::pack(v[4] * scale, v[5] * scale));
  pk.w = static_cast<int>(MmaOp<T>::pack(v[6] * scale, v[7] * scale));
  return pk;
}
template <typename T>
__device__ __forceinline__ void store8(T* dst, const float* v, float scale) {
  *reinterpret_cast<int4*>(dst) = pack8<T>(v, scale);
}

// Lines of the peer exchange: 8 data bytes and the call number twice per
// 16-byte store, so a line read back with both numbers equal to the call's
// has arrived whole (each 8-byte half lands atomically).
__device__ __forceinline__ void st_line(void* ptr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_line(const void* ptr) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr)
               : "memory");
  return v;
}

// acc[0..8) += wt * (v0, v1).
__device__ __forceinline__ void axpy8(float wt, float4 v0, float4 v1, float* acc) {
  acc[0] = fmaf(wt, v0.x, acc[0]);
  acc[1] = fmaf(wt, v0.y, acc[1]);
  acc[2] = fmaf(wt, v0.z, acc[2]);
  acc[3] = fmaf(wt, v0.w, acc[3]);
  acc[4] = fmaf(wt, v1.x, acc[4]);
  acc[5] = fmaf(wt, v1.y, acc[5]);
  acc[6] = fmaf(wt, v1.z, acc[6]);
  acc[7] = fmaf(wt, v1.w, acc[7]);
}

// ===========================================================================
// Balanced decode.  The sub-blocks of the batch, ordered by (sequence b,
// segment x, position), form one index space of `total` sub-blocks, where a
// segment is one KV-head pack (PK = 2: two KV heads; PK = 1: one KV head and
// a tile of <= 16 of its query heads) of one sequence.  CTA c owns
// [c*total/G, (c+1)*total/G); warp w of a CTA owns the w-th of NW equal parts
// of it.
// ===========================================================================
constexpr int kFlatMaxBatch = 1024;
constexpr int kDecodeFlags = PA_DECODE_EARLY_INPUTS | PA_DECODE_EARLY_QUERY;  // accepted flag bits

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
  int grid;     // CTAs of the main kernel
  int early;    // PA_DECODE_EARLY_INPUTS: read metadata and pools before the PDL wait
  int early_q;  // PA_DECODE_EARLY_QUERY (with early): load the first query rows before it too
  float out_scale;  // output factor: 1, or the V scale of an FP8 pool
  float k_scale, v_scale;  // FP8 pools: the fused write stores x / scale
  float* part;  // [grid][2][16][D + 4] records of segments shared with other CTAs
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
  // Head all-gather fused into the combine (xworld 0: none): `out` points at
  // this rank's first head inside the [B, xworld * Hq, D] output of all
  // ranks; rank q's heads start Hq * (q - xrank) heads away.  xareas are the
  // ranks' exchange areas (pa_head_allgather's layout), this rank's at xrank.
  uint8_t* xareas[PA_PEER_MAX_RANKS];
  int xrank, xworld;
  int64_t xline_bytes;  // bytes of lines per rank and slot: B * SPS * 16 * (D / 8) * 32
  uint64_t xlimit_ns;
};

// A segment's place in the index space.
struct Seg {
  int b, segx;
  int64_t start, end;
};

// The segment holding sub-block x (pre = per-sequence sub-block prefix sums).
__device__ __forceinline__ Seg seg_at(const int* pre, int B, int SPS, int64_t x) {
  int lo = 0, hi = B - 1;  // largest b with pre[b] * SPS <= x
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if ((int64_t)pre[mid] * SPS <= x) lo = mid; else hi = mid - 1;
  }
  Seg s;
  s.b = lo;
  const int64_t base = (int64_t)pre[lo] * SPS;
  const int nsub = pre[lo + 1] - pre[lo];
  s.segx = static_cast<int>((x - base) / nsub);
  s.start = base + (int64_t)s.segx * nsub;
  s.end = s.start + nsub;
  return s;
}

__device__ __forceinline__ Seg seg_by_id(const int* pre, int SPS, int sid) {
  Seg s;
  s.b = sid / SPS;
  s.segx = sid - s.b * SPS;
  const int nsub = pre[s.b + 1] - pre[s.b];
  s.start = (int64_t)pre[s.b] * SPS + (int64_t)s.segx * nsub;
  s.end = s.start + nsub;
  return s;
}

// First KV head, first query head and head count (PK = 1) of a segment.
template <int PK>
__device__ __forceinline__ void seg_heads(const FlatParams& p, int segx, int& kvh0, int& h0, int& hn) {
  if (PK == 2) {
    kvh0 = 2 * segx;
    h0 = kvh0 * p.group;
    hn = 2 * p.group;
  } else {
    const int kvh = segx / p.HT, ht = segx - kvh * p.HT;
    kvh0 = kvh;
    h0 = kvh * p.group + ht * 16;
    hn = min(16, p.group - ht * 16);
  }
}

// KV8: FP8 pools.  A ring stage then holds e4m3 tiles (16 tokens x 64
// bytes, 1 KB, 64-byte swizzle) that the MMA fragments are loaded from.
template <int D, int PK, int NW, int STAGES, int NSUB = 1, bool KV8 = false>
struct FlatCfg {
  static constexpr int kColTiles = D / 64;
  static constexpr int kTile8 = kSub * 64;  // one FP8 tile: 16 tokens x 64 bytes
  static constexpr int kStageBytes = 2 * kColTiles * PK * (KV8 ? kTile8 : kTileBytes);  // K + V of a sub-block
  static constexpr int kRingBytes = NW * STAGES * kStageBytes;
  static constexpr int kRec = D + 4;  // record floats per row
  static constexpr int kRecBytes = 16 * kRec * 4;
  static constexpr int kStagingBytes = NW * kRecBytes;  // first-piece record per warp
  static constexpr int kPrefixBytes = (kFlatMaxBatch + 1) * 4;
  static constexpr int kOffStaging = kRingBytes;
  static constexpr int kOffPrefix = kOffStaging + kStagingBytes;
  static constexpr int kOffBars = kOffPrefix + ((kPrefixBytes + 15) & ~15);
  static constexpr size_t kSmem = 1024 + kOffBars + NW * STAGES * 8 + 64;
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  static_assert(STAGES * kStageBytes >= kRecBytes, "a warp's ring holds its last-piece record at the end");
  __device__ __forceinline__ static int rec_area(int warp) { return warp * STAGES * kStageBytes; }
};

// TQ: query / output elements.  KV8: FP8 pools, f16 MMAs on fragments
// converted from the e4m3 tiles in registers (T is the MMA element type).
template <typename TQ, int D, int PK, int NW, int STAGES, int NSUB, int CTAS, bool KV8>
__global__ void __launch_bounds__(NW * 32, CTAS) decode_flat_kernel(const __grid_constant__ CUtensorMap tmap_k,
                                                                   const __grid_constant__ CUtensorMap tmap_v,
                                                                   FlatParams p) {
  using T = typename std::conditional<KV8, __half, TQ>::type;
  using C = FlatCfg<D, PK, NW, STAGES, NSUB, KV8>;
  using WS = WarpState<T, D, PK, KV8>;
  constexpr int kTileX = KV8 ? C::kTile8 : kTileBytes;  // bytes of one staged tile
  static_assert(STAGES >= NSUB, "a consume step takes NSUB staged sub-blocks");
  constexpr int NT = NW * 32;
  constexpr int kRec = C::kRec;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* staging = reinterpret_cast<float*>(smem + C::kOffStaging);
  int* pre = reinterpret_cast<int*>(smem + C::kOffPrefix);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
  __shared__ int warp_sums[NW];
  __shared__ int ent_seg[2 * NW];  // segment id of warp w's cut first (2w) / last (2w+1) piece, or -1
  __shared__ int run_sid[2 * NW], run_nrec[2 * NW], run_rec[2 * NW][2 * NW];  // records: float offsets into smem
  __shared__ int nruns_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
#if PA_DECODE_KV_EVICT_FIRST
  // The pools are streamed once per call: their lines leave L2 first, so
  // the stream does not evict the queries, metadata, records and code that
  // this layer's tail and the next layer read again.
  const uint64_t kv_policy = l2_evict_first_policy();
#endif
  uint8_t* ring = smem + warp * STAGES * C::kStageBytes;
  uint64_t* wbar = bars + warp * STAGES;
  // Shared-memory set-up needs no global data: it overlaps the previous
  // kernel under programmatic dependent launch.
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&wbar[s], 1);
    fence_barrier_init();
  }
  if (tid == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  const int64_t cap = p.bt_width * (int64_t)p.bs;
  // Wait for the previous kernel before touching global memory — or, when the
  // caller vouches that it writes none of the metadata and pools
  // (PA_DECODE_EARLY_INPUTS), only before the first read of q / new_k /
  // new_v and the first write, so the start-up (scan, block-table loads, the
  // first TMA copies) overlaps the previous kernel's tail.  With
  // PA_DECODE_EARLY_QUERY the first query rows are read before it as well.  Let the next PDL
  // kernel launch early either way (it waits for this one).
  if (!p.early) grid_dep_wait();
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
  // With fewer sub-blocks than CTAs, the first `total` CTAs take one each.
  const int G = static_cast<int>(total < (int64_t)gridDim.x ? total : (int64_t)gridDim.x);
  const int c = blockIdx.x;
  if (c >= G) {  // whole CTA, before any further barrier
    if (p.early) grid_dep_wait();
    return;
  }
  const int64_t clo = (int64_t)c * total / G, chi = (int64_t)(c + 1) * total / G;
  const int64_t lo = clo + (chi - clo) * warp / NW, hi = clo + (chi - clo) * (warp + 1) / NW;
  const int nj = static_cast<int>(hi - lo);  // this warp's sub-blocks

  // Lane i caches the TMA row coordinate and first KV head of sub-block
  // tb + i of the slice, so a TMA issue never waits on a block-table load.
  int tb = -32, my_y = 0, my_kv = 0;
  auto refill = [&](int j) {  // warp-uniform
    tb = j & ~31;
    const int jj = tb + lane;
    if (jj < nj) {
      const int64_t xx = lo + jj;
      const Seg s = seg_at(pre, p.B, p.SPS, xx);
      const int tok0 = static_cast<int>(xx - s.start) * kSub;
      const int64_t pb = p.bt[(int64_t)s.b * p.bt_stride + tok0 / p.bs];
      my_y = static_cast<int>(pb * p.bs + tok0 % p.bs);
      int kvh0, h0, hn;
      seg_heads<PK>(p, s.segx, kvh0, h0, hn);
      my_kv = kvh0;
    }
  };
  auto issue = [&](int j) {  // warp-uniform call, lane 0 issues
    if (j >= tb + 32) refill(j);
    const int y = __shfl_sync(0xffffffffu, my_y, j & 31);
    const int kv = __shfl_sync(0xffffffffu, my_kv, j & 31);
    if (lane == 0) {
      const int stage = j % STAGES;
      uint8_t* st = ring + stage * C::kStageBytes;
      mbar_arrive_expect_tx(&wbar[stage], C::kStageBytes);
#pragma unroll
      for (int ct = 0; ct < C::kColTiles; ++ct)
#pragma unroll
        for (int h = 0; h < PK; ++h) {
#if PA_DECODE_KV_EVICT_FIRST
          tma_load_3d_hint(st + (ct * PK + h) * kTileX, &tmap_k, &wbar[stage], ct * 64, kv + h, y, kv_policy);
          tma_load_3d_hint(st + ((C::kColTiles + ct) * PK + h) * kTileX, &tmap_v, &wbar[stage], ct * 64, kv + h, y,
                           kv_policy);
#else
          tma_load_3d(st + (ct * PK + h) * kTileX, &tmap_k, &wbar[stage], ct * 64, kv + h, y);
          tma_load_3d(st + ((C::kColTiles + ct) * PK + h) * kTileX, &tmap_v, &wbar[stage], ct * 64, kv + h, y);
#endif
        }
    }
  };
  int issued = 0;
  for (; issued < STAGES && issued < nj; ++issued) issue(issued);
  const TQ* qbase = reinterpret_cast<const TQ*>(p.q);
  WS ws;
  Seg pc{};
  if (nj > 0) pc = seg_at(pre, p.B, p.SPS, lo);
  if (p.early_q && nj > 0) {
    // The caller vouches that q is complete at launch: the first piece's
    // query fragments load now, and the first MMAs need nothing from after
    // the wait.
    int kvh0, h0, hn;
    seg_heads<PK>(p, pc.segx, kvh0, h0, hn);
    WS::template load_q<TQ>(ws.qa, qbase + (int64_t)pc.b * p.q_s0, p.q_s1, h0, p.group, hn, lane);
  }
#if PA_DECODE_Q_PREFETCH
  if (p.early && !p.early_q && nj > 0) {
    // The first piece's query rows go to L2 while the previous kernel
    // finishes, so their load after the wait hits L2 instead of queueing in
    // HBM behind every CTA's first ring copies.
    int kvh0, h0, hn;
    seg_heads<PK>(p, pc.segx, kvh0, h0, hn);
    constexpr int kLines = (D * (int)sizeof(TQ) + 127) / 128;
    const TQ* qrow = qbase + (int64_t)pc.b * p.q_s0;
    for (int i = lane; i < hn * kLines; i += 32)
      prefetch_l2(qrow + (int64_t)(h0 + i / kLines) * p.q_s1 + (i % kLines) * (128 / (int)sizeof(TQ)));
  }
#endif
  if (p.early) grid_dep_wait();

  TQ* out = reinterpret_cast<TQ*>(p.out);
  int jc = 0;  // sub-blocks of this slice consumed so far
  bool ok = true;
  int first_sid = -1, last_sid = -1;
  if (!p.early_q && nj > 0) {
    int kvh0, h0, hn;
    seg_heads<PK>(p, pc.segx, kvh0, h0, hn);
    WS::template load_q<TQ>(ws.qa, qbase + (int64_t)pc.b * p.q_s0, p.q_s1, h0, p.group, hn, lane);
  }
  int64_t x = lo;
  while (x < hi) {
    const int b = pc.b, segx = pc.segx;
    int kvh0, h0, hn;
    seg_heads<PK>(p, segx, kvh0, h0, hn);
    const int64_t pend = min(pc.end, hi);
    const bool whole = pc.start >= lo && pc.end <= hi;
    int64_t ctx = p.context_lens[b];
    ctx = ctx > cap ? cap : ctx;
    // The next piece's Q fragments load while this piece streams.
    Seg nc = pc;
    uint32_t qn[WS::kKK][4];
    if (pend < hi) {
      nc = seg_at(pre, p.B, p.SPS, pend);
      int kvn, h0n, hnn;
      seg_heads<PK>(p, nc.segx, kvn, h0n, hnn);
      WS::template load_q<TQ>(qn, qbase + (int64_t)nc.b * p.q_s0, p.q_s1, h0n, p.group, hnn, lane);
    }
    ws.reset();
    const int jend = static_cast<int>(pend - lo);
    while (jc < jend) {
      const int n = (jend - jc >= NSUB) ? NSUB : 1;
      uint32_t stg[NSUB];
      int valid[NSUB];
#pragma unroll
      for (int u = 0; u < NSUB; ++u) {
        if (u < n) {
          const int j = jc + u;
          const int stage = j % STAGES;
          if (ok) ok = mbar_wait(&wbar[stage], (j / STAGES) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
          uint8_t* tiles = ring + stage * C::kStageBytes;
          stg[u] = smem_u32(tiles);
          const int64_t sub = lo + j - pc.start;
          valid[u] = static_cast<int>(min((int64_t)kSub, ctx - sub * kSub));
          if (p.new_k != nullptr && (sub + 1) * kSub >= ctx) {
            // Fused KV write: the sub-block holding the new token (position
            // ctx - 1) gets its K/V rows from new_k / new_v in place of the
            // pool's, and they are stored to the pools (by the head-tile-0
            // segment when PK = 1).  One 16-byte chunk per lane and step:
            // (K/V, column tile, head of the pack, chunk of the 128-byte row).
            const int r = static_cast<int>(ctx - 1 - sub * kSub);
            constexpr int kChunks = 2 * C::kColTiles * PK * 8;
            const bool store_pool = PK == 2 || segx % p.HT == 0;
            const int64_t slot = p.slots[b];
            for (int i = lane; i < kChunks; i += 32) {
              const int cc = i & 7, t = i >> 3;  // t = (kv * kColTiles + ct) * PK + h
              const int h = t % PK, kvct = t / PK;
              const int kv = kvct / C::kColTiles, ct = kvct - kv * C::kColTiles;
              const int64_t src = ((int64_t)b * p.Hkv + kvh0 + h) * D + ct * 64 + cc * 8;
              const int4 val =
                  __ldg(reinterpret_cast<const int4*>(reinterpret_cast<const TQ*>(kv ? p.new_v : p.new_k) + src));
              const int64_t pool_el = (slot * p.Hkv + kvh0 + h) * D + ct * 64 + cc * 8;
              if (KV8) {
                // Quantize as the FP8 scatter does (x / scale, saturated,
                // nearest even); the 8 bytes go to the staged tile (half of
                // a swizzled 16-byte chunk) and to the pools.
                const TQ* e = reinterpret_cast<const TQ*>(&val);
                const float sc = kv ? p.v_scale : p.k_scale;
                uint32_t f8[2] = {0u, 0u};
#pragma unroll
                for (int k2 = 0; k2 < 8; ++k2) {
                  const uint32_t b8 =
                      __nv_cvt_float_to_fp8(__fdiv_rn(Elem<TQ>::to_f32(e[k2]), sc), __NV_SATFINITE, __NV_E4M3);
                  f8[k2 >> 2] |= b8 << (8 * (k2 & 3));
                }
                *reinterpret_cast<uint2*>(tiles + t * C::kTile8 + swz64(r, cc >> 1) + (cc & 1) * 8) =
                    make_uint2(f8[0], f8[1]);
                if (store_pool && slot >= 0 && slot < p.num_slots)
                  *reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(kv ? p.v_pool : p.k_pool) + pool_el) =
                      make_uint2(f8[0], f8[1]);
              } else {
                *reinterpret_cast<int4*>(tiles + t * kTileBytes + r * 128 + ((cc ^ (r & 7)) << 4)) = val;
                if (store_pool && slot >= 0 && slot < p.num_slots)
                  *reinterpret_cast<int4*>(reinterpret_cast<TQ*>(kv ? p.v_pool : p.k_pool) + pool_el) = val;
              }
            }
            fence_proxy_async_smem();  // before the stage is refilled by TMA
            __syncwarp();
          }
        }
      }
      if (!ok) break;
      if (n == NSUB) ws.template consume<NSUB>(stg, valid, p.scale_log2, lane);
      else ws.template consume<1>(stg, valid, p.scale_log2, lane);
      __syncwarp();
      for (int u = 0; u < n; ++u)
          if (issued < nj) issue(issued++);
      jc += n;
    }
    if (!ok) break;
    ws.reduce_l();
    if (whole) {
      ws.store_out(out + (int64_t)b * p.o_s0, p.o_s1, h0, p.group, hn, lane, p.out_scale);
    } else if (x == lo) {  // cut at the slice start: park the record until the end
      ws.store(staging + warp * 16 * kRec, lane);
      first_sid = b * p.SPS + segx;
    } else {  // cut at the slice end: the last piece, kept in registers
      last_sid = b * p.SPS + segx;
    }
    x = pend;
    if (x < hi) {
      pc = nc;
#pragma unroll
      for (int kk = 0; kk < WS::kKK; ++kk)
#pragma unroll
        for (int e = 0; e < 4; ++e) ws.qa[kk][e] = qn[kk][e];
    }
  }
  if (!ok) {
    // A bounded wait gave up (status already recorded): wait, again bounded,
    // for this warp's copies still in flight so none lands after the CTA has
    // exited; the outputs are garbage and the status word says so.
    for (int j = jc; j < issued; ++j) mbar_wait(&wbar[j % STAGES], (j / STAGES) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
    first_sid = last_sid = -1;
  }
  // This warp's copies have all landed: its ring is free for the last-piece
  // record.
  if (last_sid >= 0) ws.store(reinterpret_cast<float*>(smem + C::rec_area(warp)), lane);
  if (lane == 0) {
    ent_seg[2 * warp] = first_sid;
    ent_seg[2 * warp + 1] = last_sid;
  }
  __syncthreads();

  // ---- merge the pieces cut by warp boundaries (shared memory) -----------
  // Entries in order (warp, first/last) form runs of equal segments.  A run
  // whose segment lies inside this CTA's range is merged to the output;
  // otherwise to this CTA's record of the segment in global memory — slot 0
  // when the segment starts before the range, else slot 1 — which
  // decode_combine_kernel merges with the other CTAs' records.
  if (tid == 0) {
    int n = 0, prev = -1;
    for (int f = 0; f < 2 * NW; ++f) {
      const int sid = ent_seg[f];
      if (sid < 0) continue;
      if (sid != prev) {
        run_sid[n] = sid;
        run_nrec[n] = 0;
        ++n;
        prev = sid;
      }
      // Entry f's record: the warp's record area (last piece) or its staging slot.
      run_rec[n - 1][run_nrec[n - 1]++] =
          (f & 1) ? C::rec_area(f >> 1) / 4 : (C::kOffStaging + (f >> 1) * C::kRecBytes) / 4;
    }
    nruns_s = n;
  }
  __syncthreads();
  const float* smem_f = reinterpret_cast<const float*>(smem);
  constexpr int kItems = 16 * (D / 8);  // (row, 8 columns)
  const int nruns = nruns_s;
  for (int w = tid; w < nruns * kItems; w += NT) {
    const int ri = w / kItems, it = w - ri * kItems;
    const int sid = run_sid[ri], nrec = run_nrec[ri];
    const int r = it / (D / 8), d = 8 * (it - r * (D / 8));
    const Seg S = seg_by_id(pre, p.SPS, sid);
    int kvh0, h0, hn;
    seg_heads<PK>(p, S.segx, kvh0, h0, hn);
    const int hh = row_head<PK>(r, p.group, hn);
    if (hh < 0) continue;
    // Two passes (the maximum, then independent weighted sums) keep the
    // records' contributions free of a serial rescale chain.
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 2 * NW; ++k)
      if (k < nrec) mx = fmaxf(mx, smem_f[run_rec[ri][k] + r * kRec]);
    float l = 0.f;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 2 * NW; ++k) {
      if (k >= nrec) break;
      const float* rec = smem_f + run_rec[ri][k] + r * kRec;
      const float wt = exp2f(rec[0] - mx);
      l = fmaf(wt, rec[1], l);
      axpy8(wt, *reinterpret_cast<const float4*>(rec + 4 + d), *reinterpret_cast<const float4*>(rec + 8 + d), acc);
    }
    if (S.start >= clo && S.end <= chi) {
      store8<TQ>(out + (int64_t)S.b * p.o_s0 + (int64_t)(h0 + hh) * p.o_s1 + d, acc, p.out_scale / l);
    } else {
      float* row = p.part + (((int64_t)c * 2 + (S.start < clo ? 0 : 1)) * 16 + r) * kRec;
      if (d == 0) *reinterpret_cast<float2*>(row) = make_float2(mx, l);
      *reinterpret_cast<float4*>(row + 4 + d) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(row + 8 + d) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// Second stage of the balanced decode: segments cut by CTA boundaries.  CTA
// (segment, slab of kCombineRows rows) merges the records that CTAs c0..c1
// of the main kernel wrote for the segment; segments that one CTA finished
// return at once.  Launched with PDL right behind the main kernel: the
// segment's bounds come from the context lengths (an input the main kernel
// does not write) before the wait, so only the record loads remain after it.
// Its CTAs are small (64 threads, at most 128 registers) so they fit beside
// the main kernel's CTAs, and each lets the next kernel launch as soon as it
// starts: that kernel's CTAs then take each SM the main kernel frees and run
// their own start-up while this merge is still pending.  A CTA covers ROWS
// rows; when segments span many CTAs (long sequences) ROWS shrinks so the
// records of one item are split over several threads (stripes).
constexpr int kCombineThreads = 64;

template <typename T, int D, int PK, int ROWS, bool XCHG = false>
__global__ void __launch_bounds__(kCombineThreads, 8) decode_combine_kernel(FlatParams p) {
  constexpr int kRec = D + 4;
  constexpr int kCombineRows = ROWS;
  constexpr int kItems = kCombineRows * (D / 8);  // (row, 8 columns) per CTA
  constexpr int kStripes = kCombineThreads / kItems;
  static_assert(kStripes >= 1 && kCombineThreads % kItems == 0, "combine layout");
  __shared__ float sm_m[kCombineThreads], sm_l[kCombineThreads];
  __shared__ float4 sm_acc[kCombineThreads][2];
  __shared__ int wsum[2][kCombineThreads / 32];
  __shared__ uint32_t call_s;
  const int tid = threadIdx.x;
  const int sid = blockIdx.x;
  const int b = sid / p.SPS, segx = sid - b * p.SPS;
  const int64_t cap = p.bt_width * (int64_t)p.bs;
  grid_dep_launch();
  int before = 0, all = 0;
  for (int i = tid; i < p.B; i += kCombineThreads) {
    int64_t ctx = p.context_lens[i];
    ctx = ctx > cap ? cap : ctx;
    const int cnt = ctx > 0 ? static_cast<int>((ctx + kSub - 1) / kSub) : 0;
    all += cnt;
    before += i < b ? cnt : 0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    before += __shfl_xor_sync(0xffffffffu, before, o);
    all += __shfl_xor_sync(0xffffffffu, all, o);
  }
  if ((tid & 31) == 0) {
    wsum[0][tid >> 5] = before;
    wsum[1][tid >> 5] = all;
  }
  __syncthreads();
  before = all = 0;
#pragma unroll
  for (int w = 0; w < kCombineThreads / 32; ++w) {
    before += wsum[0][w];
    all += wsum[1][w];
  }
  int64_t ctx = p.context_lens[b];
  ctx = ctx > cap ? cap : ctx;
  const int nsub = ctx > 0 ? static_cast<int>((ctx + kSub - 1) / kSub) : 0;
  // With the exchange every CTA takes part to the end (its rows go to the
  // peers, and it counts in for the call number); otherwise a CTA without
  // rows to merge returns at once.
  if (!XCHG && nsub == 0) return;
  const int64_t total = (int64_t)all * p.SPS;
  const int G = static_cast<int>(total < (int64_t)p.grid ? total : (int64_t)p.grid);
  const int64_t start = (int64_t)before * p.SPS + (int64_t)segx * nsub, end = start + nsub;
  auto cta_of = [&](int64_t xx) { return static_cast<int>(((xx + 1) * G - 1) / total); };
  const int c0 = nsub > 0 ? cta_of(start) : 0, c1 = nsub > 0 ? cta_of(end - 1) : 0;
  const bool merged_here = nsub > 0 && c0 != c1;  // else the main kernel finished it inside one CTA
  if (!XCHG && !merged_here) return;
  int kvh0, h0, hn;
  seg_heads<PK>(p, segx, kvh0, h0, hn);
  const int item = tid % kItems, stripe = tid / kItems;
  const int r = blockIdx.y * kCombineRows + item / (D / 8), d = 8 * (item % (D / 8));
  const int hh = row_head<PK>(r, p.group, hn);
  grid_dep_wait();  // the main kernel's records (and outputs) are complete and visible
  if constexpr (XCHG) {
    if (tid == 0) call_s = next_call_number(*reinterpret_cast<volatile uint32_t*>(p.xareas[p.xrank] + 132));
  }
  float mrun = -INFINITY, lrun = 0.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (merged_here && hh >= 0) {
    for (int cb = c0 + stripe; cb <= c1; cb += 8 * kStripes) {  // eight records' loads in flight
      float2 ml[8];
      float4 v0[8], v1[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int cc = cb + u * kStripes;
        ml[u] = make_float2(-INFINITY, 0.f);
        v0[u] = v1[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (cc <= c1) {
          // The segment starts inside CTA c0's range (slot 1 there) and
          // before the range of every later CTA (slot 0).
          const int sl = cc == c0 ? 1 : 0;
          const float* rec = p.part + (((int64_t)cc * 2 + sl) * 16 + r) * kRec;
          ml[u] = __ldcg(reinterpret_cast<const float2*>(rec));
          v0[u] = __ldcg(reinterpret_cast<const float4*>(rec + 4 + d));
          v1[u] = __ldcg(reinterpret_cast<const float4*>(rec + 8 + d));
        }
      }
      float mx = mrun;
#pragma unroll
      for (int u = 0; u < 8; ++u) mx = fmaxf(mx, ml[u].x);
      if (mx == -INFINITY) continue;
      const float a = exp2f(mrun - mx);  // 0 on the first batch
      lrun *= a;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= a;
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float wt = exp2f(ml[u].x - mx);  // 0 for absent records
        lrun = fmaf(wt, ml[u].y, lrun);
        axpy8(wt, v0[u], v1[u], acc);
      }
      mrun = mx;
    }
  }
  if (kStripes > 1) {
    sm_m[tid] = mrun;
    sm_l[tid] = lrun;
    sm_acc[tid][0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    sm_acc[tid][1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    __syncthreads();
    if (!XCHG && (stripe != 0 || hh < 0)) return;
    if (stripe == 0 && hh >= 0) {
      float mx = -INFINITY;
#pragma unroll
      for (int s2 = 0; s2 < kStripes; ++s2) mx = fmaxf(mx, sm_m[s2 * kItems + item]);
      lrun = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < kStripes; ++s2) {
        const int t2 = s2 * kItems + item;
        const float wt = exp2f(sm_m[t2] - mx);
        lrun = fmaf(wt, sm_l[t2], lrun);
        axpy8(wt, sm_acc[t2][0], sm_acc[t2][1], acc);
      }
    }
  }
  if (!XCHG && hh < 0) return;
  T* out = reinterpret_cast<T*>(p.out);
  T* dst = out + (int64_t)b * p.o_s0 + (int64_t)(h0 + hh) * p.o_s1 + d;
  if constexpr (!XCHG) {
    store8<T>(dst, acc, p.out_scale / lrun);
  } else {
    // This thread owns output (row r, columns d..d+7) of this rank's heads.
    const bool own = nsub > 0 && hh >= 0 && stripe == 0;
    int4 fin = make_int4(0, 0, 0, 0);
    if (own) {
      if (merged_here) {
        fin = pack8<T>(acc, p.out_scale / lrun);
        *reinterpret_cast<int4*>(dst) = fin;
      } else {
        fin = *reinterpret_cast<const int4*>(dst);  // written by the main kernel
      }
    }
    __syncthreads();  // call_s
    const uint32_t n = call_s;
    const int64_t slot_off = 256 + (int64_t)(n & 1u) * p.xworld * p.xline_bytes;
    const int64_t line = (((int64_t)sid * 16 + r) * (D / 8) + d / 8) * 32;
    if (own) {
      for (int q = 0; q < p.xworld; ++q) {
        if (q == p.xrank) continue;
        uint8_t* l = p.xareas[q] + slot_off + p.xrank * p.xline_bytes + line;
        st_line(l, (uint32_t)fin.x, n, (uint32_t)fin.y, n);
        st_line(l + 16, (uint32_t)fin.z, n, (uint32_t)fin.w, n);
      }
    }
    __syncthreads();
    uint8_t* mine = p.xareas[p.xrank];
    uint32_t* arrivals = reinterpret_cast<uint32_t*>(mine + 128);
    if (tid == 0 && atomicAdd(arrivals, 1u) == gridDim.x * gridDim.y - 1) {
      *reinterpret_cast<volatile uint32_t*>(arrivals) = 0u;
      *reinterpret_cast<volatile uint32_t*>(mine + 132) = n;
    }
    if (own) {
      // The peers' rows of the same (segment, row, columns), polled (bounded).
      const uint64_t t0 = globaltimer_ns();
      for (int q = 0; q < p.xworld; ++q) {
        if (q == p.xrank) continue;
        const uint8_t* l = mine + slot_off + q * p.xline_bytes + line;
        uint4 a, c;
        bool got = true;
        for (uint32_t i = 0;; ++i) {
          a = ld_line(l);
          c = ld_line(l + 16);
          if (a.y == n && a.w == n && c.y == n && c.w == n) break;
          if ((i & 63) == 63 && globaltimer_ns() - t0 > p.xlimit_ns) {
            record_status(reinterpret_cast<int*>(mine + 136), PA_DEVICE_TIMEOUT_PEER);
            record_status(p.status, PA_DEVICE_TIMEOUT_PEER);
            got = false;
            break;
          }
        }
        if (!got) break;
        *reinterpret_cast<int4*>(dst + (int64_t)(q - p.xrank) * p.Hq * p.o_s1) =
            make_int4((int)a.x, (int)a.z, (int)c.x, (int)c.z);
      }
    }
  }
}

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
#if PA_DECODE_KV_EVICT_FIRST
  const uint64_t kv_policy = l2_evict_first_policy();  // pools streamed once
#endif
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
#if PA_DECODE_KV_EVICT_FIRST
      tma_load_3d_hint(st + ct * kTileBytes, &tmap_k, &wbar[stage], ct * 64, kvh, y, kv_policy);
      tma_load_3d_hint(st + (C::kColTiles + ct) * kTileBytes, &tmap_v, &wbar[stage], ct * 64, kvh, y, kv_policy);
#else
      tma_load_3d(st + ct * kTileBytes, &tmap_k, &wbar[stage], ct * 64, kvh, y);
      tma_load_3d(st + (C::kColTiles + ct) * kTileBytes, &tmap_v, &wbar[stage], ct * 64, kvh, y);
#endif
    }
  };
  if (lane == 0) {
    for (int j = 0; j < STAGES && j < nj; ++j) issue(j);
  }
  using WS = WarpState<T, D, 1>;
  WS ws;
  ws.reset();
  WS::load_q(ws.qa, reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_s0, p.q_s1, h0, p.group, hn, lane);
  bool ok = true;
  for (int j = 0; j < nj; ++j) {
    const int stage = j % STAGES;
    if (ok) ok = mbar_wait(&wbar[stage], (j / STAGES) & 1, p.status, PA_DEVICE_TIMEOUT_TMA);
    const uint32_t kbase = smem_u32(ring + stage * C::kStageBytes);
    const int valid = static_cast<int>(min((int64_t)kSub, ctx - (int64_t)(s0 + warp + j * NW) * kSub));
    ws.template consume<1>(&kbase, &valid, p.scale_log2, lane);
    __syncwarp();
    if (lane == 0 && j + STAGES < nj) issue(j + STAGES);
  }
  ws.reduce_l();
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

// Shapes of the balanced kernel: warps per CTA, ring stages per warp and
// sub-blocks per consume step, per (head_dim, KV heads per warp).  Two CTAs
// per SM (~87 KB of shared memory each at D = 64), so one CTA's start-up and
// merge tail overlap the other's streaming and, with PDL, the next kernel's
// CTAs move in as soon as one exits.  A stage is one sub-block of every head
// of the pack: 8 KB (D = 64, PK = 2) to 16 KB (D = 128, PK = 2).
// FP8 pools halve a stage: at D = 64 they take one more ring stage, at
// D = 128 twice the warps (8 per SM), since an FP8 byte costs twice the MMA
// and conversion work of a BF16 byte and one warp per scheduler cannot hide
// that latency.
template <int D, int PK, bool KV8 = false> struct FlatShape;
template <> struct FlatShape<64, 2> { static constexpr int NW = 4, ST = 2, NSUB = 1; };
template <> struct FlatShape<64, 1> { static constexpr int NW = 4, ST = 4, NSUB = 2; };
template <> struct FlatShape<128, 2> { static constexpr int NW = 2, ST = 2, NSUB = 1; };
template <> struct FlatShape<128, 1> { static constexpr int NW = 2, ST = 4, NSUB = 2; };
template <> struct FlatShape<64, 2, true> { static constexpr int NW = 4, ST = 3, NSUB = 1; };
template <> struct FlatShape<64, 1, true> { static constexpr int NW = 4, ST = 4, NSUB = 2; };
template <> struct FlatShape<128, 2, true> { static constexpr int NW = 4, ST = 2, NSUB = 1; };
template <> struct FlatShape<128, 1, true> { static constexpr int NW = 4, ST = 4, NSUB = 2; };
constexpr int kFlatCtasPerSm = 2;
constexpr int kSplitNW = 4, kSplitST = 4;

// Two KV heads per warp when a GQA group fits half the MMA rows.
bool flat_pack2(int hq, int hkv) { return hkv % 2 == 0 && hq / hkv <= 8; }

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

// Every CTA of an exchanging combine polls for its peers' rows, so all of its
// CTAs must be resident at once: true when the grid fits the device's
// occupancy for the kernel.
template <typename K>
bool fits_resident(K kern, int64_t ctas) {
  static int per_sm[64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return false;
  if (per_sm[dev] == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kCombineThreads, 0) != cudaSuccess || n <= 0)
      return false;
    per_sm[dev] = n;
  }
  return ctas <= (int64_t)per_sm[dev] * num_sms(dev);
}

template <typename T, int D, int PK, bool KV8>
int launch_flat(const FlatParams& p, const CUtensorMap& tk, const CUtensorMap& tv, int grid, cudaStream_t st) {
  using S = FlatShape<D, PK, KV8>;
  using C = FlatCfg<D, PK, S::NW, S::ST, S::NSUB, KV8>;
  auto kern = decode_flat_kernel<T, D, PK, S::NW, S::ST, S::NSUB, kFlatCtasPerSm, KV8>;
  // One item per thread (ROWS = 512 / D) unless segments span more than eight
  // CTAs on average; then one row per CTA and the records go over stripes.
  constexpr int kRowsWide = kCombineThreads * 8 / D;
  const bool wide = (int64_t)grid <= 8 * (int64_t)p.B * p.SPS;
  const dim3 cgrid(p.B * p.SPS, wide ? 16 / kRowsWide : 16);
  if (p.xworld > 1) {
    const int64_t ctas = (int64_t)cgrid.x * cgrid.y;
    const bool ok = wide ? fits_resident(decode_combine_kernel<T, D, PK, kRowsWide, true>, ctas)
                         : fits_resident(decode_combine_kernel<T, D, PK, 1, true>, ctas);
    if (!ok) return PA_ERR_UNSUPPORTED;  // checked before anything is launched
  }
  static bool done[64] = {};
  if (!set_smem_attr(kern, C::kSmem, done)) return PA_ERR_CUDA;
  const int r = launch_pdl(kern, dim3(grid), dim3(S::NW * 32), C::kSmem, st, tk, tv, p);
  if (r != PA_OK) return r;
  if (p.xworld > 1)
    return wide ? launch_pdl(decode_combine_kernel<T, D, PK, kRowsWide, true>, cgrid, dim3(kCombineThreads), 0, st, p)
                : launch_pdl(decode_combine_kernel<T, D, PK, 1, true>, cgrid, dim3(kCombineThreads), 0, st, p);
  if (!wide) return launch_pdl(decode_combine_kernel<T, D, PK, 1>, cgrid, dim3(kCombineThreads), 0, st, p);
  return launch_pdl(decode_combine_kernel<T, D, PK, kRowsWide>, cgrid, dim3(kCombineThreads), 0, st, p);
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

// Which kernel a call uses and how much workspace it needs.
struct DecodePlan {
  enum Kind { kFlat, kSplit, kGeneric } kind;
  int grid;          // flat: CTAs
  int split_sub;     // split: sub-blocks per partition
  int split_tokens;  // generic: tokens per partition
  int splits;        // split / generic: partitions per sequence (max)
  size_t ws_bytes;
};

// Workspace of the balanced kernel: status word, the ticket range of the
// other decode kernels (unused here, kept so one zeroing rule serves every
// path), then two partial records of 16 rows x (D + 4) floats per CTA.
size_t flat_ws_bytes(int batch, int hq, int D, int grid) {
  return 256 + align256(sizeof(int) * (size_t)batch * hq) + align256((size_t)grid * 2 * 16 * (D + 4) * sizeof(float));
}

DecodePlan plan_decode(int batch, int hkv, int hq, int D, int bs, int64_t bt_width, int partition_tokens,
                       int dtype) {
  DecodePlan pl{};
  const int group = hq / hkv;
  const int sms = num_sms(current_device());
  const int64_t max_tok = bt_width * bs;
  if (tc_shape_ok(dtype, D, bs) && batch <= kFlatMaxBatch) {
    // Explicit partitions (partition_tokens > 0) take the balanced kernel as
    // well: its pieces are LSE-merged exactly like partitions, only cut where
    // the load balance puts them.
    pl.kind = DecodePlan::kFlat;
    pl.grid = sms * kFlatCtasPerSm;
    pl.ws_bytes = flat_ws_bytes(batch, hq, D, pl.grid);
    return pl;
  }
  if (tc_shape_ok(dtype, D, bs)) {
    pl.kind = DecodePlan::kSplit;
    const int64_t max_sub = (max_tok + kSub - 1) / kSub;
    int64_t split = partition_tokens > 0 ? (partition_tokens + kSub - 1) / kSub : max_sub;
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

// Head all-gather fused into the decode (pa_paged_decode_allgather).
struct Exchange {
  int rank, world;
  void* const* areas;
  int64_t area_bytes;
  int64_t wait_limit_ns;
};

int decode_impl(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer, const void* v_pool_layer,
                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                int64_t bt_stride, int64_t bt_width, const int64_t* context_lens, void* out, int64_t o_s0,
                int64_t o_s1, int batch, int num_q_heads, float scale, int dtype, int partition_tokens,
                void* workspace, size_t workspace_bytes, void* stream, const FusedWrite* fw, bool* fused,
                int flags = 0, int kv_dtype = -1, float k_scale = 1.f, float v_scale = 1.f,
                const Exchange* xc = nullptr);

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

extern "C" int pa_paged_decode_ex(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k, const void* new_v,
                                  const int64_t* slot_mapping, void* k_pool_layer, void* v_pool_layer,
                                  int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                                  const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                                  const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                                  int num_q_heads, float scale, int dtype, int partition_tokens, int flags,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  using namespace pa;
  if (batch < 0 || (flags & ~kDecodeFlags)) return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  const bool write = new_k != nullptr || new_v != nullptr || slot_mapping != nullptr;
  if (!write)
    return decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim,
                       block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch, num_q_heads, scale,
                       dtype, partition_tokens, workspace, workspace_bytes, stream, nullptr, nullptr, flags);
  if (new_k == nullptr || new_v == nullptr || slot_mapping == nullptr || partition_tokens != 0) return PA_ERR_INVALID;
  if (!((reinterpret_cast<uintptr_t>(new_k) | reinterpret_cast<uintptr_t>(new_v)) & 15)) {
    FusedWrite fw{new_k, new_v, slot_mapping};
    bool fused = false;
    const int r = decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads,
                              head_dim, block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch,
                              num_q_heads, scale, dtype, 0, workspace, workspace_bytes, stream, &fw, &fused, flags);
    if (r != PA_OK || fused) return r;
  }
  // Not fusable here: the scatter, then decode; the decode then reads pool
  // rows the scatter just wrote, so it waits before its first read.
  return pa_paged_decode_write(q, q_s0, q_s1, new_k, new_v, slot_mapping, k_pool_layer, v_pool_layer, num_blocks,
                               block_size, num_kv_heads, head_dim, block_tables, bt_stride, bt_width, context_lens, out,
                               o_s0, o_s1, batch, num_q_heads, scale, dtype, workspace, workspace_bytes, stream);
}

extern "C" size_t pa_decode_allgather_bytes(int batch, int num_kv_heads, int num_q_heads, int head_dim,
                                            int world) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0 || head_dim <= 0 ||
      head_dim % 8 || world < 1 || world > PA_PEER_MAX_RANKS)
    return 0;
  const int group = num_q_heads / num_kv_heads;
  const bool pk2 = pa::flat_pack2(num_q_heads, num_kv_heads);
  const int sps = pk2 ? num_kv_heads / 2 : num_kv_heads * ((group + 15) / 16);
  const int64_t lines = (int64_t)batch * sps * 16 * (head_dim / 8) * 32;
  return static_cast<size_t>(256 + 2 * (int64_t)world * lines);
}

extern "C" int pa_paged_decode_allgather(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k,
                                         const void* new_v, const int64_t* slot_mapping, void* k_pool_layer,
                                         void* v_pool_layer, int64_t num_blocks, int block_size, int num_kv_heads,
                                         int head_dim, const int64_t* block_tables, int64_t bt_stride,
                                         int64_t bt_width, const int64_t* context_lens, void* out, int64_t o_s0,
                                         int64_t o_s1, int batch, int num_q_heads, float scale, int dtype, int flags,
                                         int rank, int world, void* const* areas, int64_t area_bytes,
                                         int64_t wait_limit_ns, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  using namespace pa;
  if (batch < 0 || (flags & ~kDecodeFlags)) return PA_ERR_INVALID;
  if (world < 2 || world > PA_PEER_MAX_RANKS || rank < 0 || rank >= world || areas == nullptr) return PA_ERR_INVALID;
  if (wait_limit_ns < 0 || wait_limit_ns > 2000000000LL) return PA_ERR_INVALID;
  for (int r = 0; r < world; ++r)
    if (areas[r] == nullptr || (reinterpret_cast<uintptr_t>(areas[r]) & 255)) return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  const bool write = new_k != nullptr || new_v != nullptr || slot_mapping != nullptr;
  if (write && (new_k == nullptr || new_v == nullptr || slot_mapping == nullptr)) return PA_ERR_INVALID;
  if (write && ((reinterpret_cast<uintptr_t>(new_k) | reinterpret_cast<uintptr_t>(new_v)) & 15))
    return PA_ERR_UNSUPPORTED;
  if (dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16) return PA_ERR_UNSUPPORTED;
  const Exchange xc{rank, world, areas, area_bytes, wait_limit_ns};
  FusedWrite fw{new_k, new_v, slot_mapping};
  bool fused = false;
  const int r = decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim,
                            block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch, num_q_heads,
                            scale, dtype, 0, workspace, workspace_bytes, stream, write ? &fw : nullptr, &fused, flags,
                            -1, 1.f, 1.f, &xc);
  if (r == PA_OK && write && !fused) return PA_ERR_UNSUPPORTED;  // not reached: the exchange needs the fused kernel
  return r;
}

namespace pa {
namespace {

int decode_impl(const void* q, int64_t q_s0, int64_t q_s1, const void* k_pool_layer, const void* v_pool_layer,
                int64_t num_blocks, int block_size, int num_kv_heads, int head_dim, const int64_t* block_tables,
                int64_t bt_stride, int64_t bt_width, const int64_t* context_lens, void* out, int64_t o_s0,
                int64_t o_s1, int batch, int num_q_heads, float scale, int dtype, int partition_tokens,
                void* workspace, size_t workspace_bytes, void* stream, const FusedWrite* fw, bool* fused,
                int flags, int kv_dtype, float k_scale, float v_scale, const Exchange* xc) {
  if (batch < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks <= 0 || bt_width <= 0 || partition_tokens < 0 || (flags & ~kDecodeFlags))
    return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  if (q == nullptr || k_pool_layer == nullptr || v_pool_layer == nullptr || block_tables == nullptr ||
      context_lens == nullptr || out == nullptr)
    return PA_ERR_INVALID;
  if (dtype != PA_DTYPE_F32 && dtype != PA_DTYPE_F16 && dtype != PA_DTYPE_BF16) return PA_ERR_UNSUPPORTED;
  if (batch > 65535) return PA_ERR_INVALID;
  const bool kv8 = kv_dtype == PA_DTYPE_FP8_E4M3;
  if (kv_dtype != -1 && !kv8) return PA_ERR_UNSUPPORTED;
  if (kv8 && (!(k_scale > 0.f) || !(v_scale > 0.f) || isinf(k_scale) || isinf(v_scale))) return PA_ERR_INVALID;
  if (!kv8) k_scale = v_scale = 1.f;
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
  if (fw != nullptr && pl.kind != DecodePlan::kFlat) {
    if (fused != nullptr) *fused = false;  // only the balanced kernel fuses the write
    return PA_OK;
  }
  if (xc != nullptr && pl.kind != DecodePlan::kFlat) return PA_ERR_UNSUPPORTED;  // the exchange rides the combine
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  if (ws == nullptr || workspace_bytes < pl.ws_bytes || (reinterpret_cast<uintptr_t>(ws) & 255))
    return PA_ERR_WORKSPACE;
  int* status = reinterpret_cast<int*>(ws);

  if (pl.kind == DecodePlan::kFlat || pl.kind == DecodePlan::kSplit) {
    if (kv8 && pl.kind != DecodePlan::kFlat) return PA_ERR_UNSUPPORTED;  // batches > 1024 with FP8 pools
    CUtensorMap tk, tv;
    const uint64_t slots = static_cast<uint64_t>(num_blocks) * block_size;
    const uint64_t s1b = static_cast<uint64_t>(head_dim) * (kv8 ? 1 : 2);
    const uint64_t s2b = s1b * num_kv_heads;
    const int map_dtype = kv8 ? PA_DTYPE_FP8_E4M3 : dtype;
    // Rows of one KV head are 128 B (64 B with FP8) with a Hkv-row stride; a
    // wider L2 promotion would drag the other heads' rows in ahead of their
    // readers.  The swizzle spans one row, so the MMA fragment loads (8 rows
    // of one 16-byte column) hit distinct banks.
    const CUtensorMapSwizzle swz_mode = kv8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    const CUtensorMapL2promotion l2p = kv8 ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B : CU_TENSOR_MAP_L2_PROMOTION_L2_128B;
    if (make_map_3d(&tk, map_dtype, k_pool_layer, head_dim, num_kv_heads, slots, s1b, s2b, 64, 1, 16, swz_mode,
                    l2p) != PA_OK ||
        make_map_3d(&tv, map_dtype, v_pool_layer, head_dim, num_kv_heads, slots, s1b, s2b, 64, 1, 16, swz_mode,
                    l2p) != PA_OK)
      return PA_ERR_CUDA;
    const float scale_log2 = scale * k_scale * 1.4426950408889634f;
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
      const bool pk2 = flat_pack2(num_q_heads, num_kv_heads);
      p.HT = pk2 ? 1 : (group + 15) / 16;
      p.SPS = pk2 ? num_kv_heads / 2 : num_kv_heads * p.HT;
      p.bs = block_size;
      p.scale_log2 = scale_log2;
      p.grid = pl.grid;
      p.early = (flags & PA_DECODE_EARLY_INPUTS) ? 1 : 0;
      p.early_q = p.early && (flags & PA_DECODE_EARLY_QUERY) ? 1 : 0;
      p.out_scale = v_scale;
      p.k_scale = k_scale;
      p.v_scale = v_scale;
      p.part = reinterpret_cast<float*>(ws + 256 + align256(sizeof(int) * (size_t)batch * num_q_heads));
      p.status = status;
      p.new_k = fw ? fw->new_k : nullptr;
      p.new_v = fw ? fw->new_v : nullptr;
      p.slots = fw ? fw->slots : nullptr;
      p.k_pool = const_cast<void*>(k_pool_layer);
      p.v_pool = const_cast<void*>(v_pool_layer);
      p.num_slots = static_cast<int64_t>(num_blocks) * block_size;
      for (int i = 0; i < PA_PEER_MAX_RANKS; ++i) p.xareas[i] = nullptr;
      p.xrank = 0;
      p.xworld = 0;
      p.xline_bytes = 0;
      p.xlimit_ns = kWaitLimitNs;
      if (xc != nullptr) {
        p.xrank = xc->rank;
        p.xworld = xc->world;
        p.xline_bytes = (int64_t)batch * p.SPS * 16 * (head_dim / 8) * 32;
        if (256 + 2 * (int64_t)xc->world * p.xline_bytes > xc->area_bytes) return PA_ERR_CAPACITY;
        for (int i = 0; i < xc->world; ++i) p.xareas[i] = static_cast<uint8_t*>(xc->areas[i]);
        if (xc->wait_limit_ns > 0) p.xlimit_ns = static_cast<uint64_t>(xc->wait_limit_ns);
      }
      if (fused != nullptr) *fused = fw != nullptr;
      const int g = pl.grid;
      using B16 = __nv_bfloat16;
      if (kv8) {
        if (dtype == PA_DTYPE_BF16) {
          if (head_dim == 64)
            return pk2 ? launch_flat<B16, 64, 2, true>(p, tk, tv, g, st) : launch_flat<B16, 64, 1, true>(p, tk, tv, g, st);
          return pk2 ? launch_flat<B16, 128, 2, true>(p, tk, tv, g, st) : launch_flat<B16, 128, 1, true>(p, tk, tv, g, st);
        }
        if (head_dim == 64)
          return pk2 ? launch_flat<__half, 64, 2, true>(p, tk, tv, g, st)
                     : launch_flat<__half, 64, 1, true>(p, tk, tv, g, st);
        return pk2 ? launch_flat<__half, 128, 2, true>(p, tk, tv, g, st)
                   : launch_flat<__half, 128, 1, true>(p, tk, tv, g, st);
      }
      if (dtype == PA_DTYPE_BF16) {
        if (head_dim == 64)
          return pk2 ? launch_flat<B16, 64, 2, false>(p, tk, tv, g, st) : launch_flat<B16, 64, 1, false>(p, tk, tv, g, st);
        return pk2 ? launch_flat<B16, 128, 2, false>(p, tk, tv, g, st) : launch_flat<B16, 128, 1, false>(p, tk, tv, g, st);
      }
      if (head_dim == 64)
        return pk2 ? launch_flat<__half, 64, 2, false>(p, tk, tv, g, st)
                   : launch_flat<__half, 64, 1, false>(p, tk, tv, g, st);
      return pk2 ? launch_flat<__half, 128, 2, false>(p, tk, tv, g, st)
                 : launch_flat<__half, 128, 1, false>(p, tk, tv, g, st);
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
  g.scale = scale * k_scale;
  g.out_scale = v_scale;
  g.split_tokens = pl.split_tokens;
  g.max_splits = pl.splits;
  g.part_ml = pl.splits > 1 ? reinterpret_cast<float*>(ws + wl.part_ml) : nullptr;
  g.part_o = pl.splits > 1 ? reinterpret_cast<float*>(ws + wl.part_o) : nullptr;
  g.tickets = pl.splits > 1 ? reinterpret_cast<int*>(ws + wl.tickets) : nullptr;
  g.status = status;
  return launch_attn_generic(g, dtype, pl.splits, st, kv8 ? PA_DTYPE_FP8_E4M3 : dtype);
}

}  // namespace
}  // namespace pa

extern "C" int pa_kv_scatter_fp8(const void* k, int64_t k_s0, int64_t k_s1, int64_t k_s2, const void* v,
                                 int64_t v_s0, int64_t v_s1, int64_t v_s2, int src_dtype, const void* slot_mapping,
                                 int slot_is_int64, int64_t num_tokens, void* k_pool_layer, void* v_pool_layer,
                                 int64_t num_slots, int num_kv_heads, int head_dim, float k_scale, float v_scale,
                                 void* stream);

extern "C" int pa_paged_decode_fp8(const void* q, int64_t q_s0, int64_t q_s1, const void* new_k, const void* new_v,
                                   const int64_t* slot_mapping, void* k_pool_layer, void* v_pool_layer,
                                   int64_t num_blocks, int block_size, int num_kv_heads, int head_dim,
                                   const int64_t* block_tables, int64_t bt_stride, int64_t bt_width,
                                   const int64_t* context_lens, void* out, int64_t o_s0, int64_t o_s1, int batch,
                                   int num_q_heads, float scale, int dtype, float k_scale, float v_scale,
                                   int partition_tokens, int flags, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  using namespace pa;
  if (batch < 0 || (flags & ~kDecodeFlags)) return PA_ERR_INVALID;
  if (batch == 0) return PA_OK;
  const bool write = new_k != nullptr || new_v != nullptr || slot_mapping != nullptr;
  if (write) {
    if (new_k == nullptr || new_v == nullptr || slot_mapping == nullptr || partition_tokens != 0)
      return PA_ERR_INVALID;
    if (!((reinterpret_cast<uintptr_t>(new_k) | reinterpret_cast<uintptr_t>(new_v)) & 15)) {
      FusedWrite fw{new_k, new_v, slot_mapping};
      bool fused = false;
      const int r = decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads,
                                head_dim, block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch,
                                num_q_heads, scale, dtype, 0, workspace, workspace_bytes, stream, &fw, &fused, flags,
                                PA_DTYPE_FP8_E4M3, k_scale, v_scale);
      if (r != PA_OK || fused) return r;
    }
    // Not fusable here: quantizing scatter, then decode (which then waits
    // before its first read: the scatter just wrote pool rows).
    const int64_t s1 = head_dim, s0 = (int64_t)num_kv_heads * head_dim;
    const int r = pa_kv_scatter_fp8(new_k, s0, s1, 1, new_v, s0, s1, 1, dtype, slot_mapping, 1, batch, k_pool_layer,
                                    v_pool_layer, num_blocks * (int64_t)block_size, num_kv_heads, head_dim, k_scale,
                                    v_scale, stream);
    if (r != PA_OK) return r;
    flags = 0;
  }
  return decode_impl(q, q_s0, q_s1, k_pool_layer, v_pool_layer, num_blocks, block_size, num_kv_heads, head_dim,
                     block_tables, bt_stride, bt_width, context_lens, out, o_s0, o_s1, batch, num_q_heads, scale, dtype,
                     partition_tokens, workspace, workspace_bytes, stream, nullptr, nullptr, flags, PA_DTYPE_FP8_E4M3,
                     k_scale, v_scale);
}
