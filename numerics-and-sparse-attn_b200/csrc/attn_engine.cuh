// Warp-level GQA decode-attention engine on mma.sync m16n8k16 (fp16 in, fp32
// accumulate), shared by the dense, sink+window and KIVI kernels.
//
// One warp consumes 16 cached tokens at a time for the 8 query heads of one
// KV head:
//   S^T[16 tok x 8 heads]  = K[16 x 128] . Q^T[128 x 8]     (8 k-steps)
//   online softmax per head (column), exp2 domain
//   P^T B-operand          = movmatrix.trans of the fp16-packed S^T fragment
//   O^T[128 x 8] += V^T[128 x 16] . P^T[16 x 8]             (8 m-tiles)
// The group of 8 query heads is exactly the n = 8 of the instruction, so no
// lanes are wasted on padding.  K and V tiles are read from shared memory in
// the layout TMA produces with CU_TENSOR_MAP_SWIZZLE_128B for 64-element
// (128-byte) boxes: two regions [dims 0-63] and [dims 64-127], each
// rows x 128 B, 16-byte chunk c of row r stored at chunk c ^ (r % 8).  That
// makes every ldmatrix phase conflict-free.
#pragma once

#include "common.cuh"

namespace nsa {

struct WarpAttn {
  float m[2];       // running max (log2 domain) of heads 2t, 2t+1
  float l[2];       // per-lane partial softmax denominators of heads 2t, 2t+1
  float acc[8][4];  // O^T fragments: dims 16j+g / 16j+g+8, heads 2t / 2t+1
  uint32_t qb[8][2];

  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      m[i] = -INFINITY;
      l[i] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[j][c] = 0.f;
  }

  // Q^T B-fragments from an unswizzled [8 heads][128] fp16 smem block whose
  // rows are `row_bytes` apart.
  __device__ __forceinline__ void load_q(uint32_t qbase, int lane, uint32_t row_bytes = 256) {
    const int mi = lane >> 3, head = lane & 7;
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
      const int dim = 16 * (ks + (mi >> 1)) + (mi & 1) * 8;
      ldmatrix_x4(qbase + head * row_bytes + dim * 2, qb[ks][0], qb[ks][1], qb[ks + 1][0], qb[ks + 1][1]);
    }
  }

  // Online-softmax step for N blocks of 16 rows: raw scores s[h][] of rows g /
  // g+8 of block h for heads 2t / 2t+1 (g = lane / 4, t = lane % 4); rescales
  // the running state once and returns each block's P^T B-fragments (pb[h][0]:
  // rows 2t, 2t+1; pb[h][1]: rows 2t+8, 2t+9; column = head g).
  template <int N>
  __device__ __forceinline__ void softmax_rows(float (&s)[N][4], const bool (&valid_lo)[N], const bool (&valid_hi)[N],
                                               float scale_log2, uint32_t (&pb)[N][2]) {
    // scores in log2 units; masked rows -> -inf
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int h = 0; h < N; ++h) {
      s[h][0] = valid_lo[h] ? s[h][0] * scale_log2 : -INFINITY;
      s[h][1] = valid_lo[h] ? s[h][1] * scale_log2 : -INFINITY;
      s[h][2] = valid_hi[h] ? s[h][2] * scale_log2 : -INFINITY;
      s[h][3] = valid_hi[h] ? s[h][3] * scale_log2 : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(s[h][0], s[h][2]));
      mx1 = fmaxf(mx1, fmaxf(s[h][1], s[h][3]));
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m[0], mx0);
    const float mn1 = fmaxf(m[1], mx1);
    // reference point: 0 while nothing valid has been seen (avoids inf - inf)
    const float b0 = (mn0 == -INFINITY) ? 0.f : mn0;
    const float b1 = (mn1 == -INFINITY) ? 0.f : mn1;
    const float al0 = fast_exp2(m[0] - b0);
    const float al1 = fast_exp2(m[1] - b1);
    float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
    for (int h = 0; h < N; ++h) {
      const float p0 = fast_exp2(s[h][0] - b0);
      const float p1 = fast_exp2(s[h][1] - b1);
      const float p2 = fast_exp2(s[h][2] - b0);
      const float p3 = fast_exp2(s[h][3] - b1);
      sum0 += p0 + p2;
      sum1 += p1 + p3;
      pb[h][0] = movmatrix_trans(pack_half2(p0, p1));  // P[tok 2t,2t+1][head g]
      pb[h][1] = movmatrix_trans(pack_half2(p2, p3));  // P[tok 2t+8,2t+9][head g]
    }
    l[0] = l[0] * al0 + sum0;
    l[1] = l[1] * al1 + sum1;
    m[0] = mn0;
    m[1] = mn1;
    if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {  // skipped while no running max moves
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc[j][0] *= al0;
        acc[j][1] *= al1;
        acc[j][2] *= al0;
        acc[j][3] *= al1;
      }
    }
  }

  __device__ __forceinline__ void softmax16(float (&s)[4], bool valid_lo, bool valid_hi, float scale_log2,
                                            uint32_t& pb0, uint32_t& pb1) {
    float sh[1][4] = {{s[0], s[1], s[2], s[3]}};
    const bool vl[1] = {valid_lo}, vh[1] = {valid_hi};
    uint32_t pb[1][2];
    softmax_rows<1>(sh, vl, vh, scale_log2, pb);
    pb0 = pb[0][0];
    pb1 = pb[0][1];
  }

  // Consume tokens [row0, row0+16) of a swizzled tile whose regions are
  // `region_bytes` apart (rows kRowBytes apart, see tile_off).  valid_lo /
  // valid_hi: validity of rows row0+g and row0+g+8 for this lane (g = lane / 4).
  template <uint32_t kRowBytes = 128>
  __device__ __forceinline__ void consume16(uint32_t kbase, uint32_t vbase, uint32_t region_bytes, int row0,
                                            bool valid_lo, bool valid_hi, float scale_log2, int lane) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    {
      // two accumulators halve the dependent mma chain of the 8 k-steps
      float s2[4] = {0.f, 0.f, 0.f, 0.f};
      const uint32_t row = row0 + ((lane >> 3) & 1) * 8 + (lane & 7);
      const uint32_t hi = lane >> 4;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a0, a1, a2, a3;
        const uint32_t addr = kbase + tile_off<kRowBytes>(row, 8 * (ks >> 2) + 2 * (ks & 3) + hi, region_bytes);
        ldmatrix_x4(addr, a0, a1, a2, a3);
        if (ks & 1)
          mma_16816(s2, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
        else
          mma_16816(s, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) s[c] += s2[c];
    }
    uint32_t pb0, pb1;
    softmax16(s, valid_lo, valid_hi, scale_log2, pb0, pb1);
    {
      const uint32_t mi = lane >> 3;
      const uint32_t row = row0 + (mi >> 1) * 8 + (lane & 7);
      const uint32_t hi = mi & 1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t a0, a1, a2, a3;
        const uint32_t addr = vbase + tile_off<kRowBytes>(row, 8 * (j >> 2) + 2 * (j & 3) + hi, region_bytes);
        ldmatrix_x4_trans(addr, a0, a1, a2, a3);
        mma_16816(acc[j], a0, a1, a2, a3, pb0, pb1);
      }
    }
  }

  // Consume N blocks of 16 tokens, rows [row0, row0 + 16N) of a swizzled tile
  // (regions `region_bytes` apart, rows kRowBytes apart), with one softmax
  // step for all of them.  valid_lo[h] / valid_hi[h]: validity of rows
  // row0+16h+g and row0+16h+g+8.
  template <int N, uint32_t kRowBytes = 128>
  __device__ __forceinline__ void consume_rows(uint32_t kbase, uint32_t vbase, uint32_t region_bytes, int row0,
                                               const bool (&valid_lo)[N], const bool (&valid_hi)[N], float scale_log2,
                                               int lane) {
    float s[N][4], s2[N][4];
#pragma unroll
    for (int h = 0; h < N; ++h)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[h][c] = s2[h][c] = 0.f;
    {
      const uint32_t hi = lane >> 4;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int h = 0; h < N; ++h) {
          const uint32_t row = row0 + 16 * h + ((lane >> 3) & 1) * 8 + (lane & 7);
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(kbase + tile_off<kRowBytes>(row, 8 * (ks >> 2) + 2 * (ks & 3) + hi, region_bytes), a0, a1, a2,
                      a3);
          mma_16816((ks & 1) ? s2[h] : s[h], a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < N; ++h)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[h][c] += s2[h][c];
    uint32_t pb[N][2];
    softmax_rows<N>(s, valid_lo, valid_hi, scale_log2, pb);
    const uint32_t mi = lane >> 3;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int h = 0; h < N; ++h) {
        const uint32_t row = row0 + 16 * h + (mi >> 1) * 8 + (lane & 7);
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4_trans(vbase + tile_off<kRowBytes>(row, 8 * (j >> 2) + 2 * (j & 3) + (mi & 1), region_bytes), a0,
                          a1, a2, a3);
        mma_16816(acc[j], a0, a1, a2, a3, pb[h][0], pb[h][1]);
      }
    }
  }
};

// Cross-warp merge buffers for the epilogue of one (unit, token-range) piece.
// First, each warp of group 1 hands its raw state to the warp of group 0
// with the same index (identical fragment layout, so the merge is
// element-wise in registers).  Then the group-0 warps publish their
// merged states to `red`, which aliases `xfer`.  red.o rows are padded to
// 132 floats so the fragment scatter is conflict-free.
constexpr int kRedStride = 132;
constexpr int kXferWords = 36;  // 32 accumulators + 2 maxima + 2 partial sums
struct alignas(16) EpilogueSmem {  // 16-byte aligned: merge_warps reads float4s
  union {
    float xfer[kGroupWarps][kXferWords][32];
    struct {
      float o[kGroupWarps][kGroupHeads][kRedStride];
      float m[kGroupWarps][kGroupHeads];
      float l[kGroupWarps][kGroupHeads];
    } red;
  };
  int ticket;
};

__device__ __forceinline__ void warp_xfer_out(const WarpAttn& st, EpilogueSmem& ep, int wq, int lane) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) ep.xfer[wq][4 * j + c][lane] = st.acc[j][c];
  ep.xfer[wq][32][lane] = st.m[0];
  ep.xfer[wq][33][lane] = st.m[1];
  ep.xfer[wq][34][lane] = st.l[0];
  ep.xfer[wq][35][lane] = st.l[1];
}

__device__ __forceinline__ void warp_xfer_in(WarpAttn& st, const EpilogueSmem& ep, int wq, int lane) {
  float fa[2], fb[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float mb = ep.xfer[wq][32 + h][lane];
    const float mn = fmaxf(st.m[h], mb);
    fa[h] = (st.m[h] == -INFINITY) ? 0.f : fast_exp2(st.m[h] - mn);
    fb[h] = (mb == -INFINITY) ? 0.f : fast_exp2(mb - mn);
    st.m[h] = mn;
    st.l[h] = fa[h] * st.l[h] + fb[h] * ep.xfer[wq][34 + h][lane];
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) st.acc[j][c] = fa[c & 1] * st.acc[j][c] + fb[c & 1] * ep.xfer[wq][4 * j + c][lane];
}

// Publish a group-0 warp's (merged) state to the epilogue buffers.
__device__ __forceinline__ void warp_publish(const WarpAttn& st, EpilogueSmem& ep, int wq, int lane) {
  const int g = lane >> 2, t = lane & 3;
  float l0 = st.l[0], l1 = st.l[1];
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ep.red.o[wq][2 * t][16 * j + g] = st.acc[j][0];
    ep.red.o[wq][2 * t + 1][16 * j + g] = st.acc[j][1];
    ep.red.o[wq][2 * t][16 * j + g + 8] = st.acc[j][2];
    ep.red.o[wq][2 * t + 1][16 * j + g + 8] = st.acc[j][3];
  }
  if (g == 0) {
    ep.red.m[wq][2 * t] = st.m[0];
    ep.red.m[wq][2 * t + 1] = st.m[1];
    ep.red.l[wq][2 * t] = l0;
    ep.red.l[wq][2 * t + 1] = l1;
  }
}

// Merge the published group-0 warp states for one head and N consecutive dims.
// Returns the normalized output in o[4] and the piece's log2-sum-exp in lse
// (-inf when the piece saw no valid token; o is then 0/0 = NaN).
template <int N>
__device__ __forceinline__ void merge_warps(const EpilogueSmem& ep, int head, int d0, float (&o)[N], float& lse) {
  float mstar = -INFINITY;
#pragma unroll
  for (int w = 0; w < kGroupWarps; ++w) mstar = fmaxf(mstar, ep.red.m[w][head]);
  float f[kGroupWarps];
  float L = 0.f;
#pragma unroll
  for (int w = 0; w < kGroupWarps; ++w) {
    const float mw = ep.red.m[w][head];
    f[w] = (mw == -INFINITY) ? 0.f : fast_exp2(mw - mstar);
    L += f[w] * ep.red.l[w][head];
  }
  static_assert(N % 4 == 0, "float4 reads of the published rows");
#pragma unroll
  for (int i = 0; i < N; i += 4) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kGroupWarps; ++w) {  // rows are 528 bytes apart and d0 % 4 == 0: 16-byte aligned
      const float4 v = *reinterpret_cast<const float4*>(&ep.red.o[w][head][d0 + i]);
      a.x += f[w] * v.x;
      a.y += f[w] * v.y;
      a.z += f[w] * v.z;
      a.w += f[w] * v.w;
    }
    // L == 0 (nothing attended): 0/0 = NaN, as the reference
    o[i] = __fdividef(a.x, L);
    o[i + 1] = __fdividef(a.y, L);
    o[i + 2] = __fdividef(a.z, L);
    o[i + 3] = __fdividef(a.w, L);
  }
  lse = (L > 0.f) ? mstar + __log2f(L) : -INFINITY;
}

__device__ __forceinline__ void store_half4(__half* dst, const float (&o)[4]) {
  uint2 v;
  v.x = pack_half2(o[0], o[1]);
  v.y = pack_half2(o[2], o[3]);
  *reinterpret_cast<uint2*>(dst) = v;
}
__device__ __forceinline__ void store_half8(__half* dst, const float (&o)[8]) {  // dst 16-byte aligned
  uint4 v;
  v.x = pack_half2(o[0], o[1]);
  v.y = pack_half2(o[2], o[3]);
  v.z = pack_half2(o[4], o[5]);
  v.w = pack_half2(o[6], o[7]);
  *reinterpret_cast<uint4*>(dst) = v;
}

// Split-K partials of one unit: `n` pieces, each [8 heads] lse and
// [8 heads][128] normalized outputs.  Log-sum-exp combine with warp shuffles:
// the calling warp reduces heads [head0, head0 + n_heads); lanes hold pieces
// for the max / sum, then 4 dims each for the weighted output sum.  Reads use
// ld.global.cg (the partials were written by other SMs); every partial read
// is zeroed again so the workspace is all-zero between launches whatever its
// next layout.
__device__ __forceinline__ void combine_pieces(float* part_lse, float* part_o, int n, __half* out, int head0,
                                               int n_heads, int lane) {
  for (int head = head0; head < head0 + n_heads; ++head) {
    float M = -INFINITY;
    for (int i = lane; i < n; i += 32) M = fmaxf(M, __ldcg(part_lse + i * kGroupHeads + head));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float W = 0.f;
    for (int i = lane; i < n; i += 32) {
      const float x = __ldcg(part_lse + i * kGroupHeads + head);
      W += (x == -INFINITY) ? 0.f : fast_exp2(x - M);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) W += __shfl_xor_sync(0xffffffffu, W, off);
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int base = 0; base < n; base += 32) {
      const int i = base + lane;
      const float x = (i < n) ? __ldcg(part_lse + i * kGroupHeads + head) : -INFINITY;
      const float wi = (x == -INFINITY) ? 0.f : fast_exp2(x - M);
      const int cnt = min(32, n - base);
      for (int j = 0; j < cnt; ++j) {
        const float wj = __shfl_sync(0xffffffffu, wi, j);
        float4* src = reinterpret_cast<float4*>(part_o + ((base + j) * kGroupHeads + head) * kHeadDim) + lane;
        if (wj != 0.f) {
          const float4 v = __ldcg(src);
          a.x += wj * v.x;
          a.y += wj * v.y;
          a.z += wj * v.z;
          a.w += wj * v.w;
        }
        __stcg(src, make_float4(0.f, 0.f, 0.f, 0.f));
      }
    }
    __syncwarp();
    for (int i = lane; i < n; i += 32) __stcg(part_lse + i * kGroupHeads + head, 0.f);
    const float inv = __fdividef(1.f, W);  // W == 0 (no valid token anywhere) -> inf * 0 = NaN, as the reference's 0/0
    __half2* dst = reinterpret_cast<__half2*>(out + head * kHeadDim + lane * 4);
    dst[0] = __floats2half2_rn(a.x * inv, a.y * inv);
    dst[1] = __floats2half2_rn(a.z * inv, a.w * inv);
  }
}

}  // namespace nsa
