// KIVI 2-bit sink + window decode attention (reference: quant_kernel.py
// :316-581) over either the reference's 14-tensor layout or the streaming
// ring layout of nsa_kivi_stream_cache.
//
// Per (batch, kv_head) unit the work is a fixed list of items:
//   Q-batches  up to 8 quantized 32-token groups (slot 0 of batch 0 is the
//              padded sink group, then window groups in physical order),
//              staged into shared memory with 1-D bulk copies (3 KiB/group);
//   F-tiles    64 slots of the fp16 residual (ring), staged by TMA with the
//              128-byte swizzle exactly like the fp16 kernel.
// Items that hold no attended token are skipped by producer and consumers
// alike (both derive it from the same per-unit metadata).  Consumers: two
// groups of 4 warps take alternate items.  For a Q-batch each warp
// dequantizes 16-token halves of groups into a private fp16 tile (swizzled
// like a TMA tile; unattended tokens are written as zeros) and runs the same
// mma.sync engine on it, so both regimes accumulate into one online softmax.
// Split-K / unit-aligned scheduling and the in-launch combine are the fp16
// kernel's.
#include <cstdlib>

#include "attn_engine.cuh"
#include "host_util.h"

namespace nsa {
namespace {

constexpr int kStages = 4;
static_assert(kStages % kGroups == 0, "each stage must belong to one consumer group");
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kRegionBytes = kTile * 128;
constexpr uint32_t kTileBytes = 2 * kRegionBytes;
constexpr uint32_t kStageBytes = 2 * kTileBytes;  // 32 KiB
constexpr uint32_t kQBytes = kGroupHeads * kHeadDim * 2;
constexpr int kBatchGroups = 8;                   // quantized groups per Q-batch
// Q-batch stage layout (byte offsets); one slot per group
constexpr uint32_t kOffKP = 0, kOffKS = 8192, kOffKZ = 10240, kOffVP = 12288, kOffVS = 20480, kOffVZ = 22528;
constexpr uint32_t kScratchRegion = 16 * 128;     // 16 rows x 64 dims fp16
constexpr uint32_t kScratchTile = 2 * kScratchRegion;

struct KiviMeta {
  int32_t n_sink;    // attended sink tokens
  int32_t grp_head;  // physical window-group slot of the oldest live group
  int32_t n_grp;     // live window groups
  int32_t tok_skip;  // unattended tokens at the start of the oldest live group
  int32_t res_head;  // physical residual slot of the oldest live token
  int32_t n_res;     // live residual tokens
  int32_t res_skip;  // unattended live residual tokens (oldest first)
  int32_t pad;
};

struct Smem {
  uint8_t stage[kStages][kStageBytes];  // 1024-aligned
  uint8_t scratch[kConsumerWarps][2][kScratchTile];
  uint8_t q[2][kQBytes];
  KiviMeta meta[2];
  EpilogueSmem ep;
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t q_full[2];
  uint64_t q_empty[2];
};

struct KParams {
  const __half* q;
  __half* o;
  int64_t n_units;
  int n_kv_heads;
  int layout;  // 0: reference 14-tensor layout; 1: streaming ring
  int64_t seq_len;
  const int64_t* unit_lens;
  int window, sink, residual, n_groups, res_cap;
  int n_qb, n_ft;
  int64_t tiles_per_unit;  // items per unit
  int64_t total_tiles;
  int n_ctas;
  int unit_aligned;
  int max_pieces;
  float scale_log2;
  const uint8_t* ks_p;
  const __half* ks_s;
  const __half* ks_z;
  const uint8_t* vs_p;
  const __half* vs_s;
  const __half* vs_z;
  const uint8_t* kw_p;
  const __half* kw_s;
  const __half* kw_z;
  const uint8_t* vw_p;
  const __half* vw_s;
  const __half* vw_z;
  int* counters;
  float* part_lse;
  float* part_o;
  int* err;
};

__device__ __forceinline__ int32_t clampi(int64_t x, int64_t lo, int64_t hi) {
  return static_cast<int32_t>(x < lo ? lo : (x > hi ? hi : x));
}

// Per-unit metadata from the unit's length (see nsa_kivi_stream_cache and
// _kv_indices, sparse_kernel.py:15-46, for the two layouts).
__device__ __forceinline__ KiviMeta make_meta(const KParams& p, int64_t unit) {
  KiviMeta m;
  const int64_t S = p.sink, W = p.window, R = p.residual, NG = p.n_groups;
  if (p.layout == 0) {
    const int64_t len = p.seq_len;
    const int64_t nw = W - R;  // window-old tokens
    const int64_t n_inv = clampi(S - len + W, 0, W);  // window indices < n_inv are not attended
    m.n_sink = clampi(len, 0, S);
    m.grp_head = 0;
    m.n_grp = static_cast<int32_t>(NG);
    m.tok_skip = clampi(n_inv, 0, nw);
    m.res_head = 0;
    m.n_res = static_cast<int32_t>(R);
    m.res_skip = clampi(n_inv - nw, 0, R);
  } else {
    const int64_t len = p.unit_lens[unit];
    const int64_t C = p.res_cap;
    const int64_t n_stream = len > S ? len - S : 0;
    const int64_t F = n_stream > R ? (n_stream - R) / 32 : 0;  // flushed groups
    const int64_t first = (len - W > S) ? len - W : S;         // oldest attended position
    m.n_sink = clampi(len, 0, S);
    m.n_res = static_cast<int32_t>(n_stream - 32 * F);
    m.res_head = static_cast<int32_t>((32 * F) % C);
    m.res_skip = clampi(first - S - 32 * F, 0, m.n_res);
    m.n_grp = static_cast<int32_t>(F < NG ? F : NG);
    m.grp_head = NG > 0 ? static_cast<int32_t>((F - m.n_grp) % NG) : 0;
    m.tok_skip = clampi(first - S - 32 * (F - m.n_grp), 0, 32 * int64_t(m.n_grp));
  }
  return m;
}

// Distance of window-group slot p from the oldest live group (>= n_grp: dead).
__device__ __forceinline__ int grp_age(const KParams& p, const KiviMeta& m, int gp) {
  int d = gp - m.grp_head;
  if (d < 0) d += p.n_groups;
  return d;
}

// Attended token j (0..31) of batch slot `slot` of Q-batch `b`?
__device__ __forceinline__ bool q_token_valid(const KParams& p, const KiviMeta& m, int b, int slot, int j) {
  const int v = kBatchGroups * b + slot;
  if (v == 0) return j < m.n_sink;
  if (v > p.n_groups) return false;
  const int age = grp_age(p, m, v - 1);
  return age < m.n_grp && 32 * age + j >= m.tok_skip;
}

__device__ __forceinline__ bool q_slot_live(const KParams& p, const KiviMeta& m, int b, int slot) {
  const int v = kBatchGroups * b + slot;
  if (v == 0) return m.n_sink > 0;
  if (v > p.n_groups) return false;
  const int age = grp_age(p, m, v - 1);
  return age < m.n_grp && 32 * age + 31 >= m.tok_skip;
}

__device__ __forceinline__ bool res_slot_valid(const KParams& p, const KiviMeta& m, int r) {
  if (r >= p.res_cap) return false;
  int d = r - m.res_head;
  if (d < 0) d += p.res_cap;
  return d >= m.res_skip && d < m.n_res;
}

// Whether item `it` of a unit holds any attended token.
__device__ __forceinline__ bool item_live(const KParams& p, const KiviMeta& m, int it) {
  if (it < p.n_qb) {
    for (int s = 0; s < kBatchGroups; ++s)
      if (q_slot_live(p, m, it, s)) return true;
    return false;
  }
  // attended residual slots form the ring interval [a, a + len) mod C
  const int r0 = (it - p.n_qb) * kTile, r1 = min(r0 + kTile, p.res_cap);
  const int len = m.n_res - m.res_skip;
  if (len <= 0 || r1 <= r0) return false;
  int a = m.res_head + m.res_skip;
  if (a >= p.res_cap) a -= p.res_cap;
  const int e = a + len;
  if (max(a, r0) < min(min(e, p.res_cap), r1)) return true;
  return e > p.res_cap && r0 < e - p.res_cap;
}

// CTA owning global item X under the even split of `total` items over `ctas`.
__device__ __forceinline__ int64_t owner_cta(int64_t X, int64_t total, int64_t ctas) {
  return ((X + 1) * ctas + total - 1) / total - 1;
}

struct Piece {
  int64_t unit, t_begin, t_end;
  int slot, n_pieces;
};

struct PieceIter {
  int64_t X, X1;
  __device__ __forceinline__ PieceIter(const KParams& p) {
    const int64_t c = blockIdx.x;
    if (p.unit_aligned) {
      X = (c * p.n_units / p.n_ctas) * p.tiles_per_unit;
      X1 = ((c + 1) * p.n_units / p.n_ctas) * p.tiles_per_unit;
    } else {
      X = c * p.total_tiles / p.n_ctas;
      X1 = (c + 1) * p.total_tiles / p.n_ctas;
    }
  }
  __device__ __forceinline__ bool next(const KParams& p, Piece& pc) {
    if (X >= X1) return false;
    const int64_t tpu = p.tiles_per_unit;
    pc.unit = X / tpu;
    const int64_t ub = pc.unit * tpu, ue = ub + tpu;
    const int64_t e = min(X1, ue);
    pc.t_begin = X - ub;
    pc.t_end = e - ub;
    if (p.unit_aligned) {
      pc.slot = 0;
      pc.n_pieces = 1;
    } else {
      const int64_t c0 = owner_cta(ub, p.total_tiles, p.n_ctas);
      const int64_t c1 = owner_cta(ue - 1, p.total_tiles, p.n_ctas);
      pc.slot = static_cast<int>(blockIdx.x - c0);
      pc.n_pieces = static_cast<int>(c1 - c0 + 1);
    }
    X = e;
    return true;
  }
};

// ---------------------------------------------------------------- dequant
// 2-bit codes -> fp16 via the 1024 + c exponent trick: (bits | 0x6400) is
// the half 1024 + bits, exact for bits < 1024.
__device__ __forceinline__ __half2 u32_as_h2(uint32_t x) { return *reinterpret_cast<__half2*>(&x); }
__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Dequantize K of 16 tokens (half `hf` of batch slot `slot`) into a swizzled
// [2][16][64] fp16 tile.  Lane = (byte row br = lane/8: tokens 4br..4br+3,
// channel chunk cc = lane%8: channels 16cc..16cc+15).
__device__ __forceinline__ void dequant_k16(uint32_t stage, uint32_t dst, int slot, int hf, int lane,
                                            uint32_t valid_mask /* bit t: token t (0..15) attended */) {
  const int br = lane >> 3, cc = lane & 7;
  uint4 codes;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(codes.x), "=r"(codes.y), "=r"(codes.z), "=r"(codes.w)
               : "r"(stage + kOffKP + slot * 1024 + (4 * hf + br) * 128 + 16 * cc));
  uint32_t sc[8], zr[8];
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(sc[0]), "=r"(sc[1]), "=r"(sc[2]), "=r"(sc[3])
               : "r"(stage + kOffKS + slot * 256 + 32 * cc));
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(sc[4]), "=r"(sc[5]), "=r"(sc[6]), "=r"(sc[7])
               : "r"(stage + kOffKS + slot * 256 + 32 * cc + 16));
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(zr[0]), "=r"(zr[1]), "=r"(zr[2]), "=r"(zr[3])
               : "r"(stage + kOffKZ + slot * 256 + 32 * cc));
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(zr[4]), "=r"(zr[5]), "=r"(zr[6]), "=r"(zr[7])
               : "r"(stage + kOffKZ + slot * 256 + 32 * cc + 16));
  __half2 s2[8], nz2[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s2[i] = u32_as_h2(sc[i]);
    nz2[i] = __hneg2(__hmul2(s2[i], u32_as_h2(zr[i])));
  }
  const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
  const __half2 k1024 = u32_as_h2(0x64006400u);
  // region of channels 16cc..: cc/4; chunks 2cc, 2cc+1 (mod 8).  Lanes with
  // cc >= 4 store the second chunk first so a phase spreads over all banks.
  const uint32_t region = dst + (cc >> 2) * kScratchRegion;
  const uint32_t ch0 = (2 * cc) & 7;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int row = 4 * br + j;
    const bool ok = (valid_mask >> row) & 1u;
    uint32_t out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t x = __byte_perm(w[i >> 1], 0u, (i & 1) ? 0x4342u : 0x4140u);  // [b_lo, 0, b_hi, 0]
      const uint32_t c = ((x >> (2 * j)) & 0x00030003u) | 0x64006400u;
      const __half2 v = __hfma2(__hsub2(u32_as_h2(c), k1024), s2[i], nz2[i]);
      out[i] = ok ? h2_as_u32(v) : 0u;
    }
    const bool swap = (cc >> 2) & 1;
    const uint32_t a0 = region + swz128(row, swap ? ch0 + 1 : ch0);
    const uint32_t a1 = region + swz128(row, swap ? ch0 : ch0 + 1);
    uint32_t f[4], sc2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[i] = swap ? out[4 + i] : out[i];
      sc2[i] = swap ? out[i] : out[4 + i];
    }
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a0), "r"(f[0]), "r"(f[1]), "r"(f[2]), "r"(f[3]));
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a1), "r"(sc2[0]), "r"(sc2[1]), "r"(sc2[2]),
                 "r"(sc2[3]));
  }
}

// Dequantize V of 16 tokens into a swizzled [2][16][64] fp16 tile.
// Lane = (token tau = lane/2, channel half hv = lane%2: channels 64hv..+63).
__device__ __forceinline__ void dequant_v16(uint32_t stage, uint32_t dst, int slot, int hf, int lane,
                                            uint32_t valid_mask) {
  const int tau = lane >> 1, hv = lane & 1;
  const int trow = 16 * hf + tau;  // token within the 32-token group
  uint4 codes;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(codes.x), "=r"(codes.y), "=r"(codes.z), "=r"(codes.w)
               : "r"(stage + kOffVP + slot * 1024 + trow * 32 + 16 * hv));
  uint32_t sc, zr;  // groups 2hv, 2hv+1 of this token
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(sc) : "r"(stage + kOffVS + slot * 256 + trow * 8 + 4 * hv));
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(zr) : "r"(stage + kOffVZ + slot * 256 + trow * 8 + 4 * hv));
  const __half2 s_pair = u32_as_h2(sc), z_pair = u32_as_h2(zr);
  const __half2 nz_pair = __hneg2(__hmul2(s_pair, z_pair));
  const bool ok = (valid_mask >> tau) & 1u;
  const __half2 k1024 = u32_as_h2(0x64006400u);
  const __half2 quarter_hi = __halves2half2(__float2half_rn(1.f), __float2half_rn(0.25f));
  const uint32_t region = dst + hv * kScratchRegion;
  // The two lanes of a token write chunks ch and ch ^ 4 at the same time
  // (different banks); chunk ch = channels 8ch..8ch+7 of this half = bytes
  // 2ch, 2ch+1 of the loaded 16; its channel group is ch / 4.
#pragma unroll
  for (int ci = 0; ci < 8; ++ci) {
    const int ch = ci ^ (hv << 2);
    const uint32_t wsel = (ch < 2) ? codes.x : (ch < 4) ? codes.y : (ch < 6) ? codes.z : codes.w;
    const __half2 s = (ch < 4) ? __low2half2(s_pair) : __high2half2(s_pair);
    const __half2 nz = (ch < 4) ? __low2half2(nz_pair) : __high2half2(nz_pair);
    uint32_t out[4];
#pragma unroll
    for (int bb = 0; bb < 2; ++bb) {
      const uint32_t k = (2 * ch + bb) & 3;
      const uint32_t x = __byte_perm(wsel, 0u, 0x4040u | (k << 8) | k);  // [b, 0, b, 0]
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        // channels (4 byte + 2hh, +1): bits 4hh..4hh+1 (lo) and 4hh+2..+3 (hi, scaled by 4)
        const uint32_t c = ((x >> (4 * hh)) & 0x000C0003u) | 0x64006400u;
        const __half2 cv = __hmul2(__hsub2(u32_as_h2(c), k1024), quarter_hi);
        const __half2 v = __hfma2(cv, s, nz);
        out[2 * bb + hh] = ok ? h2_as_u32(v) : 0u;
      }
    }
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(region + swz128(tau, ch)), "r"(out[0]), "r"(out[1]),
                 "r"(out[2]), "r"(out[3]));
  }
}

// Zero the V rows of slots that are not attended, so stale or
// uninitialised cache memory (possibly NaN) cannot reach the P.V product.
__device__ __forceinline__ void zero_invalid_v_rows(uint32_t vbase, uint32_t region_bytes, int row0, bool v_lo,
                                                    bool v_hi, int lane) {
  const unsigned bad = __ballot_sync(0xffffffffu, !(v_lo && v_hi));
  if (bad == 0) return;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (h == 0 ? v_lo : v_hi) continue;
    const uint32_t row = row0 + g + 8 * h;
    // each of the 4 lanes of row group g clears 4 of the row's 16 chunks
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t chunk = 4 * t + c;  // 0..15
      const uint32_t a = vbase + (chunk >> 3) * region_bytes + swz128(row, chunk & 7);
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(a), "r"(0u));
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kThreads, 1)
    kivi_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), kGroupWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&sm.q_full[s]), 1);
      mbar_init(smem_u32(&sm.q_empty[s]), kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  // CTA-local live item k lives in stage k % kStages, phase (k / kStages) & 1,
  // and is consumed by group k % kGroups.
  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      int qs = 0;
      uint32_t qphase = 0, k = 0;
      PieceIter it(p);
      Piece pc;
      while (it.next(p, pc)) {
        if (!mbar_wait(smem_u32(&sm.q_empty[qs]), qphase ^ 1, p.err)) return;
        const KiviMeta meta = make_meta(p, pc.unit);
        sm.meta[qs] = meta;  // published by the arrive below (release)
        mbar_arrive_expect_tx(smem_u32(&sm.q_full[qs]), kQBytes);
        bulk_load(smem_u32(sm.q[qs]), p.q + pc.unit * kGroupHeads * kHeadDim, kQBytes, smem_u32(&sm.q_full[qs]));
        if (++qs == 2) { qs = 0; qphase ^= 1; }
        const int64_t u = pc.unit;
        for (int64_t t = pc.t_begin; t < pc.t_end; ++t) {
          const int itm = static_cast<int>(t);
          if (!item_live(p, meta, itm)) continue;
          const uint32_t stage = k % kStages, phase = (k / kStages) & 1;
          ++k;
          if (!mbar_wait(smem_u32(&sm.empty[stage]), phase ^ 1, p.err)) return;
          const uint32_t fb = smem_u32(&sm.full[stage]);
          const uint32_t sd = smem_u32(sm.stage[stage]);
          if (itm < p.n_qb) {
            // Q-batch: sink group (slot 0 of batch 0) + window groups [p0, p1)
            const int b = itm;
            const bool has_sink = (b == 0);
            const int p0 = b == 0 ? 0 : kBatchGroups * b - 1;
            const int p1 = min(p.n_groups, kBatchGroups * b + kBatchGroups - 1);
            const int so = p0 + 1 - kBatchGroups * b;  // batch slot of group p0
            const uint32_t ng = p1 > p0 ? p1 - p0 : 0;
            const uint32_t bytes = (has_sink ? 3072u : 0u) + ng * 3072u;
            mbar_arrive_expect_tx(fb, bytes);
            if (has_sink) {
              bulk_load(sd + kOffKP, p.ks_p + u * 1024, 1024, fb);
              bulk_load(sd + kOffKS, p.ks_s + u * 128, 256, fb);
              bulk_load(sd + kOffKZ, p.ks_z + u * 128, 256, fb);
              bulk_load(sd + kOffVP, p.vs_p + u * 1024, 1024, fb);
              bulk_load(sd + kOffVS, p.vs_s + u * 128, 256, fb);
              bulk_load(sd + kOffVZ, p.vs_z + u * 128, 256, fb);
            }
            if (ng) {
              const int64_t gbase = u * p.n_groups + p0;
              bulk_load(sd + kOffKP + so * 1024, p.kw_p + gbase * 1024, ng * 1024, fb);
              bulk_load(sd + kOffKS + so * 256, p.kw_s + gbase * 128, ng * 256, fb);
              bulk_load(sd + kOffKZ + so * 256, p.kw_z + gbase * 128, ng * 256, fb);
              bulk_load(sd + kOffVP + so * 1024, p.vw_p + gbase * 1024, ng * 1024, fb);
              bulk_load(sd + kOffVS + so * 256, p.vw_s + gbase * 128, ng * 256, fb);
              bulk_load(sd + kOffVZ + so * 256, p.vw_z + gbase * 128, ng * 256, fb);
            }
          } else {
            mbar_arrive_expect_tx(fb, kStageBytes);
            const int row = (itm - p.n_qb) * kTile;
            const int uu = static_cast<int>(u);
            tma_load_3d(sd, &tmK, fb, 0, row, uu);
            tma_load_3d(sd + kRegionBytes, &tmK, fb, 64, row, uu);
            tma_load_3d(sd + kTileBytes, &tmV, fb, 0, row, uu);
            tma_load_3d(sd + kTileBytes + kRegionBytes, &tmV, fb, 64, row, uu);
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int grp = warp / kGroupWarps, wq = warp % kGroupWarps;
  const int g = lane >> 2;
  int qs = 0;
  uint32_t qphase = 0, k = 0;
  bool aborted = false;
  WarpAttn st;
  const uint32_t scr_k = smem_u32(sm.scratch[warp][0]);
  const uint32_t scr_v = smem_u32(sm.scratch[warp][1]);
  PieceIter it(p);
  Piece pc;
  while (it.next(p, pc)) {
    if (!aborted && !mbar_wait(smem_u32(&sm.q_full[qs]), qphase, p.err)) aborted = true;
    // Q fragments are reloaded from the slot for every 16-token job (so they
    // are not live across the dequantization); the slot is released after
    // the piece's last job.
    const uint32_t qaddr = smem_u32(sm.q[qs]);
    const int qslot = qs;
    const KiviMeta meta = sm.meta[qs];
    if (++qs == 2) { qs = 0; qphase ^= 1; }
    st.reset();
    for (int64_t t = pc.t_begin; t < pc.t_end; ++t) {
      const int itm = static_cast<int>(t);
      if (!item_live(p, meta, itm)) continue;
      const uint32_t kk = k++;
      if ((kk % kGroups) != static_cast<uint32_t>(grp)) continue;
      const uint32_t stage = kk % kStages, phase = (kk / kStages) & 1;
      if (!aborted && !mbar_wait(smem_u32(&sm.full[stage]), phase, p.err)) aborted = true;
      const uint32_t sd = smem_u32(sm.stage[stage]);
      const bool is_q = itm < p.n_qb;
      // Jobs of 16 tokens for this warp: a Q-batch has 16 half-groups (this
      // warp takes every 4th, dequantized into its scratch tile); an F-tile
      // has one (rows 16wq.. of the TMA tile).  One engine call site serves
      // both so the kernel stays within its register budget.
      for (int mt = wq; mt < (is_q ? 2 * kBatchGroups : wq + 1); mt += kGroupWarps) {
        uint32_t kb, vb, rb;
        int row0;
        bool v_lo, v_hi;
        if (is_q) {
          const int slot = mt >> 1, hf = mt & 1;
          // validity of the 16 tokens of this half (bit t = token 16hf + t)
          uint32_t vm = 0;
          if (lane < 16) vm = q_token_valid(p, meta, itm, slot, 16 * hf + lane) ? 1u : 0u;
          vm = __ballot_sync(0xffffffffu, vm != 0) & 0xffffu;
          if (vm == 0) continue;
          dequant_k16(sd, scr_k, slot, hf, lane, vm);
          dequant_v16(sd, scr_v, slot, hf, lane, vm);
          __syncwarp();
          kb = scr_k;
          vb = scr_v;
          rb = kScratchRegion;
          row0 = 0;
          v_lo = (vm >> g) & 1u;
          v_hi = (vm >> (g + 8)) & 1u;
        } else {
          const int r0 = (itm - p.n_qb) * kTile + 16 * wq;
          v_lo = res_slot_valid(p, meta, r0 + g);
          v_hi = res_slot_valid(p, meta, r0 + g + 8);
          kb = sd;
          vb = sd + kTileBytes;
          rb = kRegionBytes;
          row0 = 16 * wq;
          zero_invalid_v_rows(vb, rb, row0, v_lo, v_hi, lane);
        }
        st.load_q(qaddr, lane);
        st.consume16(kb, vb, rb, row0, v_lo, v_hi, p.scale_log2, lane);
        __syncwarp();  // scratch is rewritten by the next job
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.empty[stage]));
    }

    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sm.q_empty[qslot]));

    // ---- epilogue (as in the fp16 kernel)
    if (grp == 1) warp_xfer_out(st, sm.ep, wq, lane);
    consumer_sync();
    if (grp == 0) warp_xfer_in(st, sm.ep, wq, lane);
    consumer_sync();
    if (grp == 0) warp_publish(st, sm.ep, wq, lane);
    consumer_sync();
    const int ct = threadIdx.x;
    const int hh = ct >> 5, d0 = (ct & 31) * 4;
    float o[4], lse;
    merge_warps(sm.ep, hh, d0, o, lse);
    __half* out = p.o + pc.unit * kGroupHeads * kHeadDim;
    if (pc.n_pieces == 1) {
      store_half4(out + hh * kHeadDim + d0, o);
    } else {
      const int64_t pidx = pc.unit * p.max_pieces + pc.slot;
      float* po = p.part_o + (pidx * kGroupHeads + hh) * kHeadDim + d0;
      *reinterpret_cast<float4*>(po) = make_float4(o[0], o[1], o[2], o[3]);
      if ((ct & 31) == 0) p.part_lse[pidx * kGroupHeads + hh] = lse;
      __threadfence();
      consumer_sync();
      if (ct == 0) sm.ep.ticket = atomicAdd(p.counters + pc.unit, 1);
      consumer_sync();
      if (sm.ep.ticket == pc.n_pieces - 1) {
        __threadfence();
        const int64_t base = pc.unit * p.max_pieces;
        combine_pieces(p.part_lse + base * kGroupHeads, p.part_o + base * kGroupHeads * kHeadDim, pc.n_pieces, out,
                       warp, lane);
        if (ct == 0) p.counters[pc.unit] = 0;
      }
    }
    consumer_sync();
  }
}

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

struct Plan {
  int64_t n_units, items, total;
  int n_qb, n_ft, n_ctas, max_pieces, unit_aligned;
};

Plan plan(int64_t n_units, int n_groups, int res_cap) {
  Plan s;
  s.n_units = n_units;
  s.n_qb = (n_groups + 1 + kBatchGroups - 1) / kBatchGroups;
  s.n_ft = (res_cap + kTile - 1) / kTile;
  s.items = s.n_qb + s.n_ft;
  s.total = n_units * s.items;
  const int sms = current_device().sm_count > 0 ? current_device().sm_count : 148;
  s.n_ctas = static_cast<int>(s.total < sms ? (s.total > 0 ? s.total : 1) : sms);
  const char* env = getenv("NSA_SPLIT_MODE");
  const int64_t per_cta = (n_units + sms - 1) / sms;
  bool whole = n_units >= sms && (s.items <= 32 || per_cta * sms * 4 <= n_units * 5);
  if (env && env[0] == 's') whole = false;
  if (env && env[0] == 'u' && n_units >= sms) whole = true;
  s.unit_aligned = whole ? 1 : 0;
  if (whole) {
    s.n_ctas = sms;
    s.max_pieces = 1;
  } else {
    int64_t mp = (s.items * s.n_ctas + s.total - 1) / s.total + 1;
    if (mp > s.items) mp = s.items;
    s.max_pieces = static_cast<int>(mp);
  }
  return s;
}

size_t ws_bytes(const Plan& s) {
  const size_t counters = ((s.n_units * sizeof(int)) + 255) & ~size_t(255);
  const size_t pieces = static_cast<size_t>(s.n_units) * s.max_pieces;
  const size_t lse = ((pieces * kGroupHeads * sizeof(float)) + 255) & ~size_t(255);
  return counters + lse + pieces * kGroupHeads * kHeadDim * sizeof(float);
}

int launch(KParams& p, const Plan& s, const void* k_res, const void* v_res, void* ws, size_t wsb,
           cudaStream_t stream) {
  if (s.n_units == 0) return NSA_OK;
  const size_t need = ws_bytes(s);
  if (!ws || wsb < need)
    return fail(NSA_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, ws ? wsb : size_t(0));
  if (!aligned16(ws)) return fail(NSA_ERR_ALIGN, "workspace must be 16-byte aligned");
  uint8_t* w = static_cast<uint8_t*>(ws);
  const size_t counters = ((s.n_units * sizeof(int)) + 255) & ~size_t(255);
  const size_t pieces = static_cast<size_t>(s.n_units) * s.max_pieces;
  const size_t lse = ((pieces * kGroupHeads * sizeof(float)) + 255) & ~size_t(255);
  p.counters = reinterpret_cast<int*>(w);
  p.part_lse = reinterpret_cast<float*>(w + counters);
  p.part_o = reinterpret_cast<float*>(w + counters + lse);
  p.n_units = s.n_units;
  p.n_qb = s.n_qb;
  p.n_ft = s.n_ft;
  p.tiles_per_unit = s.items;
  p.total_tiles = s.total;
  p.n_ctas = s.n_ctas;
  p.unit_aligned = s.unit_aligned;
  p.max_pieces = s.max_pieces;
  p.err = device_error_word();
  if (!p.err) return fail(NSA_ERR_CUDA, "device error word unavailable");

  CUtensorMap mk, mv;
  const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(p.res_cap),
                            static_cast<uint64_t>(s.n_units)};
  const uint64_t strides[2] = {kHeadDim * 2, static_cast<uint64_t>(p.res_cap) * kHeadDim * 2};
  const uint32_t box[3] = {64, kTile, 1};
  int rc = encode_tiled(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, k_res, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tiled(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, v_res, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  const int dev = current_device().device;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kivi_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    attr_set[dev] = true;
  }
  kivi_decode_kernel<<<s.n_ctas, kThreads, kSmemBytes, stream>>>(mk, mv, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "kivi_decode_kernel launch");
}

bool all_aligned(std::initializer_list<const void*> ptrs) {
  for (const void* x : ptrs)
    if (!x || !aligned16(x)) return false;
  return true;
}

}  // namespace

int kivi_check_stream_cache(const nsa_kivi_stream_cache& c) {
  if (c.head_dim != kHeadDim) return fail(NSA_ERR_UNSUPPORTED, "head_dim must be 128");
  if (c.batch < 0 || c.n_kv_heads <= 0) return fail(NSA_ERR_INVALID, "batch >= 0 and n_kv_heads > 0 required");
  if (c.sink < 1 || c.sink > 32) return fail(NSA_ERR_INVALID, "sink must be in [1, 32]");
  if (c.residual < 32 || c.residual % 32) return fail(NSA_ERR_INVALID, "residual must be a positive multiple of 32");
  if (c.window < 0 || (c.window >= c.residual && (c.window - c.residual) % 32))
    return fail(NSA_ERR_INVALID, "window - residual must be a multiple of 32");
  const int64_t ng = c.window >= c.residual ? (c.window - c.residual) / 32 : 0;
  if (c.n_groups != ng) return fail(NSA_ERR_INVALID, "n_groups must be (window - residual) / 32");
  if (!c.unit_lens) return fail(NSA_ERR_INVALID, "unit_lens must not be NULL");
  if (!all_aligned({c.sink_k, c.sink_v, c.k_sink_packed, c.k_sink_scale, c.k_sink_zero, c.v_sink_packed,
                    c.v_sink_scale, c.v_sink_zero, c.k_res, c.v_res}))
    return fail(NSA_ERR_ALIGN, "stream cache tensors must be non-null and 16-byte aligned");
  if (ng > 0 && !all_aligned({c.k_win_packed, c.k_win_scale, c.k_win_zero, c.v_win_packed, c.v_win_scale,
                              c.v_win_zero}))
    return fail(NSA_ERR_ALIGN, "window tensors must be non-null and 16-byte aligned");
  return NSA_OK;
}

}  // namespace nsa

using namespace nsa;

extern "C" {

size_t nsa_kivi_workspace_bytes(int64_t batch, int64_t n_kv_heads, int64_t window, int64_t residual) {
  if (batch < 0 || n_kv_heads <= 0 || window < residual || residual <= 0) return 0;
  return ws_bytes(plan(batch * n_kv_heads, static_cast<int>((window - residual) / 32), static_cast<int>(residual)));
}

int nsa_kivi_decode(const void* q, const void* k_res, const void* v_res, const void* k_sink_packed,
                    const void* k_sink_scale, const void* k_sink_zero, const void* v_sink_packed,
                    const void* v_sink_scale, const void* v_sink_zero, const void* k_win_packed,
                    const void* k_win_scale, const void* k_win_zero, const void* v_win_packed,
                    const void* v_win_scale, const void* v_win_zero, void* o, int64_t batch, int64_t n_heads,
                    int64_t n_kv_heads, int64_t head_dim, int64_t seq_len, int64_t window, int64_t sink,
                    int64_t residual, int64_t group_size, int64_t bits, float sm_scale, void* workspace,
                    size_t workspace_bytes, nsa_stream_t stream) {
  clear_error();
  if (head_dim != kHeadDim) return fail(NSA_ERR_UNSUPPORTED, "head_dim must be 128");
  if (n_kv_heads <= 0 || n_heads != n_kv_heads * kGroupHeads)
    return fail(NSA_ERR_UNSUPPORTED, "n_heads must be 8 * n_kv_heads");
  if (group_size != 32 || bits != 2) return fail(NSA_ERR_UNSUPPORTED, "only group_size=32, bits=2 are implemented");
  if (batch < 0 || seq_len < 0) return fail(NSA_ERR_INVALID, "batch and seq_len must be >= 0");
  if (sink < 1 || sink > 32) return fail(NSA_ERR_UNSUPPORTED, "sink must be in [1, 32] (one padded group)");
  if (residual < 1 || window < residual || (window - residual) % 32)
    return fail(NSA_ERR_INVALID, "need window >= residual >= 1 and (window - residual) %% 32 == 0 "
                                 "(build_quantized_kv_cache's assumption)");
  const int ng = static_cast<int>((window - residual) / 32);
  if (!all_aligned({q, o, k_res, v_res, k_sink_packed, k_sink_scale, k_sink_zero, v_sink_packed, v_sink_scale,
                    v_sink_zero}) ||
      (ng > 0 && !all_aligned({k_win_packed, k_win_scale, k_win_zero, v_win_packed, v_win_scale, v_win_zero})))
    return fail(NSA_ERR_ALIGN, "all tensors must be non-null and 16-byte aligned");
  KParams p{};
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(o);
  p.n_kv_heads = static_cast<int>(n_kv_heads);
  p.layout = 0;
  p.seq_len = seq_len;
  p.window = static_cast<int>(window);
  p.sink = static_cast<int>(sink);
  p.residual = static_cast<int>(residual);
  p.n_groups = ng;
  p.res_cap = static_cast<int>(residual);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.ks_p = static_cast<const uint8_t*>(k_sink_packed);
  p.ks_s = static_cast<const __half*>(k_sink_scale);
  p.ks_z = static_cast<const __half*>(k_sink_zero);
  p.vs_p = static_cast<const uint8_t*>(v_sink_packed);
  p.vs_s = static_cast<const __half*>(v_sink_scale);
  p.vs_z = static_cast<const __half*>(v_sink_zero);
  p.kw_p = static_cast<const uint8_t*>(k_win_packed);
  p.kw_s = static_cast<const __half*>(k_win_scale);
  p.kw_z = static_cast<const __half*>(k_win_zero);
  p.vw_p = static_cast<const uint8_t*>(v_win_packed);
  p.vw_s = static_cast<const __half*>(v_win_scale);
  p.vw_z = static_cast<const __half*>(v_win_zero);
  const Plan s = plan(batch * n_kv_heads, ng, static_cast<int>(residual));
  return launch(p, s, k_res, v_res, workspace, workspace_bytes, stream);
}

size_t nsa_kivi_stream_workspace_bytes(const nsa_kivi_stream_cache* c) {
  if (!c || c->batch < 0 || c->n_kv_heads <= 0 || c->residual <= 0) return 0;
  return ws_bytes(plan(c->batch * c->n_kv_heads, static_cast<int>(c->n_groups), static_cast<int>(c->residual + 32)));
}

int nsa_kivi_stream_decode(const nsa_kivi_stream_cache* cache, const void* q, void* o, float sm_scale,
                           void* workspace, size_t workspace_bytes, nsa_stream_t stream) {
  clear_error();
  if (!cache) return fail(NSA_ERR_INVALID, "null cache");
  const nsa_kivi_stream_cache& c = *cache;
  int rc = kivi_check_stream_cache(c);
  if (rc) return rc;
  if (!all_aligned({q, o})) return fail(NSA_ERR_ALIGN, "q and o must be non-null and 16-byte aligned");
  KParams p{};
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(o);
  p.n_kv_heads = static_cast<int>(c.n_kv_heads);
  p.layout = 1;
  p.unit_lens = c.unit_lens;
  p.window = static_cast<int>(c.window);
  p.sink = static_cast<int>(c.sink);
  p.residual = static_cast<int>(c.residual);
  p.n_groups = static_cast<int>(c.n_groups);
  p.res_cap = static_cast<int>(c.residual + 32);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  p.ks_p = static_cast<const uint8_t*>(c.k_sink_packed);
  p.ks_s = static_cast<const __half*>(c.k_sink_scale);
  p.ks_z = static_cast<const __half*>(c.k_sink_zero);
  p.vs_p = static_cast<const uint8_t*>(c.v_sink_packed);
  p.vs_s = static_cast<const __half*>(c.v_sink_scale);
  p.vs_z = static_cast<const __half*>(c.v_sink_zero);
  p.kw_p = static_cast<const uint8_t*>(c.k_win_packed);
  p.kw_s = static_cast<const __half*>(c.k_win_scale);
  p.kw_z = static_cast<const __half*>(c.k_win_zero);
  p.vw_p = static_cast<const uint8_t*>(c.v_win_packed);
  p.vw_s = static_cast<const __half*>(c.v_win_scale);
  p.vw_z = static_cast<const __half*>(c.v_win_zero);
  const Plan s = plan(c.batch * c.n_kv_heads, static_cast<int>(c.n_groups), static_cast<int>(c.residual + 32));
  return launch(p, s, c.k_res, c.v_res, workspace, workspace_bytes, stream);
}

}  // extern "C"
