// KIVI 2-bit sink + window decode attention (reference: quant_kernel.py
// :316-581) over either the reference's 14-tensor layout or the streaming
// ring layout of nsa_kivi_stream_cache.
//
// Per (batch, kv_head) unit the work is a fixed list of items:
//   F-tiles    64 slots of the fp16 residual (ring), staged by TMA with the
//              128-byte swizzle (F ring, 3 x 32 KiB);
//   Q-batches  up to 6 quantized 32-token groups (slot 0 of batch 0 is the
//              padded sink group, then window groups in physical order),
//              staged with 1-D bulk copies, 3 KiB per group (Q ring, 2 x 18 KiB).
// Items holding no attended token are skipped by every role alike (all derive
// it from the same per-unit metadata).
//
// Warp roles (warp specialization):
//   warp 8      producer: issues the loads of both rings;
//   warps 4-7   dequantizers: each turns whole quantized groups (round-robin)
//               into swizzled fp16 K/V tiles in its own DQ slot, writing
//               zeros for unattended V rows;
//   warps 0-3   MMA warps: consume fp16 tiles -- residual tiles straight from
//               the F ring (warp w takes rows 16w..16w+15) and dequantized
//               groups from the DQ ring (16-token halves round-robin) -- with
//               the shared mma.sync engine, then run the epilogue.
// Dequantization thus overlaps the tensor-core work and the loads instead of
// sitting in front of them.  Every ring has all of its consumers wait on every
// phase, as parity waits require.  Scheduling (whole units per CTA, or
// stream-K with the in-launch combine) is the fp16 kernel's.
#include <cstddef>
#include <cstdlib>

#include "attn_engine.cuh"
#include "host_util.h"

namespace nsa {
namespace {

constexpr int kMmaWarps = 4;
constexpr int kDqWarps = 4;
constexpr int kProducerWarp = kMmaWarps + kDqWarps;
constexpr int kThreads = (kProducerWarp + 1) * 32;
constexpr int kFStages = 3;
constexpr int kQStages = 2;
// One DQ slot per dequantizer: a slot then alternates strictly between its
// own warp's production and the MMA warps' release, so a parity wait on it can
// never be two phases behind (a slot shared by independent producers could).
constexpr int kDqSlots = kDqWarps;
constexpr uint32_t kRegionBytes = kTile * 128;
constexpr uint32_t kTileBytes = 2 * kRegionBytes;
constexpr uint32_t kFStageBytes = 2 * kTileBytes;  // 32 KiB: K + V of 64 slots
constexpr uint32_t kQBytes = kGroupHeads * kHeadDim * 2;
constexpr int kBatchGroups = 6;                    // quantized groups per Q-batch
// Q-batch stage layout (byte offsets); one slot per group
constexpr uint32_t kOffKP = 0, kOffKS = kBatchGroups * 1024, kOffKZ = kOffKS + kBatchGroups * 256,
                   kOffVP = kOffKZ + kBatchGroups * 256, kOffVS = kOffVP + kBatchGroups * 1024,
                   kOffVZ = kOffVS + kBatchGroups * 256;
constexpr uint32_t kQStageBytes = kOffVZ + kBatchGroups * 256;  // 3 KiB per group
constexpr uint32_t kDqRegion = 32 * 128;           // 32 rows x 64 dims fp16
constexpr uint32_t kDqTile = 2 * kDqRegion;        // K (or V) of one group
constexpr uint32_t kDqSlotBytes = 2 * kDqTile;     // K + V, 16 KiB

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

struct QHeader {  // written by the producer into each Q-ring stage
  KiviMeta meta;
  int32_t item;  // Q-batch index within its unit
  int32_t end;   // 1: no more work (sentinel for the dequantizers)
};

struct Smem {
  // copy destinations first: every one stays 16-byte (TMA tiles: 1024-byte) aligned
  uint8_t f[kFStages][kFStageBytes];  // 1024-aligned
  uint8_t dq[kDqSlots][kDqSlotBytes];
  uint8_t qb[kQStages][kQStageBytes];
  uint8_t q[2][kQBytes];
  EpilogueSmem ep;
  QHeader qhdr[kQStages];
  KiviMeta meta[2];
  uint32_t dq_mask[kDqSlots];         // attended tokens of the group in each DQ slot
  uint64_t f_full[kFStages], f_empty[kFStages];
  uint64_t q_full[kQStages], q_empty[kQStages];
  uint64_t dq_full[kDqSlots], dq_empty[kDqSlots];
  uint64_t qv_full[2], qv_empty[2];
};

static_assert(offsetof(Smem, f) % 1024 == 0 && kFStageBytes % 1024 == 0, "TMA tile destinations");
static_assert(offsetof(Smem, qb) % 16 == 0 && kQStageBytes % 16 == 0, "bulk-copy destinations");
static_assert(offsetof(Smem, q) % 16 == 0 && kQBytes % 16 == 0, "bulk-copy destinations");
static_assert(offsetof(Smem, dq) % 128 == 0, "dequantized tiles");

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

__device__ __forceinline__ void lds128(uint32_t a, uint32_t& x, uint32_t& y, uint32_t& z, uint32_t& w) {
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(x), "=r"(y), "=r"(z), "=r"(w) : "r"(a));
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w));
}

// Dequantize one 32-token group (batch slot `slot` of the Q stage at `qs`)
// into the DQ slot at `dst`: K tile [2][32 rows][64 dims] then V tile, both
// swizzled like a TMA tile, rows in token order.  V rows of unattended tokens
// (bit clear in `valid`) are written as zeros so that stale or degenerate
// data (an fp16 zero point that overflowed to inf) cannot reach P.V.
__device__ __forceinline__ void dequant_group(uint32_t qs, int slot, uint32_t dst, uint32_t valid, int lane) {
  const __half2 k1024 = u32_as_h2(0x64006400u);
  {
    // K: lane = (byte row r: tokens 4r..4r+3, channel quarter cq: 32 channels)
    const int r = lane >> 2, cq = lane & 3;
    uint32_t w[8], sc[16], zr[16];
    const uint32_t src = qs + kOffKP + slot * 1024 + r * 128 + 32 * cq;
    lds128(src, w[0], w[1], w[2], w[3]);
    lds128(src + 16, w[4], w[5], w[6], w[7]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lds128(qs + kOffKS + slot * 256 + 64 * cq + 16 * i, sc[4 * i], sc[4 * i + 1], sc[4 * i + 2], sc[4 * i + 3]);
      lds128(qs + kOffKZ + slot * 256 + 64 * cq + 16 * i, zr[4 * i], zr[4 * i + 1], zr[4 * i + 2], zr[4 * i + 3]);
    }
    uint32_t x[16];
    __half2 nz[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      x[i] = __byte_perm(w[i >> 1], 0u, (i & 1) ? 0x4342u : 0x4140u);  // [b_lo, 0, b_hi, 0]
      nz[i] = __hneg2(__hmul2(u32_as_h2(sc[i]), u32_as_h2(zr[i])));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t row = 4 * r + j;
      uint32_t out[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t c = ((x[i] >> (2 * j)) & 0x00030003u) | 0x64006400u;
        out[i] = h2_as_u32(__hfma2(__hsub2(u32_as_h2(c), k1024), u32_as_h2(sc[i]), nz[i]));
      }
      // channels 32cq.. = global chunks 4cq..4cq+3: region cq/2, local chunks (4cq & 7)..
      const uint32_t region = dst + (cq >> 1) * kDqRegion;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc)
        sts128(region + swz128(row, ((4 * cq) & 7) + cc), out[4 * cc], out[4 * cc + 1], out[4 * cc + 2],
               out[4 * cc + 3]);
    }
  }
  {
    // V: lane = token (channels in bytes: byte b holds channels 4b..4b+3)
    const int tau = lane;
    const bool ok = (valid >> tau) & 1u;
    uint32_t w[8];
    const uint32_t src = qs + kOffVP + slot * 1024 + tau * 32;
    lds128(src, w[0], w[1], w[2], w[3]);
    lds128(src + 16, w[4], w[5], w[6], w[7]);
    uint32_t s01, s23, z01, z23;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(s01), "=r"(s23) : "r"(qs + kOffVS + slot * 256 + tau * 8));
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(z01), "=r"(z23) : "r"(qs + kOffVZ + slot * 256 + tau * 8));
    const __half2 sp[2] = {u32_as_h2(s01), u32_as_h2(s23)};
    const __half2 nzp[2] = {__hneg2(__hmul2(sp[0], u32_as_h2(z01))), __hneg2(__hmul2(sp[1], u32_as_h2(z23)))};
    const __half2 quarter_hi = __halves2half2(__float2half_rn(1.f), __float2half_rn(0.25f));
    const uint32_t vdst = dst + kDqTile;
#pragma unroll
    for (int ch = 0; ch < 16; ++ch) {  // 8 channels = bytes 2ch, 2ch+1; group ch / 4
      const int q = ch >> 2;
      const __half2 s = (q & 1) ? __high2half2(sp[q >> 1]) : __low2half2(sp[q >> 1]);
      const __half2 nzq = (q & 1) ? __high2half2(nzp[q >> 1]) : __low2half2(nzp[q >> 1]);
      uint32_t out[4];
#pragma unroll
      for (int bb = 0; bb < 2; ++bb) {
        const int byte = 2 * ch + bb;
        const uint32_t k = byte & 3;
        const uint32_t xb = __byte_perm(w[byte >> 2], 0u, 0x4040u | (k << 8) | k);  // [b, 0, b, 0]
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          // channels 4 byte + 2hh, +1: bits 4hh..+1 (lo) and 4hh+2..+3 (hi, as 4c)
          const uint32_t c = ((xb >> (4 * hh)) & 0x000C0003u) | 0x64006400u;
          const __half2 cv = __hmul2(__hsub2(u32_as_h2(c), k1024), quarter_hi);
          out[2 * bb + hh] = ok ? h2_as_u32(__hfma2(cv, s, nzq)) : 0u;
        }
      }
      sts128(vdst + (ch >> 3) * kDqRegion + swz128(tau, ch & 7), out[0], out[1], out[2], out[3]);
    }
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

__device__ __forceinline__ void mma_warps_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kMmaWarps * 32) : "memory");
}

// Attended-token mask (bit j = token j) of batch slot `slot` of Q-batch `b`.
__device__ __forceinline__ uint32_t group_mask(const KParams& p, const KiviMeta& m, int b, int slot) {
  uint32_t mask = 0;
  const int v = kBatchGroups * b + slot;
  if (v == 0) return m.n_sink >= 32 ? 0xffffffffu : ((1u << m.n_sink) - 1u);
  if (v > p.n_groups) return 0;
  const int age = grp_age(p, m, v - 1);
  if (age >= m.n_grp) return 0;
  const int first = m.tok_skip - 32 * age;  // tokens below this one are not attended
  if (first <= 0) return 0xffffffffu;
  if (first >= 32) return 0;
  mask = ~((1u << first) - 1u);
  return mask;
}

__global__ void __launch_bounds__(kThreads, 1)
    kivi_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const KParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(smem_u32(&sm.f_full[s]), 1);
      mbar_init(smem_u32(&sm.f_empty[s]), kMmaWarps);
    }
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(smem_u32(&sm.q_full[s]), 1);
      mbar_init(smem_u32(&sm.q_empty[s]), kDqWarps);
    }
    for (int s = 0; s < kDqSlots; ++s) {
      mbar_init(smem_u32(&sm.dq_full[s]), 1);
      mbar_init(smem_u32(&sm.dq_empty[s]), kMmaWarps);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&sm.qv_full[s]), 1);
      mbar_init(smem_u32(&sm.qv_empty[s]), kMmaWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      uint32_t nf = 0, nq = 0, nv = 0;  // items issued per ring
      PieceIter it(p);
      Piece pc;
      bool ok = true;
      while (ok && it.next(p, pc)) {
        const int64_t u = pc.unit;
        const KiviMeta meta = make_meta(p, u);
        {
          const uint32_t s = nv % 2, ph = (nv / 2) & 1;
          ++nv;
          if (!mbar_wait(smem_u32(&sm.qv_empty[s]), ph ^ 1, p.err)) break;
          sm.meta[s] = meta;  // published by the arrive below (release)
          mbar_arrive_expect_tx(smem_u32(&sm.qv_full[s]), kQBytes);
          bulk_load(smem_u32(sm.q[s]), p.q + u * kGroupHeads * kHeadDim, kQBytes, smem_u32(&sm.qv_full[s]));
        }
        // Quantized batches first when they all fit in the Q ring (their
        // dequantization then overlaps the residual tiles).  Otherwise the
        // residual tiles go first: the MMA warps consume a piece's residual
        // tiles before its groups, so a producer stuck on a full Q ring must
        // not hold back residual tiles they wait for.
        int live_q = 0;
        for (int64_t t = pc.t_begin; t < pc.t_end; ++t)
          if (t < p.n_qb && item_live(p, meta, static_cast<int>(t))) ++live_q;
        const bool q_first = live_q <= kQStages;
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int64_t t = pc.t_begin; t < pc.t_end; ++t) {
            const int itm = static_cast<int>(t);
            const bool is_q = itm < p.n_qb;
            if (is_q != ((pass == 0) == q_first) || !item_live(p, meta, itm)) continue;
            if (is_q) {
              const uint32_t s = nq % kQStages, ph = (nq / kQStages) & 1;
              ++nq;
              if (!mbar_wait(smem_u32(&sm.q_empty[s]), ph ^ 1, p.err)) { ok = false; break; }
              const uint32_t fb = smem_u32(&sm.q_full[s]);
              const uint32_t sd = smem_u32(sm.qb[s]);
              sm.qhdr[s].meta = meta;
              sm.qhdr[s].item = itm;
              sm.qhdr[s].end = 0;
              const int b = itm;
              const bool has_sink = (b == 0);
              const int p0 = b == 0 ? 0 : kBatchGroups * b - 1;
              const int p1 = min(p.n_groups, kBatchGroups * b + kBatchGroups - 1);
              const int so = p0 + 1 - kBatchGroups * b;  // batch slot of group p0
              const uint32_t ng = p1 > p0 ? p1 - p0 : 0;
              mbar_arrive_expect_tx(fb, (has_sink ? 3072u : 0u) + ng * 3072u);
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
              const uint32_t s = nf % kFStages, ph = (nf / kFStages) & 1;
              ++nf;
              if (!mbar_wait(smem_u32(&sm.f_empty[s]), ph ^ 1, p.err)) { ok = false; break; }
              const uint32_t fb = smem_u32(&sm.f_full[s]);
              const uint32_t sd = smem_u32(sm.f[s]);
              mbar_arrive_expect_tx(fb, kFStageBytes);
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
      if (ok) {
        // sentinel for the dequantizers
        const uint32_t s = nq % kQStages, ph = (nq / kQStages) & 1;
        if (mbar_wait(smem_u32(&sm.q_empty[s]), ph ^ 1, p.err)) {
          sm.qhdr[s].end = 1;
          mbar_arrive(smem_u32(&sm.q_full[s]));
        }
      }
    }
    return;
  }

  if (warp >= kMmaWarps) {
    // ------------------------------------------------------- dequantizers
    const int dw = warp - kMmaWarps;
    uint32_t nq = 0, ng = 0;  // Q stages consumed; live groups seen (all dequant warps count alike)
    for (;;) {
      const uint32_t s = nq % kQStages, ph = (nq / kQStages) & 1;
      ++nq;
      if (!mbar_wait(smem_u32(&sm.q_full[s]), ph, p.err)) return;
      const QHeader hdr = sm.qhdr[s];
      if (hdr.end) return;
      const uint32_t qs = smem_u32(sm.qb[s]);
      for (int slot = 0; slot < kBatchGroups; ++slot) {
        const uint32_t mask = group_mask(p, hdr.meta, hdr.item, slot);
        if (!mask) continue;
        const uint32_t n = ng++;
        if (static_cast<int>(n % kDqWarps) != dw) continue;
        const uint32_t ds = dw, dph = (n / kDqWarps) & 1;
        if (!mbar_wait(smem_u32(&sm.dq_empty[ds]), dph ^ 1, p.err)) return;
        dequant_group(qs, slot, smem_u32(sm.dq[ds]), mask, lane);
        if (lane == 0) sm.dq_mask[ds] = mask;
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.dq_full[ds]));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.q_empty[s]));
    }
  }

  // -------------------------------------------------------------- MMA warps
  // A timed-out wait sets `aborted`: the warp then stops waiting (the error
  // word is already set) but keeps its schedule of named barriers.
  const int g = lane >> 2;
  uint32_t nv = 0, nf = 0, ng = 0, job = 0;
  bool aborted = false;
  WarpAttn st;
  PieceIter it(p);
  Piece pc;
  while (it.next(p, pc)) {
    const uint32_t vs = nv % 2, vph = (nv / 2) & 1;
    ++nv;
    if (!aborted && !mbar_wait(smem_u32(&sm.qv_full[vs]), vph, p.err)) aborted = true;
    st.load_q(smem_u32(sm.q[vs]), lane);
    const KiviMeta meta = sm.meta[vs];
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sm.qv_empty[vs]));
    st.reset();
    // residual tiles first, then the dequantized groups (the producer issued
    // the quantized batches first so their dequantization overlaps)
    for (int64_t t = pc.t_begin; t < pc.t_end; ++t) {
      const int itm = static_cast<int>(t);
      if (itm < p.n_qb || !item_live(p, meta, itm)) continue;
      const uint32_t s = nf % kFStages, ph = (nf / kFStages) & 1;
      ++nf;
      if (!aborted && !mbar_wait(smem_u32(&sm.f_full[s]), ph, p.err)) aborted = true;
      const uint32_t sd = smem_u32(sm.f[s]);
      const int r0 = (itm - p.n_qb) * kTile + 16 * warp;
      const bool v_lo = res_slot_valid(p, meta, r0 + g);
      const bool v_hi = res_slot_valid(p, meta, r0 + g + 8);
      if (__any_sync(0xffffffffu, v_lo || v_hi)) {
        zero_invalid_v_rows(sd + kTileBytes, kRegionBytes, 16 * warp, v_lo, v_hi, lane);
        st.consume16(sd, sd + kTileBytes, kRegionBytes, 16 * warp, v_lo, v_hi, p.scale_log2, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.f_empty[s]));
    }
    for (int64_t t = pc.t_begin; t < pc.t_end; ++t) {
      const int itm = static_cast<int>(t);
      if (itm >= p.n_qb || !item_live(p, meta, itm)) continue;
      for (int slot = 0; slot < kBatchGroups; ++slot) {
        if (!group_mask(p, meta, itm, slot)) continue;
        const uint32_t n = ng++;
        const uint32_t ds = n % kDqWarps, dph = (n / kDqWarps) & 1;  // group n is in its dequantizer's slot
        if (!aborted && !mbar_wait(smem_u32(&sm.dq_full[ds]), dph, p.err)) aborted = true;
        const uint32_t mask = sm.dq_mask[ds];
        const uint32_t dbase = smem_u32(sm.dq[ds]);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t hm = (mask >> (16 * hf)) & 0xffffu;
          if (!hm) continue;
          if ((job++ % kMmaWarps) != static_cast<uint32_t>(warp)) continue;
          st.consume16(dbase, dbase + kDqTile, kDqRegion, 16 * hf, (hm >> g) & 1u, (hm >> (g + 8)) & 1u,
                       p.scale_log2, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&sm.dq_empty[ds]));
      }
    }

    // ---- epilogue: merge the 4 MMA warps, write the output or a partial
    warp_publish(st, sm.ep, warp, lane);
    mma_warps_sync();
    const int ct = threadIdx.x;  // 0..127
    const int hh = ct >> 4, d0 = (ct & 15) * 8;
    float o[8], lse;
    {
      float o4[4];
      merge_warps(sm.ep, hh, d0, o4, lse);
      for (int i = 0; i < 4; ++i) o[i] = o4[i];
      merge_warps(sm.ep, hh, d0 + 4, o4, lse);
      for (int i = 0; i < 4; ++i) o[4 + i] = o4[i];
    }
    __half* out = p.o + pc.unit * kGroupHeads * kHeadDim;
    if (pc.n_pieces == 1) {
      const float a[4] = {o[0], o[1], o[2], o[3]}, b[4] = {o[4], o[5], o[6], o[7]};
      store_half4(out + hh * kHeadDim + d0, a);
      store_half4(out + hh * kHeadDim + d0 + 4, b);
    } else {
      const int64_t pidx = pc.unit * p.max_pieces + pc.slot;
      float* po = p.part_o + (pidx * kGroupHeads + hh) * kHeadDim + d0;
      reinterpret_cast<float4*>(po)[0] = make_float4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<float4*>(po)[1] = make_float4(o[4], o[5], o[6], o[7]);
      if ((ct & 15) == 0) p.part_lse[pidx * kGroupHeads + hh] = lse;
      __threadfence();
      mma_warps_sync();
      if (ct == 0) sm.ep.ticket = atomicAdd(p.counters + pc.unit, 1);
      mma_warps_sync();
      if (sm.ep.ticket == pc.n_pieces - 1) {
        __threadfence();
        const int64_t base = pc.unit * p.max_pieces;
        combine_pieces(p.part_lse + base * kGroupHeads, p.part_o + base * kGroupHeads * kHeadDim, pc.n_pieces, out,
                       warp * (kGroupHeads / kMmaWarps), kGroupHeads / kMmaWarps, lane);
        if (ct == 0) p.counters[pc.unit] = 0;
      }
    }
    mma_warps_sync();
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
