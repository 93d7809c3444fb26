// KIVI 2-bit sink + window decode attention (reference: quant_kernel.py
// :316-581) over either the reference's 14-tensor layout or the streaming
// ring layout of nsa_kivi_stream_cache.
//
// Work: one CTA per piece, two CTAs per SM.  A piece is one unit (batch row,
// KV head) -- or, for long windows with fewer units than CTA slots, a
// contiguous part of the unit's items, merged by the split-K combine (units
// whose items all fit the stages keep one CTA at any batch).  With every unit
// resident at once, all of a launch's loads are in flight from the start.  Per unit the
// items, in issue and consumption order, are: Q-batch 0, the F-tiles, the
// other Q-batches, where
//   Q-batch    up to 5 quantized 32-token groups (slot 0 of batch 0 is the
//              padded sink group, then window groups in physical order), staged
//              raw -- codes, scales, zero points -- 3 KiB per group (Q ring,
//              2 x 15 KiB);
//   F-tile     80 slots of the fp16 residual ring, K and V (F ring, 2 x 40 KiB).
// Staging depends on the layout (Lay): the streaming cache keeps each group's
// six tensors in one record and its residual slots chunk-permuted
// (kivi_format.cuh), so a Q-batch is ONE 1-D bulk copy and an F-tile one copy
// each of K and V, landing bank-conflict free; the reference's separate
// tensors take six bulk copies per Q-batch (one per tensor) and a TMA box per
// F-tile (both 64-dim halves, 128-byte swizzle).
// Batch 0 carries most of the arithmetic, so it is loaded and consumed first
// and its dequantization overlaps the residual's transfer.  Every copy request
// costs a fixed issue time (about 40 ns on B200) whatever its size, so loads
// are few and large, and those that do not depend on the unit's length (query,
// batch 0, residual) are issued before that length is read -- except, in a
// one-layer streaming launch, the second F-tile, which waits for the length so
// that batch 0 and the first F-tile of every unit arrive first.  Q-batches
// after the first that hold no attended token are skipped by every warp alike.
//
// Warps 0-3 consume, each claiming the next job of the staged item (a
// quantized group, or 32 rows of an F-tile) from a shared-memory counter as
// soon as it is free, so the work follows the warps' real progress (the
// order in which a unit's partial sums accumulate, and so the output's last
// rounding, can differ between launches; the cache state cannot); lane 0 of
// warp 0 also issues the loads.  With no separate producer warp, a CTA is 4
// warps and two CTAs per SM leave up to 255 registers per thread, which the
// dequantization's independent chains need to overlap.  A quantized group is dequantized in
// registers straight into mma.sync fragments, with no shared-memory round trip:
//   K  S^T = (C - Z) (s*Q)^T: the per-channel scale s is folded into the query
//      once per group; C (2-bit codes as exact fp16 integers, made with the
//      1024-style magic-number trick) is the A operand; the zero-point term
//      Z (s*Q)^T is one mma chain whose A rows all equal z, computed once per
//      group and used as the initial score.  The mma's k index is permuted so
//      that each lane's codes are whole bytes of one packed row (the query
//      fragments are permuted to match), and the mma's rows are a fixed
//      permutation of the group's tokens so that a lane's two rows share a byte.
//   V  O^T += (C - Z)^T (P*s)^T per 32-channel group: c - z is exact for the
//      integer zero points, and the per-token scale is folded into the P
//      fragment of each channel group (one rounding, as in an fp16
//      dequantization of the cache).
// F-tiles go through the shared fp16 engine (consume_rows).
#include <cstddef>
#include <cstdlib>

#include "attn_engine.cuh"
#include "host_util.h"
#include "kivi_format.cuh"
#include "quant_math.cuh"

namespace nsa {
namespace {

constexpr int kCWarps = 4;                 // consumer warps (warp 0, lane 0 also issues the loads)
constexpr int kThreads = kCWarps * 32;
constexpr int kCtasPerSm = 2;
constexpr int kFRows = 80;                 // residual slots per F-tile
constexpr uint32_t kFRegion = kFRows * 128;  // 80 rows x 64 dims fp16
constexpr uint32_t kFTile = 2 * kFRegion;    // K (or V) of one F-tile: one TMA box
constexpr uint32_t kFStageBytes = 2 * kFTile;  // 40 KiB
constexpr int kFStages = 2;
constexpr int kQStages = 2;
constexpr int64_t kMaxUnitLen = int64_t(1) << 30;  // longest unit the kernels accept
constexpr int kBatchGroups = 5;            // quantized groups per Q-batch
constexpr int kQPadStride = kHeadDim + 8;  // 272-byte rows: 8 rows of an ldmatrix hit distinct banks
// Q-batch stage layout (byte offsets); one slot per group
constexpr uint32_t kOffKP = 0, kOffKS = kBatchGroups * 1024, kOffKZ = kOffKS + kBatchGroups * 256,
                   kOffVP = kOffKZ + kBatchGroups * 256, kOffVS = kOffVP + kBatchGroups * 1024,
                   kOffVZ = kOffVS + kBatchGroups * 256;
constexpr uint32_t kQStageBytes = kOffVZ + kBatchGroups * 256;  // 3 KiB per group
static_assert(kQStageBytes == kBatchGroups * kRecBytes, "a Q stage holds 5 group records");

// Staging of one cache layout.  kRec: the streaming cache (group records, a
// batch one bulk copy, record-major Q stage; chunk-permuted residual rows, an
// F-tile one bulk copy each of K and V, 256-byte rows in shared memory).
// Otherwise the reference's separate tensors (field-major Q stage, six bulk
// copies per batch; F-tiles by TMA boxes, two 128-byte-swizzled regions).
template <bool kRec>
struct Lay {
  static constexpr uint32_t kRowBytes = kRec ? 256 : 128;
  static constexpr uint32_t kRegion = kRec ? 128 : kFRegion;
  // Q stage: byte offsets of batch slot gs's fields
  static __device__ __forceinline__ uint32_t kp(int gs) { return kRec ? gs * kRecBytes + kRecKP : gs * 1024; }
  static __device__ __forceinline__ uint32_t ks(int gs) { return kRec ? gs * kRecBytes + kRecKS : kOffKS + gs * 256; }
  static __device__ __forceinline__ uint32_t kz(int gs) { return kRec ? gs * kRecBytes + kRecKZ : kOffKZ + gs * 256; }
  static __device__ __forceinline__ uint32_t vp(int gs) { return kRec ? gs * kRecBytes + kRecVP : kOffVP + gs * 1024; }
  static __device__ __forceinline__ uint32_t vs(int gs) { return kRec ? gs * kRecBytes + kRecVS : kOffVS + gs * 256; }
  static __device__ __forceinline__ uint32_t vz(int gs) { return kRec ? gs * kRecBytes + kRecVZ : kOffVZ + gs * 256; }
  // F-tile (K at 0, V at kFTile): (row, 16-byte chunk 0..15)
  static __device__ __forceinline__ uint32_t f(uint32_t row, uint32_t chunk) {
    return tile_off<kRowBytes>(row, chunk, kRegion);
  }
};

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
  union {
    uint8_t f[kFStages][kFStageBytes];  // 1024-aligned TMA tile destinations
    EpilogueSmem ep;                    // reused once every item has been consumed
  };
  uint8_t qb[kQStages][kQStageBytes];
  __half qpad[kGroupHeads][kQPadStride];  // the unit's query, rows padded: conflict-free fragment loads
  __half newtok[2][kHeadDim];             // appended token's K and V (fused append)
  uint64_t f_full[kFStages], f_empty[kFStages];
  uint64_t q_full[kQStages], q_empty[kQStages];
  int q_rel[kQStages];  // warps that have released the stage's current Q-batch
  int f_job[kFStages], q_job[kQStages], d_job;  // next job of the staged item (claimed by warps)
};

static_assert(offsetof(Smem, f) == 0 && kFStageBytes % 1024 == 0 && kFRegion % 1024 == 0, "TMA tile destinations");
static_assert(offsetof(Smem, qb) % 16 == 0 && kQStageBytes % 16 == 0, "bulk-copy destinations");
static_assert(offsetof(Smem, qpad) % 16 == 0 && (kQPadStride * 2) % 16 == 0, "16-byte stores");
static_assert(sizeof(EpilogueSmem) <= sizeof(uint8_t[kFStages][kFStageBytes]), "epilogue alias");
// The dynamic shared-memory window of a CTA starts 1024-byte aligned on sm_100
// (the kernel checks it); 1 KiB per CTA is reserved by the system.
constexpr size_t kSmemBytes = sizeof(Smem);
static_assert(kCtasPerSm * (kSmemBytes + 1024) <= 228 * 1024, "two CTAs per SM");

struct KParams {
  const __half* q;
  __half* o;
  int64_t n_units;
  int n_kv_heads;
  int layout;  // 0: reference 14-tensor layout; 1: streaming ring
  int64_t seq_len;
  int64_t* unit_lens;
  int window, sink, residual, n_groups, res_cap;
  int n_qb, n_ft, items;  // items per unit: Q-batch 0, n_ft F-tiles, Q-batches 1 .. n_qb-1
  int ppu;                // pieces (CTAs) per unit
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
  uint8_t* grp;  // stream layout: group records (kivi_format.cuh)
  int* counters;
  float* part_lse;
  float* part_o;
  int* err;
  // fused quantize-on-append (stream layout, one CTA per unit); new_k == null:
  // attention only.  The cache arrays above are then also written.
  const __half* new_k;
  const __half* new_v;
  __half* k_res;
  __half* v_res;
  __half* sink_k16;
  __half* sink_v16;
};

// Per-unit metadata from the unit's length (see nsa_kivi_stream_cache and
// _kv_indices, sparse_kernel.py:15-46, for the two layouts); `len` is the
// streaming unit's length (unused for the reference layout).
template <bool kRec>
__device__ __forceinline__ KiviMeta make_meta(const KParams& p, int len_stream) {
  // 32-bit arithmetic: lengths stay below kMaxUnitLen (checked where read)
  KiviMeta m;
  const int S = p.sink, W = p.window, R = p.residual, NG = p.n_groups;
  if constexpr (!kRec) {
    const int len = static_cast<int>(p.seq_len);  // the host caps it at kMaxUnitLen
    const int nw = W - R;                          // window-old tokens
    const int n_inv = min(max(S - len + W, 0), W);  // window indices < n_inv are not attended
    m.n_sink = min(max(len, 0), S);
    m.grp_head = 0;
    m.n_grp = NG;
    m.tok_skip = min(n_inv, nw);
    m.res_head = 0;
    m.n_res = R;
    m.res_skip = min(max(n_inv - nw, 0), R);
  } else {
    const int len = len_stream;
    const int C = p.res_cap;
    const int n_stream = len > S ? len - S : 0;
    const int F = n_stream > R ? (n_stream - R) >> 5 : 0;  // flushed groups
    const int first = max(len - W, S);                     // oldest attended position
    m.n_sink = min(len, S);
    m.n_res = n_stream - 32 * F;
    m.res_head = (32 * F) % C;
    m.res_skip = min(max(first - S - 32 * F, 0), m.n_res);
    m.n_grp = min(F, NG);
    m.grp_head = NG > 0 ? (F - m.n_grp) % NG : 0;
    m.tok_skip = min(max(first - S - 32 * (F - m.n_grp), 0), 32 * m.n_grp);
  }
  m.pad = 0;
  return m;
}

// Distance of window-group slot gp from the oldest live group (>= n_grp: dead).
__device__ __forceinline__ int grp_age(const KParams& p, const KiviMeta& m, int gp) {
  int d = gp - m.grp_head;
  if (d < 0) d += p.n_groups;
  return d;
}

// Attended-token mask (bit j = token j) of batch slot `slot` of Q-batch `b`.
__device__ __forceinline__ uint32_t group_mask(const KParams& p, const KiviMeta& m, int b, int slot) {
  const int v = kBatchGroups * b + slot;
  if (v == 0) return m.n_sink >= 32 ? 0xffffffffu : ((1u << m.n_sink) - 1u);
  if (v > p.n_groups) return 0;
  const int age = grp_age(p, m, v - 1);
  if (age >= m.n_grp) return 0;
  const int first = m.tok_skip - 32 * age;  // tokens below this one are not attended
  if (first <= 0) return 0xffffffffu;
  if (first >= 32) return 0;
  return ~((1u << first) - 1u);
}

// Attended residual slots r0 .. r0 + 31 as a mask (bit i: slot r0 + i),
// computed with warp-uniform integer arithmetic: a slot below res_cap sits
// d = (slot - res_head) mod res_cap from the oldest live slot and is attended
// iff res_skip <= d < n_res; slots from res_cap on do not exist.
__device__ __forceinline__ uint32_t res_slot_mask(const KParams& p, const KiviMeta& m, int r0) {
  const int C = p.res_cap;
  int a = r0 - m.res_head;  // d of slot r0 (before the wrap below)
  if (a < 0) a += C;
  uint32_t mk = bit_range(m.res_skip - a, m.n_res - a) & bit_range(0, C - a);  // d = a + i
  mk |= bit_range(m.res_skip + C - a, m.n_res + C - a) & bit_range(C - a, 32);  // d = a + i - C
  return mk & bit_range(0, C - r0);  // slots >= res_cap do not exist
}

// Physical residual slots [lo, hi) covering the attended ones within slots
// [a, b) (lo >= hi: none).  The attended slots are the ring segment of
// n_res - res_skip slots from res_head + res_skip; within [a, b) it is one
// run, or two when it wraps there (then the cover spans the gap as well).
__device__ __forceinline__ void attended_cover(const KParams& p, const KiviMeta& m, int a, int b, int& lo, int& hi) {
  const int C = p.res_cap, n = m.n_res - m.res_skip;
  int s0 = m.res_head + m.res_skip;
  if (s0 >= C) s0 -= C;
  lo = b;
  hi = a;
  if (n <= 0) return;
  int x = max(s0, a), y = min(min(s0 + n, C), b);
  if (x < y) {
    lo = x;
    hi = y;
  }
  y = min(s0 + n - C, b);  // the wrapped part [0, s0 + n - C)
  if (a < y) {
    lo = min(lo, a);
    hi = max(hi, y);
  }
}

// Whether Q-batch b holds any attended token.  Batch 0 counts as live always:
// its sink group is loaded before the unit's length is known.
__device__ __forceinline__ bool batch_live(const KParams& p, const KiviMeta& m, int b) {
  if (b == 0) return true;
  // a full ring whose oldest group still holds an attended token: every slot is live
  if (m.n_grp == p.n_groups && m.tok_skip < 32) return kBatchGroups * b <= p.n_groups;
  for (int s = 0; s < kBatchGroups; ++s)
    if (group_mask(p, m, b, s)) return true;
  return false;
}

// Dynamic job assignment: the jobs of a staged item (the groups of a
// Q-batch, the 32-row slices of an F-tile) are claimed in order from a
// shared-memory counter by whichever warp is free first; lane 0 claims for
// its warp.  The counter is reset when the stage is refilled (after every
// warp has released it, before the refill's barrier arrival publishes it).
constexpr int kFJobs = (kFRows + 31) / 32;
__device__ __forceinline__ int claim_job(int* counter, int lane) {
  int j = 0;
  if (lane == 0) j = atomicAdd(counter, 1);
  return __shfl_sync(0xffffffffu, j, 0);
}

// ---------------------------------------------------------------- registers
__device__ __forceinline__ __half2 u32_as_h2(uint32_t x) { return *reinterpret_cast<__half2*>(&x); }
__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ uint32_t hsub2u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hsub2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t hmul2u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t hadd2u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hadd2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ void lds128(uint32_t a, uint32_t& x, uint32_t& y, uint32_t& z, uint32_t& w) {
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(x), "=r"(y), "=r"(z), "=r"(w) : "r"(a));
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w));
}
__device__ __forceinline__ void lds64(uint32_t a, uint32_t& x, uint32_t& y) {
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(x), "=r"(y) : "r"(a));
}

// fp16 2^(10 - 2j) in both halves: OR-ing 2-bit field j of a byte (bits 2j,
// 2j+1 of the half's low byte, whose weight at that exponent is 1) into it
// gives 2^(10-2j) + code exactly; subtracting it again leaves the code.
__device__ __forceinline__ uint32_t magic2(int j) { return 0x64006400u - static_cast<uint32_t>(j) * 0x08000800u; }

// Per-lane constants of the quantized path (g = lane / 4, t = lane % 4).
struct LaneQ {
  uint32_t mk_lo, mg_lo, mk_hi, mg_hi;  // K: code fields of rows g / g+8 within their byte
  uint32_t mv, mgv, selv;               // V: code field of dims = g (mod 4), byte selector
  int tau_lo, tau_hi;                   // tokens (within a 16-token half) of mma rows g, g+8
  int tv[4];                            // tokens of the P^T k-rows 2t, 2t+1, 2t+8, 2t+9
  __device__ __forceinline__ explicit LaneQ(int lane) {
    const int g = lane >> 2, t = lane & 3;
    // mma row rho = g' + 8h (g' < 8) holds token 4*(g'/2) + ((g'/2 + g'%2 + 2h) % 4):
    // rows g and g+8 share packed K byte row g/2, and the four tokens of a
    // lane's P^T fragment are byte row t's, each once.
    const int jlo = ((g >> 1) + (g & 1)) & 3, jhi = (jlo + 2) & 3;
    mk_lo = 0x00030003u << (2 * jlo);
    mg_lo = magic2(jlo);
    mk_hi = 0x00030003u << (2 * jhi);
    mg_hi = magic2(jhi);
    tau_lo = 4 * (g >> 1) + jlo;
    tau_hi = 4 * (g >> 1) + jhi;
    mv = 0x00030003u << (2 * (g & 3));
    mgv = magic2(g & 3);
    selv = (g >> 2) ? 0x7531u : 0x6420u;
#pragma unroll
    for (int k = 0; k < 4; ++k) tv[k] = 4 * t + ((t + k) & 3);
  }
};

// Channels of lane t (t = lane % 4) on the K side: [16t, 16t+16) and
// [64+16t, 64+16t+16); 16-byte chunk i (8 channels) of them starts at byte
// chunk_off(i) + 32t of a channel-major fp16 row (codes: + 16t of a byte row).
// This spreads the four t's over distinct banks for every load.
__device__ __forceinline__ uint32_t chunk_off(int i) { return (i >> 1) * 128 + (i & 1) * 16; }

// Attend to the attended tokens (`mask`) of the quantized group in batch slot
// `gs` of the Q stage at `qs`.  qrow: this lane's query row Q[head g] + 32t
// bytes in shared memory (chunks at chunk_off).
template <bool kRec>
__device__ __forceinline__ void attend_group(WarpAttn& st, uint32_t qrow, const LaneQ& lq, uint32_t qs, int gs,
                                             uint32_t mask, float scale_log2, int lane) {
  const int g = lane >> 2, t = lane & 3;
  // ---- per group: query scaled by the K scales, zero-point term, permuted B-fragments
  uint32_t qp[8][2];
  float zb0, zb1;  // sum_d z_d * s_d * Q[h][d] for heads 2t, 2t+1
  {
    uint32_t sq[16], zn[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t s0, s1, s2, s3, q0, q1, q2, q3;
      lds128(qs + Lay<kRec>::ks(gs) + 32 * t + chunk_off(i), s0, s1, s2, s3);
      lds128(qrow + chunk_off(i), q0, q1, q2, q3);
      sq[4 * i] = hmul2u(q0, s0);
      sq[4 * i + 1] = hmul2u(q1, s1);
      sq[4 * i + 2] = hmul2u(q2, s2);
      sq[4 * i + 3] = hmul2u(q3, s3);
      lds128(qs + Lay<kRec>::kz(gs) + 32 * t + chunk_off(i), zn[4 * i], zn[4 * i + 1], zn[4 * i + 2],
             zn[4 * i + 3]);
    }
    float zc[4] = {0.f, 0.f, 0.f, 0.f}, zc2[4] = {0.f, 0.f, 0.f, 0.f};  // two chains: half the mma latency
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      // natural k order: k-cols (2t, 2t+1) = the lane's channels 4kk+{0,1}, (2t+8, 2t+9) = +{2,3}
      mma_16816((kk & 1) ? zc2 : zc, zn[2 * kk], zn[2 * kk], zn[2 * kk + 1], zn[2 * kk + 1], sq[2 * kk],
                sq[2 * kk + 1]);
      // permuted k order of the code fragments: (2t, 2t+1) = +{0,2}, (2t+8, 2t+9) = +{1,3}
      qp[kk][0] = __byte_perm(sq[2 * kk], sq[2 * kk + 1], 0x5410);
      qp[kk][1] = __byte_perm(sq[2 * kk], sq[2 * kk + 1], 0x7632);
    }
    zb0 = zc[0] + zc2[0];
    zb1 = zc[1] + zc2[1];
  }
  // ---- S^T = C.(sQ)^T - z.(sQ)^T for both 16-token halves at once (four
  // independent mma chains); a half without attended tokens is computed too
  // (its rows are masked) -- its codes are real, finite data
  const uint32_t hm[2] = {mask & 0xffffu, mask >> 16};
  float s[2][4], s2[2][4];
  {
    uint32_t kw[2][8];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      s[hf][0] = s[hf][2] = -zb0;
      s[hf][1] = s[hf][3] = -zb1;
      s2[hf][0] = s2[hf][1] = s2[hf][2] = s2[hf][3] = 0.f;
      const uint32_t src = qs + Lay<kRec>::kp(gs) + (4 * hf + (g >> 1)) * 128 + 16 * t;
      lds128(src, kw[hf][0], kw[hf][1], kw[hf][2], kw[hf][3]);
      lds128(src + 64, kw[hf][4], kw[hf][5], kw[hf][6], kw[hf][7]);
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const uint32_t w = kw[hf][kk], wh = w >> 8;  // bytes: the lane's channels 4kk+{0,1,2,3}
        const uint32_t a0 = hsub2u((w & lq.mk_lo) | lq.mg_lo, lq.mg_lo);
        const uint32_t a1 = hsub2u((w & lq.mk_hi) | lq.mg_hi, lq.mg_hi);
        const uint32_t a2 = hsub2u((wh & lq.mk_lo) | lq.mg_lo, lq.mg_lo);
        const uint32_t a3 = hsub2u((wh & lq.mk_hi) | lq.mg_hi, lq.mg_hi);
        mma_16816((kk & 1) ? s2[hf] : s[hf], a0, a1, a2, a3, qp[kk][0], qp[kk][1]);
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[hf][c] += s2[hf][c];
  }
  uint32_t pb[2][2];
  {
    const bool vlo[2] = {((hm[0] >> lq.tau_lo) & 1u) != 0, ((hm[1] >> lq.tau_lo) & 1u) != 0};
    const bool vhi[2] = {((hm[0] >> lq.tau_hi) & 1u) != 0, ((hm[1] >> lq.tau_hi) & 1u) != 0};
    st.softmax_rows<2>(s, vlo, vhi, scale_log2, pb);
  }

  // ---- O^T += (C - Z)^T.(P*s)^T: channel group G = m-tiles 2G, 2G+1
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    if (!hm[hf]) continue;
    const uint32_t vrow = qs + Lay<kRec>::vp(gs) + 16 * hf * 32;
    uint32_t vs[4][2], vz[4][2];  // scales / zero points of tokens tv[k], channel groups (0,1), (2,3)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int tok = 16 * hf + lq.tv[k];
      lds64(qs + Lay<kRec>::vs(gs) + tok * 8, vs[k][0], vs[k][1]);
      lds64(qs + Lay<kRec>::vz(gs) + tok * 8, vz[k][0], vz[k][1]);
    }
    // unattended tokens: scale and zero 0, so that their terms are exactly 0
    // whatever the stored values (P is 0 there; this keeps inf / NaN out of P.V)
    bool all_ok = true;
#pragma unroll
    for (int k = 0; k < 4; ++k) all_ok &= ((hm[hf] >> lq.tv[k]) & 1u) != 0;
    if (!__all_sync(0xffffffffu, all_ok)) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (!((hm[hf] >> lq.tv[k]) & 1u)) vs[k][0] = vs[k][1] = vz[k][0] = vz[k][1] = 0u;
    }
    uint32_t p01[4], p23[4], z01[4], z23[4];
#pragma unroll
    for (int G = 0; G < 4; ++G) {
      // pb[hf][0] holds P of tokens tv[0], tv[1] (k-rows 2t, 2t+1), pb[hf][1] of tv[2], tv[3]
      const uint32_t sel = (G & 1) ? 0x7632u : 0x5410u;
      p01[G] = hmul2u(pb[hf][0], __byte_perm(vs[0][G >> 1], vs[1][G >> 1], sel));
      p23[G] = hmul2u(pb[hf][1], __byte_perm(vs[2][G >> 1], vs[3][G >> 1], sel));
      z01[G] = hadd2u(__byte_perm(vz[0][G >> 1], vz[1][G >> 1], sel), lq.mgv);
      z23[G] = hadd2u(__byte_perm(vz[2][G >> 1], vz[3][G >> 1], sel), lq.mgv);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // m-tiles 4*half .. +3 = packed bytes 16*half .. +15
      uint32_t vw[4][4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        lds128(vrow + lq.tv[k] * 32 + 16 * half, vw[k][0], vw[k][1], vw[k][2], vw[k][3]);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = 4 * half + jj, G = j >> 1;
        // word jj: bytes 4j..4j+3 = dims 16j..16j+15; dim 16j+g is byte g/4 field g%4, dim 16j+g+8 byte 2+g/4
        const uint32_t x01 = __byte_perm(vw[0][jj], vw[1][jj], lq.selv);
        const uint32_t x23 = __byte_perm(vw[2][jj], vw[3][jj], lq.selv);
        // A = c - z (exact): (magic + c) - (magic + z)
        const uint32_t a0 = hsub2u((x01 & lq.mv) | lq.mgv, z01[G]);
        const uint32_t a1 = hsub2u(((x01 >> 8) & lq.mv) | lq.mgv, z01[G]);
        const uint32_t a2 = hsub2u((x23 & lq.mv) | lq.mgv, z23[G]);
        const uint32_t a3 = hsub2u(((x23 >> 8) & lq.mv) | lq.mgv, z23[G]);
        mma_16816(st.acc[j], a0, a1, a2, a3, p01[G], p23[G]);
      }
    }
  }
}

// Zero the V rows of slots that are not attended, so stale or
// uninitialised cache memory (possibly NaN) cannot reach the P.V product.
template <bool kRec>
__device__ __forceinline__ void zero_invalid_v_rows(uint32_t vbase, int row0, bool v_lo, bool v_hi, int lane) {
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
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vbase + Lay<kRec>::f(row, chunk)), "r"(0u));
    }
  }
  fence_proxy_async_smem();  // the stage is refilled by the async proxy later
  __syncwarp();
}

__device__ __forceinline__ void cwarps_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory"); }

// ------------------------------------------------------- fused append
// Quantize-on-append inside the decode launch (stream layout, one CTA per
// unit): the same bit-exact arithmetic and cache layout as kivi_append_kernel
// in kivi_quant.cu, which it replaces for such launches.  Its results also go
// into the staged copies this launch attends over.
__device__ __forceinline__ void sts8(uint32_t a, uint32_t v) { asm volatile("st.shared.u8 [%0], %1;" ::"r"(a), "r"(v)); }
__device__ __forceinline__ void sts16(uint32_t a, __half v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"(__half_as_ushort(v)));
}
__device__ __forceinline__ void sts64(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(a), "r"(x), "r"(y));
}

struct AppendPlan {
  bool sink = false;    // the appended token is a sink token: the sink group is re-quantized
  int f_item = -1;      // F-tile and row holding the appended token's residual slot (-1: none)
  int f_row = 0;
  int fl_batch = -1;    // Q-batch and batch slot of the window group this append flushes (-1: none)
  int fl_slot = 0;
  int fl_gs = 0;        // its window-group slot
  int fl_base = 0;      // stream index of its first token
  int fl_s0 = -1;       // its first residual slot (-1: no flush)
  __device__ __forceinline__ bool flushing(int slot) const { return fl_s0 >= 0 && slot >= fl_s0 && slot < fl_s0 + 32; }
};

// Where the append lands; pos = the unit's length before the append.  (The
// token's own stores wait until its value is needed, so that no thread
// stalls on its load early in the launch.)
__device__ __forceinline__ AppendPlan append_plan(const KParams& p, int pos) {
  AppendPlan a;
  const int S = p.sink, R = p.residual, C = p.res_cap, NG = p.n_groups;
  if (pos < S) {
    a.sink = true;
    return a;
  }
  const int i = pos - S;  // stream index
  const int slot = i % C;
  a.f_item = slot / kFRows;
  a.f_row = slot % kFRows;
  if (i + 1 - R > 0 && ((i + 1 - R) & 31) == 0 && NG > 0) {  // stream group f_old leaves the residual
    const int f_old = (i - R) >> 5;
    a.fl_gs = f_old % NG;
    a.fl_base = 32 * f_old;
    a.fl_batch = (a.fl_gs + 1) / kBatchGroups;
    a.fl_slot = (a.fl_gs + 1) % kBatchGroups;
    a.fl_s0 = a.fl_base % C;
  }
  return a;
}

// Copy the appended token (K and V rows of `tok`) into the staged F-tile at
// `row`, by one warp: lane l moves 16 bytes (8 channels) of K (l < 16) or V.
__device__ __forceinline__ void patch_residual_row(uint32_t sd, int row, uint32_t tok, int lane) {
  const int kv = lane >> 4, chunk = lane & 15;  // chunk: 8 channels
  uint32_t x, y, z, w;
  lds128(tok + kv * kHeadDim * 2 + chunk * 16, x, y, z, w);
  sts128(sd + kv * kFTile + Lay<true>::f(row, chunk), x, y, z, w);
  fence_proxy_async_smem();
  __syncwarp();
}

// One group record (K of channel c, V of token c/4 x channel group c%4) from
// the group's 32 K values of channel c and 32 V values of its token and
// channel group: into Q-stage slot `sl` at `qs` and to the cache record `rec`.
__device__ __forceinline__ void store_group_record(const float (&x)[32], const float (&y)[32], uint32_t qs, int sl,
                                                   const GroupRec& rec, int c) {
  using L = Lay<true>;
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    mn = fminf(mn, x[j]);
    mx = fmaxf(mx, x[j]);
  }
  GroupParams gp = group_params(mn, mx);
  const __half hs = __float2half_rn(gp.scale), hz = __float2half_rn(gp.zero);
  rec.ks[c] = hs;
  rec.kz[c] = hz;
  sts16(qs + L::ks(sl) + c * 2, hs);
  sts16(qs + L::kz(sl) + c * 2, hz);
#pragma unroll
  for (int bq = 0; bq < 8; ++bq) {
    uint32_t byte = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) byte |= code_of(x[4 * bq + j], gp) << (2 * j);
    rec.kp[bq * kHeadDim + c] = static_cast<uint8_t>(byte);
    sts8(qs + L::kp(sl) + bq * kHeadDim + c, byte);
  }
  const int tok = c >> 2, q = c & 3;
  mn = INFINITY;
  mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    mn = fminf(mn, y[j]);
    mx = fmaxf(mx, y[j]);
  }
  gp = group_params(mn, mx);
  const __half vhs = __float2half_rn(gp.scale), vhz = __float2half_rn(gp.zero);
  rec.vs[tok * 4 + q] = vhs;
  rec.vz[tok * 4 + q] = vhz;
  sts16(qs + L::vs(sl) + (tok * 4 + q) * 2, vhs);
  sts16(qs + L::vz(sl) + (tok * 4 + q) * 2, vhz);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) lo |= code_of(y[j], gp) << (2 * j);
#pragma unroll
  for (int j = 0; j < 16; ++j) hi |= code_of(y[16 + j], gp) << (2 * j);
  *reinterpret_cast<uint2*>(rec.vp + tok * 32 + q * 8) = make_uint2(lo, hi);
  sts64(qs + L::vp(sl) + tok * 32 + q * 8, lo, hi);
  fence_proxy_async_smem();
}

// The padded sink group of a unit holding n sink tokens (the n real ones,
// then copies of token 0), into batch 0's slot 0 and the unit's record 0.
// Out of line (with quantize_flushed_group): rare, and large once unrolled,
// it would otherwise crowd the hot loop out of the instruction cache.
__device__ __noinline__ void requantize_sink(const KParams& p, int64_t unit, int n, uint32_t qs, int c) {
  const int S = p.sink;
  float x[32], y[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __half2float(p.sink_k16[(unit * S + (j < n ? j : 0)) * kHeadDim + c]);
  const int tok = c >> 2, q = c & 3;
  const __half* vrow = p.sink_v16 + (unit * S + (tok < n ? tok : 0)) * kHeadDim + q * 32;
#pragma unroll
  for (int j = 0; j < 32; ++j) y[j] = __half2float(vrow[j]);
  store_group_record(x, y, qs, 0, group_rec(p.grp, unit, p.n_groups, 0), c);
}

// Stream group [base, base + 32) leaving the residual ring (slots s0 .. s0+31,
// never wrapping: 32 divides both base and the ring size): into Q-stage slot
// `sl` and window-group slot gs.  Read from the staged F-tiles when every
// F-tile of the unit is still resident (f_stage0: the F ring's base address),
// else from the cache.
__device__ __noinline__ void quantize_flushed_group(const KParams& p, int64_t unit, int base, int gs,
                                                       uint32_t qs, int sl, uint32_t f_stage0, int c) {
  const int C = p.res_cap;
  const int s0 = base % C;
  const int tok = c >> 2, q = c & 3;
  float x[32], y[32];
  if (f_stage0) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int slot = s0 + j, f = slot / kFRows, r = slot % kFRows;
      const uint32_t a = f_stage0 + f * kFStageBytes + Lay<true>::f(r, c >> 3) + (c & 7) * 2;
      unsigned short h;
      asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
      x[j] = __half2float(__ushort_as_half(h));
    }
    const int slot = s0 + tok, f = slot / kFRows, r = slot % kFRows;
    const uint32_t vb = f_stage0 + f * kFStageBytes + kFTile;
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // channels q*32 + 8k .. +7
      uint32_t w[4];
      lds128(vb + Lay<true>::f(r, 4 * q + k), w[0], w[1], w[2], w[3]);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f2 = __half22float2(u32_as_h2(w[e]));
        y[8 * k + 2 * e] = f2.x;
        y[8 * k + 2 * e + 1] = f2.y;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = __half2float(p.k_res[(unit * C + s0 + j) * kHeadDim + res_elem(s0 + j, c)]);
    const uint4* vrow = reinterpret_cast<const uint4*>(p.v_res + (unit * C + s0 + tok) * kHeadDim);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 v = vrow[res_chunk(s0 + tok, 4 * q + k)];
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f2 = __half22float2(u32_as_h2(w[e]));
        y[8 * k + 2 * e] = f2.x;
        y[8 * k + 2 * e + 1] = f2.y;
      }
    }
  }
  store_group_record(x, y, qs, sl, group_rec(p.grp, unit, p.n_groups, 1 + gs), c);
}

// Load issue, run by lane 0 of warp 0 (at launch start, the F-tiles of the
// free stages by lanes 0 of warps 1..kFStages).  Each ring is filled in
// order; an item is issued once warp 0 itself has consumed the previous user
// of its stage (the other warps' release is then waited for, which never
// depends on an item not yet issued).
template <bool kRec>
struct Issuer {
  const KParams& p;
  Smem& sm;
  const CUtensorMap* tmK;
  const CUtensorMap* tmV;
  int64_t unit;
  int f_next, f_end, b_next, b_end;
  uint32_t f_issued = 0, q_issued = 0;
  bool ok = true;

  __device__ __forceinline__ Issuer(const KParams& p_, Smem& sm_, const CUtensorMap* k, const CUtensorMap* v,
                                    int64_t u, int f0, int f1, int b0, int b1)
      : p(p_), sm(sm_), tmK(k), tmV(v), unit(u), f_next(f0), f_end(f1), b_next(b0), b_end(b1) {}

  // Q-batch b into Q stage s: the sink group (batch 0) and window groups p0..p1-1.
  __device__ __forceinline__ void batch(int b, uint32_t s) {
    const uint32_t fb = smem_u32(&sm.q_full[s]);
    const uint32_t sd = smem_u32(sm.qb[s]);
    if constexpr (kRec) {  // batch slot v of the unit is its record v: one copy
      const int v0 = kBatchGroups * b, v1 = min(p.n_groups + 1, v0 + kBatchGroups);
      const uint32_t bytes = static_cast<uint32_t>(v1 - v0) * kRecBytes;
      mbar_arrive_expect_tx(fb, bytes);
      bulk_load(sd, p.grp + (unit * (p.n_groups + 1) + v0) * int64_t(kRecBytes), bytes, fb);
      return;
    }
    const int p0 = b == 0 ? 0 : kBatchGroups * b - 1;  // batch slot v holds group v - 1
    const int p1 = min(p.n_groups, kBatchGroups * b + kBatchGroups - 1);
    const int so = p0 + 1 - kBatchGroups * b;
    const uint32_t ng = p1 > p0 ? p1 - p0 : 0;
    mbar_arrive_expect_tx(fb, (b == 0 ? 3072u : 0u) + ng * 3072u);
    if (ng) {
      const int64_t gbase = unit * p.n_groups + p0;
      bulk_load(sd + kOffKP + so * 1024, p.kw_p + gbase * 1024, ng * 1024, fb);
      bulk_load(sd + kOffKS + so * 256, p.kw_s + gbase * 128, ng * 256, fb);
      bulk_load(sd + kOffKZ + so * 256, p.kw_z + gbase * 128, ng * 256, fb);
      bulk_load(sd + kOffVP + so * 1024, p.vw_p + gbase * 1024, ng * 1024, fb);
      bulk_load(sd + kOffVS + so * 256, p.vw_s + gbase * 128, ng * 256, fb);
      bulk_load(sd + kOffVZ + so * 256, p.vw_z + gbase * 128, ng * 256, fb);
    }
    if (b == 0) {
      bulk_load(sd + kOffKP, p.ks_p + unit * 1024, 1024, fb);
      bulk_load(sd + kOffKS, p.ks_s + unit * 128, 256, fb);
      bulk_load(sd + kOffKZ, p.ks_z + unit * 128, 256, fb);
      bulk_load(sd + kOffVP, p.vs_p + unit * 1024, 1024, fb);
      bulk_load(sd + kOffVS, p.vs_s + unit * 128, 256, fb);
      bulk_load(sd + kOffVZ, p.vs_z + unit * 128, 256, fb);
    }
  }
  // Batch 0 (always live): the first use of Q stage 0.
  __device__ __forceinline__ void batch0() {
    batch(0, 0);
    q_issued = 1;
  }
  // F-tiles, while warp 0 has consumed the previous user of the stage (f_cons F-tiles consumed).
  __device__ __forceinline__ void pump_f(uint32_t f_cons) {
    while (ok && f_next < f_end && f_issued < f_cons + kFStages) {
      const uint32_t s = f_issued % kFStages, ph = (f_issued / kFStages) & 1;
      if (!mbar_wait(smem_u32(&sm.f_empty[s]), ph ^ 1, p.err)) {
        ok = false;
        break;
      }
      const uint32_t fb = smem_u32(&sm.f_full[s]);
      const uint32_t sd = smem_u32(sm.f[s]);
      sm.f_job[s] = 0;  // every warp has released the stage
      if constexpr (kRec) {  // rows f_next*80 .. of the unit's ring, K and V one copy each
        const int row0 = f_next * kFRows;
        const uint32_t rows = static_cast<uint32_t>(min(kFRows, p.res_cap - row0));
        mbar_arrive_expect_tx(fb, 2 * rows * 256);
        const int64_t off = (unit * p.res_cap + row0) * kHeadDim;
        bulk_load(sd, p.k_res + off, rows * 256, fb);
        bulk_load(sd + kFTile, p.v_res + off, rows * 256, fb);
      } else {
        mbar_arrive_expect_tx(fb, kFStageBytes);
        const int uu = static_cast<int>(unit);
        tma_load_4d(sd, tmK, fb, 0, f_next * kFRows, 0, uu);
        tma_load_4d(sd + kFTile, tmV, fb, 0, f_next * kFRows, 0, uu);
      }
      ++f_issued;
      ++f_next;
    }
  }
  // F-tile f_next + i into stage i, free at launch start (no wait), by any thread.
  __device__ __forceinline__ void first_f(int i) {
    const int f = f_next + i;
    if (f >= f_end) return;
    const uint32_t fb = smem_u32(&sm.f_full[i]);
    const uint32_t sd = smem_u32(sm.f[i]);
    if constexpr (kRec) {
      const int row0 = f * kFRows;
      const uint32_t rows = static_cast<uint32_t>(min(kFRows, p.res_cap - row0));
      mbar_arrive_expect_tx(fb, 2 * rows * 256);
      const int64_t off = (unit * p.res_cap + row0) * kHeadDim;
      bulk_load(sd, p.k_res + off, rows * 256, fb);
      bulk_load(sd + kFTile, p.v_res + off, rows * 256, fb);
    } else {
      mbar_arrive_expect_tx(fb, kFStageBytes);
      const int uu = static_cast<int>(unit);
      tma_load_4d(sd, tmK, fb, 0, f * kFRows, 0, uu);
      tma_load_4d(sd + kFTile, tmV, fb, 0, f * kFRows, 0, uu);
    }
  }
  // Streaming layout, F-tile f_next + i into stage i, free at launch start:
  // only the rows covering the unit's attended slots and the slots of a group
  // this launch flushes (fl_s0 >= 0: 32 slots from fl_s0; none: an arrival alone).
  __device__ __forceinline__ void first_f_sized(int i, const KiviMeta& m, int fl_s0) {
    const int f = f_next + i;
    if (f >= f_end) return;
    const uint32_t fb = smem_u32(&sm.f_full[i]);
    const uint32_t sd = smem_u32(sm.f[i]);
    const int row0 = f * kFRows;
    int lo, hi;
    const int row1 = min(row0 + kFRows, p.res_cap);
    attended_cover(p, m, row0, row1, lo, hi);
    if (fl_s0 >= 0 && max(fl_s0, row0) < min(fl_s0 + 32, row1)) {
      lo = min(lo, max(fl_s0, row0));
      hi = max(hi, min(fl_s0 + 32, row1));
    }
    const uint32_t rows = hi > lo ? static_cast<uint32_t>(hi - lo) : 0u;
    mbar_arrive_expect_tx(fb, 2 * rows * 256);
    if (!rows) return;
    const int64_t off = (unit * p.res_cap + lo) * kHeadDim;
    const uint32_t so = static_cast<uint32_t>(lo - row0) * 256;
    bulk_load(sd + so, p.k_res + off, rows * 256, fb);
    bulk_load(sd + kFTile + so, p.v_res + off, rows * 256, fb);
  }
  // The leader's account of the tiles first_f issued.
  __device__ __forceinline__ void skip_first_f() {
    const int n = min(kFStages, f_end - f_next);
    if (n > 0) {
      f_issued += n;
      f_next += n;
    }
  }
  // Live Q-batches after the first, likewise (q_cons Q-batches consumed).
  __device__ __forceinline__ void pump_q(const KiviMeta& meta, uint32_t q_cons) {
    while (ok && b_next < b_end && q_issued < q_cons + kQStages) {
      if (!batch_live(p, meta, b_next)) {
        ++b_next;
        continue;
      }
      const uint32_t s = q_issued % kQStages, ph = (q_issued / kQStages) & 1;
      if (!mbar_wait(smem_u32(&sm.q_empty[s]), ph ^ 1, p.err)) {
        ok = false;
        break;
      }
      batch(b_next, s);
      ++q_issued;
      ++b_next;
    }
  }
};

// The work of CTA `bid` of one layer's launch (tensor maps -- reference
// layout only -- and parameters in kernel-parameter space).  kAppend: the
// launch also appends new_k / new_v (streaming layout, one CTA per unit).
template <bool kRec, bool kAppend, bool kSized, bool kSimple, bool kLateTile1 = false>
__device__ __forceinline__ void kivi_decode_cta(const CUtensorMap* tmK, const CUtensorMap* tmV, const KParams& p,
                                                int bid) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  grid_launch_dependents();
  // the cache and q may come from the previous kernel of the stream: global
  // memory is read only after the wait below (the barriers are initialised
  // first, which measured 0.25 us faster per step launch)
  if (smem_u32(smem_raw) & 1023u) {  // TMA tile destinations need 1024-byte alignment
    if (threadIdx.x == 0) set_error(p.err, NSA_ERR_ALIGN);
    return;
  }
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = bid / p.ppu;
  const int piece = bid % p.ppu;
  // this piece's items [t_begin, t_end): item 0 = Q-batch 0, items 1..n_ft =
  // F-tiles 0..n_ft-1, item n_ft + b = Q-batch b (b >= 1)
  const int t_begin = piece * p.items / p.ppu, t_end = (piece + 1) * p.items / p.ppu;
  const bool has_b0 = t_begin == 0 && t_end > 0;
  const int f_begin = max(t_begin, 1) - 1, f_end = min(t_end, p.n_ft + 1) - 1;
  const int b_begin = max(max(t_begin, p.n_ft + 1) - p.n_ft, 1), b_end = t_end - p.n_ft;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFStages; ++s) {
      mbar_init(smem_u32(&sm.f_full[s]), 1);
      mbar_init(smem_u32(&sm.f_empty[s]), kCWarps);
    }
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(smem_u32(&sm.q_full[s]), 1);
      mbar_init(smem_u32(&sm.q_empty[s]), kCWarps);
      sm.q_rel[s] = 0;
      sm.q_job[s] = 0;
    }
    for (int s = 0; s < kFStages; ++s) sm.f_job[s] = 0;
    sm.d_job = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // Batch 0 goes to L2 while the previous grid finishes (a prefetch reads
  // nothing into this CTA, and L2 stays coherent with that grid's writes), so
  // its copy after the wait lands sooner: -0.5 us per attention launch, -0.3
  // per step.  Prefetching the residual tiles as well measured 0.8 us slower.
  if (kRec && has_b0 && threadIdx.x == 0)
    bulk_prefetch_l2(p.grp + unit * (p.n_groups + 1) * int64_t(kRecBytes),
                     static_cast<uint32_t>(min(p.n_groups + 1, kBatchGroups)) * kRecBytes);
  // Likewise the small inputs every thread loads right after the wait (the
  // unit's query, length and appended token): their loads then hit L2, which
  // shortens the prologue on the way to the first group (-0.15 us per step).
  if (threadIdx.x == 32) {
    bulk_prefetch_l2(p.q + unit * kGroupHeads * kHeadDim, kGroupHeads * kHeadDim * 2);
    if (kRec) prefetch_l2(p.unit_lens + unit);
    if (kAppend) {
      bulk_prefetch_l2(p.new_k + unit * kHeadDim, kHeadDim * 2);
      bulk_prefetch_l2(p.new_v + unit * kHeadDim, kHeadDim * 2);
    }
  }
  grid_dependency_wait();

  // ------------------------------------------------------------- prologue
  // Global loads of every thread go out first (the query -- 16 bytes per
  // thread -- and, when appending, the unit's length and the new token's
  // channel); then lane 0 of warp 0 issues batch 0 and the F-tiles (they do
  // not depend on the unit's length) and, once the length is known, the live
  // Q-batches the ring holds.
  const int ct = threadIdx.x;
  const uint4 qv = __ldg(reinterpret_cast<const uint4*>(p.q + (unit * kGroupHeads + (ct >> 4)) * kHeadDim +
                                                       (ct & 15) * 8));
  static_assert(kRec || !kAppend, "the reference layout never appends");
  constexpr bool appending = kAppend;
  const int64_t len64 = kRec ? p.unit_lens[unit] : 0;
  __half new_kc = __float2half_rn(0.f), new_vc = new_kc;
  if (appending) {
    new_kc = p.new_k[unit * kHeadDim + ct];
    new_vc = p.new_v[unit * kHeadDim + ct];
  }
  Issuer<kRec> iss(p, sm, tmK, tmV, unit, f_begin, f_end, b_begin, b_end);
  const bool leader = threadIdx.x == 0;
  if (leader) {
    if constexpr (!kRec) {
      prefetch_tmap(tmK);
      prefetch_tmap(tmV);
    }
    if (has_b0) iss.batch0();
    if constexpr (kRec)
      iss.skip_first_f();
    else
      iss.pump_f(0);
  }
  // streaming layout: the free stages' F-tiles, one warp each: their copies are issued while
  // lane 0 of warp 0 issues batch 0 (each copy request takes hundreds of cycles to issue):
  // -0.1 to -0.2 us.  (The reference layout's tile loads need the tensor maps lane 0 prefetches.)
  // (kLateTile1: F-tile 1 is issued once the length below has arrived)
  if (kRec && !kSized && lane == 0 && warp >= 1)
    for (int i = warp - 1; i < (kLateTile1 ? 1 : kFStages); i += kCWarps - 1) iss.first_f(i);
  int len = static_cast<int>(len64);
  if (kRec && (len64 < 0 || len64 >= kMaxUnitLen)) {  // outside what the 32-bit ring arithmetic covers
    if (threadIdx.x == 0) set_error(p.err, NSA_ERR_INVALID);
    len = 0;
  }
  const AppendPlan ap = appending && len64 == len ? append_plan(p, len) : AppendPlan{};
  if (appending && len64 == len) ++len;
  const KiviMeta meta = make_meta<kRec>(p, len);
  if (!kSimple && leader) iss.pump_q(meta, 0);
  if (kRec && kSized && lane == 0 && warp >= 1)
    for (int i = warp - 1; i < kFStages; i += kCWarps - 1) iss.first_f_sized(i, meta, ap.fl_s0);
  if (kRec && !kSized && kLateTile1 && lane == 0 && warp == 2) iss.first_f(1);
  sts128(smem_u32(&sm.qpad[ct >> 4][(ct & 15) * 8]), qv.x, qv.y, qv.z, qv.w);
  if (appending) {
    sm.newtok[0][ct] = new_kc;
    sm.newtok[1][ct] = new_vc;
  }
  cwarps_sync();

  // -------------------------------------------------------------- consumers
  // A timed-out wait sets `aborted`: the warp then stops waiting (the error
  // word is already set) but keeps its schedule of named barriers.
  const int g = lane >> 2, t = lane & 3;
  const LaneQ lq(lane);
  bool aborted = false;
  WarpAttn st;
  st.reset();
  const uint32_t qpad = smem_u32(sm.qpad);
  const uint32_t qrow = qpad + g * (kQPadStride * 2) + 32 * t;
  uint32_t nf = 0, nq = 0;
  // Steps: 0 = Q-batch 0, 1 = the F-tiles, 2 = Q-batches b_begin .., 3 = the
  // deferred slot below (one loop, so that each consumer path -- attend_group
  // above all -- is instantiated once).  A group this launch flushes is
  // quantized from the staged F-tiles after they have been consumed: when
  // every item stays staged (resident), batch 0 keeps its place and only the
  // flushed slot waits until after the F-tiles (step 3); otherwise the
  // F-tiles come first and the group is read from the cache.
  const bool flushing = ap.fl_batch >= 0;
  const bool resident = kSimple || (p.n_qb <= kQStages && p.n_ft <= kFStages && f_begin == 0 && f_end == p.n_ft);
  const bool defer_slot = flushing && resident && ap.fl_batch == 0;
  const bool f_first = flushing && !resident;
#pragma unroll 1
  for (int step = 0; step < 4; ++step) {
    const int phase = (f_first && step < 2) ? 1 - step : step;
    if (phase == 3 && !defer_slot) break;
    if (phase == 1) {
      st.load_q(qpad, lane, kQPadStride * 2);  // the residual jobs' query fragments (not held across the groups)
#pragma unroll 1
      for (int f = f_begin; f < f_end; ++f) {
        if (!kSimple && leader) iss.pump_f(nf);
        __syncwarp();
        const uint32_t s = nf % kFStages, ph = (nf / kFStages) & 1;
        ++nf;
        if (!aborted && !mbar_wait(smem_u32(&sm.f_full[s]), ph, p.err)) aborted = true;
        const uint32_t sd = smem_u32(sm.f[s]);
        // jobs of 32 rows (the last one 16): one softmax step per job, each
        // claimed by the first warp free to take it
#pragma unroll 1
        for (int j = claim_job(&sm.f_job[s], lane); j < kFJobs; j = claim_job(&sm.f_job[s], lane)) {
          const int r = 32 * j;
          const int r0 = f * kFRows + r;
          const bool two = r + 32 <= kFRows;
          // attended rows of the job (warp-uniform mask; bit i: row r + i)
          const uint32_t vm = res_slot_mask(p, meta, r0) & (two ? 0xffffffffu : 0xffffu);
          if (!vm) continue;
          bool vl[2], vh[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            vl[h] = ((vm >> (16 * h + g)) & 1u) != 0;
            vh[h] = ((vm >> (16 * h + g + 8)) & 1u) != 0;
          }
          const bool any0 = (vm & 0xffffu) != 0, any1 = (vm >> 16) != 0;
          if (ap.f_item == f && ap.f_row >= r && ap.f_row < r + (two ? 32 : 16))  // the appended token's
            patch_residual_row(sd, ap.f_row, smem_u32(sm.newtok), lane);      // staged row is stale
          // V rows of unattended slots become 0 (P is 0 there, and 0 * NaN would not
          // be), except those of a group this launch flushes: it is quantized from them
          if (vm != (two ? 0xffffffffu : 0xffffu)) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
              if (h == 0 || two)
                zero_invalid_v_rows<kRec>(sd + kFTile, r + 16 * h, vl[h] || ap.flushing(r0 + 16 * h + g),
                                          vh[h] || ap.flushing(r0 + 16 * h + g + 8), lane);
          }
          if (two && any0 && any1) {
            st.consume_rows<2, Lay<kRec>::kRowBytes>(sd, sd + kFTile, Lay<kRec>::kRegion, r, vl, vh, p.scale_log2,
                                                     lane);
          } else {
            // (selects, not vl[h]: a dynamic index would put the flags in local memory)
            const bool l1[1] = {any0 ? vl[0] : vl[1]}, h1[1] = {any0 ? vh[0] : vh[1]};
            st.consume_rows<1, Lay<kRec>::kRowBytes>(sd, sd + kFTile, Lay<kRec>::kRegion, r + (any0 ? 0 : 16), l1, h1,
                                                     p.scale_log2, lane);
          }
        }
        __syncwarp();
        if (!kSimple && lane == 0) mbar_arrive(smem_u32(&sm.f_empty[s]));
      }
      continue;
    }
    if (kSimple && phase == 2) continue;  // one Q-batch
    const int lo = phase == 2 ? b_begin : 0;
    const int hi = phase == 2 ? b_end : (phase == 3 || has_b0 ? 1 : 0);
#pragma unroll 1
    for (int b = lo; b < hi; ++b) {
      if (!batch_live(p, meta, b)) continue;
      uint32_t qs, s = 0;
      if (phase != 3) {
        if (!kSimple && leader) iss.pump_f(nf);
        __syncwarp();
        s = nq % kQStages;
        const uint32_t ph = (nq / kQStages) & 1;
        ++nq;
        if (!aborted && !mbar_wait(smem_u32(&sm.q_full[s]), ph, p.err)) aborted = true;
        qs = smem_u32(sm.qb[s]);
        if (appending && ap.sink && b == 0) {  // the sink group changed: re-quantize it into slot 0 (and the cache)
          p.sink_k16[(unit * p.sink + len - 1) * kHeadDim + ct] = new_kc;  // fp16 copy of the new sink token
          p.sink_v16[(unit * p.sink + len - 1) * kHeadDim + ct] = new_vc;
          cwarps_sync();  // the copies are read back by other threads
          requantize_sink(p, unit, static_cast<int>(len), qs, ct);
          cwarps_sync();
        }
        if (appending && ap.fl_batch == b && !defer_slot) {  // a window group was flushed: quantize it into its
          // slot (and the cache); the F-tiles were consumed before, and are still staged when resident
          quantize_flushed_group(p, unit, ap.fl_base, ap.fl_gs, qs, ap.fl_slot, resident ? smem_u32(sm.f[0]) : 0u,
                                 ct);
          cwarps_sync();
        }
      } else {  // batch 0 (stage 0) is still staged: its flushed slot now
        qs = smem_u32(sm.qb[0]);
        quantize_flushed_group(p, unit, ap.fl_base, ap.fl_gs, qs, ap.fl_slot, smem_u32(sm.f[0]), ct);
        cwarps_sync();
      }
      int* const jobs = phase == 3 ? &sm.d_job : &sm.q_job[s];  // each group claimed by the first free warp
#pragma unroll 1
      for (int gs = claim_job(jobs, lane); gs < kBatchGroups; gs = claim_job(jobs, lane)) {
        if (phase == 3 ? gs != ap.fl_slot : (defer_slot && b == 0 && gs == ap.fl_slot)) continue;
        const uint32_t mask = group_mask(p, meta, b, gs);
        if (!mask) continue;
        attend_group<kRec>(st, qrow, lq, qs, gs, mask, p.scale_log2, lane);
      }
      if (!kSimple && phase != 3) {  // release the stage; the last warp to do so refills it
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();  // this warp's reads of the stage come first
          if (atomicAdd(&sm.q_rel[s], 1) == kCWarps - 1) {
            sm.q_rel[s] = 0;
            sm.q_job[s] = 0;  // every warp has stopped claiming from this batch
            __threadfence_block();
            // the stage's next batch is two live batches on in the issue order
            // (batch 0, then the live batches from b_begin)
            const auto succ = [&](int x) {
              int y = x == 0 ? b_begin : x + 1;
              while (y < b_end && !batch_live(p, meta, y)) ++y;
              return y;
            };
            const int b1 = succ(b), b2 = b1 < b_end ? succ(b1) : b_end;
            if (b2 < b_end) {
              fence_proxy_async_smem();
              iss.batch(b2, s);
            }
          }
        }
      }
    }
  }

  // ---- epilogue: merge the 4 warps (the F ring is reused once all have finished)
  cwarps_sync();
  warp_publish(st, sm.ep, warp, lane);
  cwarps_sync();
  const int hh = ct >> 4, d0 = (ct & 15) * 8;  // this thread's head and 8 dims
  float o[8], lse;
  merge_warps<8>(sm.ep, hh, d0, o, lse);
  if (appending) {
    if (ap.f_item >= 0) {  // the new token's residual slot
      const int slot = (len - 1 - p.sink) % p.res_cap;
      p.k_res[(unit * p.res_cap + slot) * kHeadDim + res_elem(slot, ct)] = new_kc;
      p.v_res[(unit * p.res_cap + slot) * kHeadDim + res_elem(slot, ct)] = new_vc;
    }
    if (ct == 0 && len64 >= 0 && len64 < kMaxUnitLen)  // every thread read the old length at entry
      p.unit_lens[unit] = len;
  }
  __half* out = p.o + unit * kGroupHeads * kHeadDim;
  if (kSimple || p.ppu == 1) {
    store_half8(out + hh * kHeadDim + d0, o);
    return;
  }
  const int64_t pidx = unit * p.ppu + piece;
  float* po = p.part_o + (pidx * kGroupHeads + hh) * kHeadDim + d0;
  reinterpret_cast<float4*>(po)[0] = make_float4(o[0], o[1], o[2], o[3]);
  reinterpret_cast<float4*>(po)[1] = make_float4(o[4], o[5], o[6], o[7]);
  if ((ct & 15) == 0) p.part_lse[pidx * kGroupHeads + hh] = lse;
  __threadfence();
  cwarps_sync();
  if (ct == 0) sm.ep.ticket = atomicAdd(p.counters + unit, 1);
  cwarps_sync();
  if (sm.ep.ticket == p.ppu - 1) {
    __threadfence();
    const int64_t base = unit * p.ppu;
    combine_pieces(p.part_lse + base * kGroupHeads, p.part_o + base * kGroupHeads * kHeadDim, p.ppu, out,
                   warp * (kGroupHeads / kCWarps), kGroupHeads / kCWarps, lane);
    if (ct == 0) p.counters[unit] = 0;
  }
}

// kSimple: one CTA per unit, one Q-batch and every F-tile resident in its
// stage from the start, so nothing is ever refilled and no piece is merged:
// the refill, later-batch and split-K code is left out of this instantiation
// (B=32: W=256 step 7.75 -> 7.61 us, reference-layout launch -0.35 us, W=32
// 5.65 -> 4.95 us).
//
// The reference's 14-tensor layout (residual by TMA boxes).
template <bool kSimple>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    kivi_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const KParams p) {
  kivi_decode_cta<false, false, false, kSimple>(&tmK, &tmV, p, blockIdx.x);
}

// The streaming cache (every load a 1-D bulk copy): attention only, and a
// decode step (append + attention; its cold paths take p by reference).
// kSized: the window is shorter than the residual, so a launch attends few
// of the ring's slots and its F-tile copies cover only those (issued once the
// unit's length is known): W=32 6.7 -> 5.7 us, W=64 6.8 -> 6.1 us per launch
// at B=32.  Longer windows attend nearly every slot and keep the copies that
// need no length, in their own instantiation.
//
// A one-layer launch issues the copy of F-tile 1 (the second 80 slots) only
// once the unit's length has arrived, ~0.9 us after the grid wait: batch 0
// and F-tile 0 of every unit then reach the SMs first, so their work is done
// when F-tile 1 lands (W=256 step 7.59 -> 7.37 us; covering only the rows
// read as well measured 0.03 us slower, and waiting for batch 0 to land
// 0.2 us slower).  The layer-batched launch, whose CTAs start at staggered
// times, issues both at once (the late copy measured +0.19 us per layer).
template <bool kSized, bool kSimple>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) kivi_stream_decode_kernel(const KParams p) {
  kivi_decode_cta<true, false, kSized, kSimple, true>(nullptr, nullptr, p, blockIdx.x);
}
template <bool kSized, bool kSimple>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    kivi_stream_step_kernel(const __grid_constant__ KParams p) {
  kivi_decode_cta<true, true, kSized, kSimple, true>(nullptr, nullptr, p, blockIdx.x);
}

// Several layers (caches of one geometry) in one launch: layer-major CTAs,
// `per_layer` of them per layer.  Amortises the launch's fixed costs (start,
// first-byte latency, tail) over all layers when the decode loop has every
// layer's query at once.
constexpr int kMaxLayers = 64;
struct KiviLayers {
  KParams p[kMaxLayers];
  unsigned per_layer;
  int n_layers;
};
static_assert(sizeof(KiviLayers) <= 32000, "kernel parameter space");

template <bool kSized, bool kSimple>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) kivi_decode_layers_kernel(const __grid_constant__ KiviLayers L) {
  const int layer = static_cast<int>(blockIdx.x / L.per_layer);
  kivi_decode_cta<true, true, kSized, kSimple>(nullptr, nullptr, L.p[layer],
                                              static_cast<int>(blockIdx.x % L.per_layer));
}

// One of a kernel's four instantiations <kSized, kSimple>.
template <class K>
K pick(bool sized, bool simple, K ff, K ft, K tf, K tt) {
  return sized ? (simple ? tt : tf) : (simple ? ft : ff);
}
#define NSA_KIVI_PICK(kernel, sized, simple) \
  pick(sized, simple, kernel<false, false>, kernel<false, true>, kernel<true, false>, kernel<true, true>)

// Whether a streaming-cache launch sizes its F-tile copies (see above).
bool sized_f(const KParams& p) { return p.layout == 1 && p.window < p.residual; }

struct Plan {
  int64_t n_units, grid;
  int n_qb, n_ft, items, ppu;
};

// CTA slots of the current device (resident CTAs per SM x SMs); sets the
// kernel's shared-memory limit on first use per device.
int64_t cta_slots() {
  static int64_t slots[64] = {0};
  const DeviceInfo& d = current_device();
  const int dev = d.device;
  const int sms = d.sm_count > 0 ? d.sm_count : 148;
  if (dev < 0 || dev >= 64) return int64_t(sms) * kCtasPerSm;
  if (!slots[dev]) {
    int per_sm = 0;
    const auto smem = [](auto kernel) {
      return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) ==
             cudaSuccess;
    };
    bool ok = smem(kivi_decode_kernel<false>) && smem(kivi_decode_kernel<true>);
    for (int i = 0; i < 4; ++i)
      ok = ok && smem(NSA_KIVI_PICK(kivi_stream_decode_kernel, i & 1, i >> 1)) &&
           smem(NSA_KIVI_PICK(kivi_stream_step_kernel, i & 1, i >> 1)) &&
           smem(NSA_KIVI_PICK(kivi_decode_layers_kernel, i & 1, i >> 1));
    if (!ok || cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kivi_decode_kernel<false>, kThreads, kSmemBytes) !=
            cudaSuccess ||
        per_sm < 1) {
      cudaGetLastError();
      per_sm = 1;
    }
    slots[dev] = int64_t(sms) * per_sm;
  }
  return slots[dev];
}

Plan plan(int64_t n_units, int n_groups, int res_cap) {
  Plan s;
  s.n_units = n_units;
  s.n_qb = (n_groups + 1 + kBatchGroups - 1) / kBatchGroups;
  s.n_ft = (res_cap + kFRows - 1) / kFRows;
  s.items = s.n_qb + s.n_ft;
  // fewer units than CTA slots: split each unit's items so that the slots
  // fill -- unless every item of a unit is resident in its stages from the
  // start: such a unit is a short chain whose split pieces would only add the
  // merge (and, for a decode step, a separate append launch)
  const int64_t slots = cta_slots();
  const bool resident = s.n_qb <= kQStages && s.n_ft <= kFStages;
  int64_t ppu = (!resident && n_units > 0 && n_units < slots) ? slots / n_units : 1;
  if (ppu > s.items) ppu = s.items;
  if (ppu < 1) ppu = 1;
  s.ppu = static_cast<int>(ppu);
  s.grid = n_units * ppu;
  return s;
}

// Whether a launch of plan s can take the kSimple instantiation.
bool simple(const Plan& s) { return s.ppu == 1 && s.n_qb == 1 && s.n_ft <= kFStages; }

size_t ws_bytes(const Plan& s) {
  const size_t counters = ((s.n_units * sizeof(int)) + 255) & ~size_t(255);
  const size_t pieces = static_cast<size_t>(s.n_units) * s.ppu;
  const size_t lse = ((pieces * kGroupHeads * sizeof(float)) + 255) & ~size_t(255);
  return counters + lse + pieces * kGroupHeads * kHeadDim * sizeof(float);
}

// Completes p for plan s (workspace carving, device error word) and, for the
// reference layout, encodes the residual tensor maps.
int prepare(KParams& p, const Plan& s, const void* k_res, const void* v_res, void* ws, size_t wsb, CUtensorMap* mk,
            CUtensorMap* mv) {
  const size_t need = ws_bytes(s);
  if (!ws || wsb < need)
    return fail(NSA_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, ws ? wsb : size_t(0));
  if (!aligned16(ws)) return fail(NSA_ERR_ALIGN, "workspace must be 16-byte aligned");
  if (s.grid > 0x7fffffff) return fail(NSA_ERR_UNSUPPORTED, "too many units for one launch");
  uint8_t* w = static_cast<uint8_t*>(ws);
  const size_t counters = ((s.n_units * sizeof(int)) + 255) & ~size_t(255);
  const size_t pieces = static_cast<size_t>(s.n_units) * s.ppu;
  const size_t lse = ((pieces * kGroupHeads * sizeof(float)) + 255) & ~size_t(255);
  p.counters = reinterpret_cast<int*>(w);
  p.part_lse = reinterpret_cast<float*>(w + counters);
  p.part_o = reinterpret_cast<float*>(w + counters + lse);
  p.n_units = s.n_units;
  p.n_qb = s.n_qb;
  p.n_ft = s.n_ft;
  p.items = s.items;
  p.ppu = s.ppu;
  p.err = device_error_word();
  if (!p.err) return fail(NSA_ERR_CUDA, "device error word unavailable");
  if (p.layout != 0) return NSA_OK;
  // residual [units][res_cap][128] viewed as [units][2 halves][res_cap][64] (dims
  // innermost first): one box brings 80 slots x both 64-dim halves, each half a
  // 128-byte-swizzled region of 80 rows
  const uint64_t dims[4] = {64, static_cast<uint64_t>(p.res_cap), 2, static_cast<uint64_t>(s.n_units)};
  const uint64_t strides[3] = {kHeadDim * 2, 128, static_cast<uint64_t>(p.res_cap) * kHeadDim * 2};
  const uint32_t box[4] = {64, kFRows, 2, 1};
  int rc = encode_tiled(mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, k_res, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  return encode_tiled(mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, v_res, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch(KParams& p, const Plan& s, const void* k_res, const void* v_res, void* ws, size_t wsb,
           cudaStream_t stream) {
  if (s.n_units == 0) return NSA_OK;
  CUtensorMap mk, mv;
  int rc = prepare(p, s, k_res, v_res, ws, wsb, &mk, &mv);
  if (rc) return rc;
  cta_slots();  // sets the shared-memory limit
  const dim3 grid(static_cast<unsigned>(s.grid));
  const bool sz = sized_f(p), sp = simple(s);
  cudaError_t e =
      p.layout == 0 ? launch_kernel(sp ? kivi_decode_kernel<true> : kivi_decode_kernel<false>, grid, dim3(kThreads),
                                    kSmemBytes, stream, mk, mv, p)
      : p.new_k ? launch_kernel(NSA_KIVI_PICK(kivi_stream_step_kernel, sz, sp), grid, dim3(kThreads), kSmemBytes, stream, p)
                : launch_kernel(NSA_KIVI_PICK(kivi_stream_decode_kernel, sz, sp), grid, dim3(kThreads), kSmemBytes,
                                stream, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "kivi decode launch");
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
  if (c.batch == 0) return NSA_OK;  // an empty cache: its (empty) tensors may be NULL
  if (!c.unit_lens) return fail(NSA_ERR_INVALID, "unit_lens must not be NULL");
  if (!all_aligned({c.sink_k, c.sink_v, c.groups, c.k_res, c.v_res}))
    return fail(NSA_ERR_ALIGN, "stream cache tensors must be non-null and 16-byte aligned");
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
  if (batch > 0 &&  // an empty batch reads and writes nothing: its (empty) tensors may be NULL
      (!all_aligned({q, o, k_res, v_res, k_sink_packed, k_sink_scale, k_sink_zero, v_sink_packed, v_sink_scale,
                     v_sink_zero}) ||
       (ng > 0 && !all_aligned({k_win_packed, k_win_scale, k_win_zero, v_win_packed, v_win_scale, v_win_zero}))))
    return fail(NSA_ERR_ALIGN, "all tensors must be non-null and 16-byte aligned");
  KParams p{};
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(o);
  p.n_kv_heads = static_cast<int>(n_kv_heads);
  p.layout = 0;
  p.seq_len = seq_len < kMaxUnitLen ? seq_len : kMaxUnitLen;  // same attended set beyond S + W
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

namespace {

// Kernel parameters of a streaming-cache launch (attention only).
void stream_params(const nsa_kivi_stream_cache& c, const void* q, void* o, float sm_scale, KParams& p) {
  p = KParams{};
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
  p.grp = static_cast<uint8_t*>(c.groups);
  p.k_res = static_cast<__half*>(c.k_res);
  p.v_res = static_cast<__half*>(c.v_res);
}

// Whether a decode step may append inside the attention launch (NSA_FUSED_APPEND=0
// turns it off, for comparison).
bool fused_append_enabled() {
  static const bool on = [] {
    const char* e = getenv("NSA_FUSED_APPEND");
    return !(e && e[0] == '0');
  }();
  return on;
}

Plan stream_plan(const nsa_kivi_stream_cache& c) {
  return plan(c.batch * c.n_kv_heads, static_cast<int>(c.n_groups), static_cast<int>(c.residual + 32));
}

}  // namespace

int nsa_kivi_stream_decode(const nsa_kivi_stream_cache* cache, const void* q, void* o, float sm_scale,
                           void* workspace, size_t workspace_bytes, nsa_stream_t stream) {
  clear_error();
  if (!cache) return fail(NSA_ERR_INVALID, "null cache");
  const nsa_kivi_stream_cache& c = *cache;
  int rc = kivi_check_stream_cache(c);
  if (rc) return rc;
  if (c.batch > 0 && !all_aligned({q, o})) return fail(NSA_ERR_ALIGN, "q and o must be non-null and 16-byte aligned");
  KParams p;
  stream_params(c, q, o, sm_scale, p);
  return launch(p, stream_plan(c), c.k_res, c.v_res, workspace, workspace_bytes, stream);
}

int nsa_kivi_stream_decode_step(const nsa_kivi_stream_cache* cache, const void* new_k, const void* new_v,
                                const void* q, void* o, float sm_scale, void* workspace, size_t workspace_bytes,
                                nsa_stream_t stream) {
  clear_error();
  if (!cache) return fail(NSA_ERR_INVALID, "null cache");
  const nsa_kivi_stream_cache& c = *cache;
  int rc = kivi_check_stream_cache(c);
  if (rc) return rc;
  if (c.batch > 0 && !all_aligned({q, o, new_k, new_v}))
    return fail(NSA_ERR_ALIGN, "q, o, new_k and new_v must be non-null and 16-byte aligned");
  const Plan s = stream_plan(c);
  if (s.n_units == 0) return NSA_OK;
  if (s.ppu == 1 && fused_append_enabled()) {
    KParams p;
    stream_params(c, q, o, sm_scale, p);
    p.new_k = static_cast<const __half*>(new_k);
    p.new_v = static_cast<const __half*>(new_v);
    p.sink_k16 = static_cast<__half*>(c.sink_k);
    p.sink_v16 = static_cast<__half*>(c.sink_v);
    return launch(p, s, c.k_res, c.v_res, workspace, workspace_bytes, stream);
  }
  // split units: append in its own launch, then attend
  rc = nsa_kivi_append(cache, new_k, new_v, stream);
  if (rc) return rc;
  return nsa_kivi_stream_decode(cache, q, o, sm_scale, workspace, workspace_bytes, stream);
}

int nsa_kivi_stream_step_launches(const nsa_kivi_stream_cache* c) {
  if (!c || c->batch < 0 || c->n_kv_heads <= 0 || c->residual <= 0) return 0;
  return stream_plan(*c).ppu == 1 && fused_append_enabled() ? 1 : 2;
}

int nsa_kivi_stream_decode_step_layers(const nsa_kivi_stream_cache* caches, int64_t n_layers,
                                       const void* const* new_k, const void* const* new_v, const void* const* q,
                                       void* const* o, float sm_scale, void* workspace, size_t workspace_bytes,
                                       nsa_stream_t stream) {
  clear_error();
  if (n_layers < 0) return fail(NSA_ERR_INVALID, "n_layers must be >= 0");
  if (n_layers == 0) return NSA_OK;
  if (!caches || !new_k || !new_v || !q || !o) return fail(NSA_ERR_INVALID, "null pointer");
  const nsa_kivi_stream_cache& c0 = caches[0];
  for (int64_t l = 0; l < n_layers; ++l) {
    const nsa_kivi_stream_cache& c = caches[l];
    int rc = kivi_check_stream_cache(c);
    if (rc) return rc;
    if (c.batch != c0.batch || c.n_kv_heads != c0.n_kv_heads || c.window != c0.window || c.sink != c0.sink ||
        c.residual != c0.residual)
      return fail(NSA_ERR_INVALID, "all layers' caches must have the geometry of layer 0");
    if (c.batch > 0 && !all_aligned({q[l], o[l], new_k[l], new_v[l]}))
      return fail(NSA_ERR_ALIGN, "q, o, new_k and new_v of every layer must be non-null and 16-byte aligned");
  }
  const Plan s = stream_plan(c0);
  if (s.n_units == 0) return NSA_OK;
  if (s.ppu != 1 || !fused_append_enabled() || s.grid * kMaxLayers > 0x7fffffff) {
    for (int64_t l = 0; l < n_layers; ++l) {  // one step per layer
      int rc = nsa_kivi_stream_decode_step(&caches[l], new_k[l], new_v[l], q[l], o[l], sm_scale, workspace,
                                           workspace_bytes, stream);
      if (rc) return rc;
    }
    return NSA_OK;
  }
  static thread_local KiviLayers L;  // kept off the stack
  cta_slots();
  for (int64_t l0 = 0; l0 < n_layers; l0 += kMaxLayers) {
    const int n = static_cast<int>(n_layers - l0 < kMaxLayers ? n_layers - l0 : kMaxLayers);
    for (int i = 0; i < n; ++i) {
      const nsa_kivi_stream_cache& c = caches[l0 + i];
      KParams& p = L.p[i];
      stream_params(c, q[l0 + i], o[l0 + i], sm_scale, p);
      p.new_k = static_cast<const __half*>(new_k[l0 + i]);
      p.new_v = static_cast<const __half*>(new_v[l0 + i]);
      p.sink_k16 = static_cast<__half*>(c.sink_k);
      p.sink_v16 = static_cast<__half*>(c.sink_v);
      int rc = prepare(p, s, c.k_res, c.v_res, workspace, workspace_bytes, nullptr, nullptr);
      if (rc) return rc;
    }
    L.per_layer = s.grid;
    L.n_layers = n;
    cudaError_t e = launch_kernel(NSA_KIVI_PICK(kivi_decode_layers_kernel, sized_f(L.p[0]), simple(s)),
                                  dim3(static_cast<unsigned>(s.grid * n)), dim3(kThreads), kSmemBytes, stream, L);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "kivi_decode_layers_kernel launch");
  }
  return NSA_OK;
}

}  // extern "C"
