// Dense causal GQA decode and StreamingLLM sink+window decode over float16
// KV caches (reference: dense_kernel.py:21-82, sparse_kernel.py:15-118).
//
// Work decomposition (stream-K split-K): the global space of
// (unit = batch*kv_head, 64-token tile) is cut into one contiguous, equal
// slice per persistent CTA (one CTA per SM).  A slice covers pieces of one or
// more units; a unit split across k CTAs leaves k partial results that the
// last CTA to finish (atomic ticket, no waiting) merges with a log-sum-exp
// combine.  Per CTA: warp 4 issues TMA loads of K/V tiles into a 6-stage
// shared-memory ring (and the 8x128 Q block of each piece into a 2-slot
// ring); warps 0-3 each consume 16 tokens of every tile on the tensor cores.
#include <cstddef>
#include <cstdlib>
#include <mutex>

#include "attn_engine.cuh"
#include "host_util.h"

namespace nsa {

namespace {

// Even, so tile k's stage (k % kStages) is always consumed by the same group
// (k % kGroups): a group then observes every phase of its stages' barriers,
// which parity waits require.
constexpr int kStages = 6;
static_assert(kStages % kGroups == 0, "each stage must belong to one consumer group");
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr uint32_t kRegionBytes = kTile * 128;       // one 64-dim half of a tile
constexpr uint32_t kTileBytes = 2 * kRegionBytes;    // K (or V) tile, 16 KiB
constexpr uint32_t kStageBytes = 2 * kTileBytes;     // K + V
constexpr uint32_t kQBytes = kGroupHeads * kHeadDim * 2;

// Per-piece facts the consumers need, computed once by the producer and
// published with the piece's Q block.
struct PieceMeta {
  int64_t len;  // sequence length (tokens appended so far)
  int32_t head; // ring head (sparse)
  int32_t n_inv;  // sparse: window slots with logical index < n_inv are not valid
};

struct Smem {
  uint8_t kv[kStages][kStageBytes];  // 1024-aligned (swizzle atom)
  uint8_t q[2][kQBytes];
  PieceMeta meta[2];
  EpilogueSmem ep;
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t q_full[2];
  uint64_t q_empty[2];
};

static_assert(offsetof(Smem, kv) % 1024 == 0 && kStageBytes % 1024 == 0, "TMA tile destinations");
static_assert(offsetof(Smem, q) % 16 == 0 && kQBytes % 16 == 0, "bulk-copy destinations");

enum Mode : int { kDense = 0, kSparse = 1 };

struct Params {
  const __half* q;
  __half* o;
  int64_t n_units;
  int n_kv_heads;
  int mode;
  int64_t tiles_per_unit;
  int64_t total_tiles;
  int n_ctas;
  int64_t seq_len;
  const int64_t* seq_lens;
  const int32_t* ring_heads;
  int window;
  int sink;
  float scale_log2;
  int max_pieces;
  int unit_aligned;  // 1: every CTA takes whole units (no split-K, no combine)
  int* counters;
  float* part_lse;
  float* part_o;
  int* err;
  // ring cache with per-unit lengths (sparse mode; null: seq_len / seq_lens /
  // ring_heads): unit u holds unit_lens[u] tokens, position p >= sink at slot
  // sink + (p - sink) % window, so its ring head is (len - sink) % window.
  int64_t* unit_lens;
  // one-launch append (window kernel only; null: attention only): the token
  // new_k/new_v[u] is stored at position unit_lens[u] of k_w/v_w first.
  const __half* new_k;
  const __half* new_v;
  __half* k_w;
  __half* v_w;
};

// CTA owning global tile X under the even split of `total` tiles over `ctas`.
__device__ __forceinline__ int64_t owner_cta(int64_t X, int64_t total, int64_t ctas) {
  return ((X + 1) * ctas + total - 1) / total - 1;
}

__device__ __forceinline__ int64_t unit_len(const Params& p, int64_t unit) {
  return p.seq_lens ? p.seq_lens[unit / p.n_kv_heads] : p.seq_len;
}

__device__ __forceinline__ PieceMeta make_meta(const Params& p, int64_t unit) {
  PieceMeta m;
  if (p.unit_lens) {
    m.len = p.unit_lens[unit] + (p.new_k ? 1 : 0);
    m.head = (m.len > p.sink && p.window > 0) ? static_cast<int32_t>((m.len - p.sink) % p.window) : 0;
  } else {
    m.len = unit_len(p, unit);
    m.head = p.ring_heads ? p.ring_heads[unit / p.n_kv_heads] : 0;
  }
  // window slot with logical index i holds position len - W + i: valid iff >= S
  const int64_t n_inv = int64_t(p.sink) - (m.len - p.window);
  m.n_inv = static_cast<int32_t>(n_inv < 0 ? 0 : (n_inv > p.window ? p.window : n_inv));
  return m;
}

// Slot validity (sparse_kernel.py:15-46 plus the ring head), division-free:
// sink slot s valid iff s < len; window slot s has logical index
// (s - S - head) mod W, computed with one conditional add since both terms
// lie in [0, W).
__device__ __forceinline__ bool slot_valid(const Params& p, int64_t slot, const PieceMeta& m) {
  if (p.mode == kDense) return slot < m.len;
  const int s = static_cast<int>(slot);
  if (s < p.sink) return s < m.len;
  if (s >= p.sink + p.window) return false;
  int x = s - p.sink - m.head;
  if (x < 0) x += p.window;
  return x >= m.n_inv;
}

// Valid slots r0 .. r0 + 31 of a sink+window cache as a mask (bit i: slot
// r0 + i), the set slot_valid gives, from warp-uniform arithmetic.  Needs
// window >= 32, so that 32 consecutive slots wrap the ring at most once.
__device__ __forceinline__ uint32_t window_slot_mask(const Params& p, int r0, const PieceMeta& m) {
  const int S = p.sink, W = p.window;
  const int ns = m.len < S ? static_cast<int>(m.len) : S;  // sink slots s < min(S, len)
  uint32_t mk = bit_range(0, ns - r0);
  const int i0 = max(S - r0, 0);  // bit of the first window slot in the range
  if (i0 < 32) {
    int a = r0 + i0 - S - m.head;  // in (-W, W)
    if (a < 0) a += W;             // logical index of slot r0 + i0
    const int wrap = i0 + W - a;   // first bit whose logical index wraps to 0
    mk |= bit_range(i0 + m.n_inv - a, wrap) & bit_range(i0, 32);  // index a + i - i0 >= n_inv
    mk |= bit_range(wrap + m.n_inv, 32);                           // index i - wrap >= n_inv
    mk &= bit_range(0, S + W - r0);                                // slots >= S + W do not exist
  }
  return mk;
}

// Number of tiles of `unit` that can hold a valid slot (dense: up to len).
__device__ __forceinline__ int64_t unit_tiles(const Params& p, int64_t unit) {
  if (p.mode == kDense && !p.unit_lens) {
    const int64_t len = unit_len(p, unit);
    return min(p.tiles_per_unit, (len + kTile - 1) / kTile);
  }
  return p.tiles_per_unit;
}

struct Piece {
  int64_t unit, t_begin, t_end;  // tiles [t_begin, t_end) of unit (after length clipping)
  int slot, n_pieces;
};

// Iterates the pieces of this CTA's slice in order.
struct PieceIter {
  int64_t X, X1;
  __device__ __forceinline__ PieceIter(const Params& p) {
    const int64_t c = blockIdx.x;
    if (p.unit_aligned) {
      X = (c * p.n_units / p.n_ctas) * p.tiles_per_unit;
      X1 = ((c + 1) * p.n_units / p.n_ctas) * p.tiles_per_unit;
    } else {
      X = c * p.total_tiles / p.n_ctas;
      X1 = (c + 1) * p.total_tiles / p.n_ctas;
    }
  }
  __device__ __forceinline__ bool next(const Params& p, Piece& pc) {
    if (X >= X1) return false;
    const int64_t tpu = p.tiles_per_unit;
    pc.unit = X / tpu;
    const int64_t ub = pc.unit * tpu, ue = ub + tpu;
    const int64_t e = min(X1, ue);
    const int64_t nt = unit_tiles(p, pc.unit);
    pc.t_begin = min(X - ub, nt);
    pc.t_end = min(e - ub, nt);
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

__global__ void __launch_bounds__(kThreads, 1)
    fp16_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                       const Params p) {
  extern __shared__ uint8_t smem_raw[];
  grid_launch_dependents();
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), kGroupWarps);  // released by the group that consumed it
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&sm.q_full[s]), 1);
      mbar_init(smem_u32(&sm.q_empty[s]), kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // This CTA's first tile goes to L2 while the previous grid finishes (its
  // position follows from the plan alone; a prefetch reads nothing into the
  // CTA, and L2 stays coherent with that grid's writes): -0.37 us per W=512
  // launch, -0.14 at W=1024 (B=32).
  if (warp == kConsumerWarps && lane == 0) {
    const PieceIter it0(p);
    if (it0.X < it0.X1) {
      const int u0 = static_cast<int>(it0.X / p.tiles_per_unit);
      const int r0 = static_cast<int>((it0.X - int64_t(u0) * p.tiles_per_unit) * kTile);
      tma_prefetch_3d(&tmK, 0, r0, u0);
      tma_prefetch_3d(&tmK, 64, r0, u0);
      tma_prefetch_3d(&tmV, 0, r0, u0);
      tma_prefetch_3d(&tmV, 64, r0, u0);
    }
  }
  // the cache and q may come from the previous kernel of the stream: global
  // memory is read only after this wait (the barriers are initialised first:
  // -0.12 us per W=1024 launch at B=32)
  grid_dependency_wait();

  // CTA-local tile k (over all pieces in order) lives in stage k % kStages,
  // phase (k / kStages) & 1, and is consumed by group k % kGroups.
  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tmK);
      prefetch_tmap(&tmV);
      int qs = 0;
      uint32_t qphase = 0;
      uint32_t k = 0;
      PieceIter it(p);
      Piece pc;
      while (it.next(p, pc)) {
        // on a timed-out wait the producer stops issuing; consumers then time
        // out once each and finish without waiting (see below)
        if (!mbar_wait(smem_u32(&sm.q_empty[qs]), qphase ^ 1, p.err)) return;
        sm.meta[qs] = make_meta(p, pc.unit);  // published by the arrive below (release)
        mbar_arrive_expect_tx(smem_u32(&sm.q_full[qs]), kQBytes);
        bulk_load(smem_u32(sm.q[qs]), p.q + pc.unit * kGroupHeads * kHeadDim, kQBytes, smem_u32(&sm.q_full[qs]));
        if (++qs == 2) { qs = 0; qphase ^= 1; }
        const int u = static_cast<int>(pc.unit);
        for (int64_t t = pc.t_begin; t < pc.t_end; ++t, ++k) {
          const uint32_t stage = k % kStages, phase = (k / kStages) & 1;
          if (!mbar_wait(smem_u32(&sm.empty[stage]), phase ^ 1, p.err)) return;
          const uint32_t fb = smem_u32(&sm.full[stage]);
          mbar_arrive_expect_tx(fb, kStageBytes);
          const uint32_t kd = smem_u32(sm.kv[stage]);
          const int row = static_cast<int>(t * kTile);
          tma_load_3d(kd, &tmK, fb, 0, row, u);
          tma_load_3d(kd + kRegionBytes, &tmK, fb, 64, row, u);
          tma_load_3d(kd + kTileBytes, &tmV, fb, 0, row, u);
          tma_load_3d(kd + kTileBytes + kRegionBytes, &tmV, fb, 64, row, u);
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  // A timed-out wait sets `aborted`: the warp then stops waiting (the error
  // word is already set) but keeps its schedule of named barriers, so the
  // other consumer warps can never be left waiting on it.
  const int grp = warp / kGroupWarps, wq = warp % kGroupWarps;
  int qs = 0;
  uint32_t qphase = 0;
  uint32_t k = 0;
  bool aborted = false;
  const int g = lane >> 2;
  WarpAttn st;
  PieceIter it(p);
  Piece pc;
  while (it.next(p, pc)) {
    if (!aborted && !mbar_wait(smem_u32(&sm.q_full[qs]), qphase, p.err)) aborted = true;
    st.load_q(smem_u32(sm.q[qs]), lane);
    const PieceMeta meta = sm.meta[qs];
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sm.q_empty[qs]));
    if (++qs == 2) { qs = 0; qphase ^= 1; }
    st.reset();
    for (int64_t t = pc.t_begin; t < pc.t_end; ++t, ++k) {
      if ((k % kGroups) != static_cast<uint32_t>(grp)) continue;
      const uint32_t stage = k % kStages, phase = (k / kStages) & 1;
      const int64_t r0 = t * kTile + 16 * wq;
      const bool v_lo = slot_valid(p, r0 + g, meta);
      const bool v_hi = slot_valid(p, r0 + g + 8, meta);
      if (!aborted && !mbar_wait(smem_u32(&sm.full[stage]), phase, p.err)) aborted = true;
      const uint32_t kd = smem_u32(sm.kv[stage]);
      st.consume16(kd, kd + kTileBytes, kRegionBytes, 16 * wq, v_lo, v_hi, p.scale_log2, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&sm.empty[stage]));
    }

    // ---- epilogue: merge the two groups, then the warps, then write the
    // output or a split-K partial
    if (grp == 1) warp_xfer_out(st, sm.ep, wq, lane);
    consumer_sync();
    if (grp == 0) warp_xfer_in(st, sm.ep, wq, lane);
    consumer_sync();
    if (grp == 0) warp_publish(st, sm.ep, wq, lane);
    consumer_sync();
    const int ct = threadIdx.x;  // 0..255
    const int hh = ct >> 5, d0 = (ct & 31) * 4;
    float o[4], lse;
    merge_warps<4>(sm.ep, hh, d0, o, lse);
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
                       warp * kGroupHeads / kConsumerWarps, kGroupHeads / kConsumerWarps, lane);
        if (ct == 0) p.counters[pc.unit] = 0;  // ready for the next launch
      }
    }
    consumer_sync();  // epilogue buffers are reused by the next piece
  }
}

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// ---------------------------------------------------------------------------
// Short sink+window caches with at least one unit per SM: one CTA of 4 warps
// per unit, two CTAs per SM, so that every unit's tiles are requested at
// once.  The unit's S+W slots come in 96-slot tiles, K and V each as one TMA
// box holding both 64-dim halves (2-stage ring: 192 slots in flight, the rest
// as soon as the first tile is consumed); lane 0 of warp 0 issues them.  Warps
// claim 32-slot jobs as they free up (wclaim) and run the shared fp16 engine;
// the epilogue merges the 4 warps (its buffers reuse the ring).
namespace win {
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kRows = 96;
constexpr int kStages = 2;
constexpr uint32_t kRegion = kRows * 128;  // 96 slots x 64 dims fp16
constexpr uint32_t kTile = 2 * kRegion;    // K (or V) of a tile
constexpr uint32_t kStageB = 2 * kTile;    // 48 KiB
constexpr int kQPad = kHeadDim + 8;        // 272-byte query rows: conflict-free ldmatrix
constexpr int64_t kMaxSlots = 4 * kRows;   // longer caches use the persistent kernel
struct Smem {
  union {
    uint8_t kv[kStages][kStageB];  // 1024-aligned TMA destinations
    EpilogueSmem ep;               // after every tile has been consumed
  };
  __half qpad[kGroupHeads][kQPad];
  __half newtok[2][kHeadDim];  // appended token's K and V
  uint64_t full[kStages], empty[kStages];
  int job[kStages];  // next 32-slot job of the staged tile
};
static_assert(offsetof(Smem, kv) == 0 && kStageB % 1024 == 0 && kRegion % 1024 == 0, "TMA tile destinations");
static_assert(sizeof(EpilogueSmem) <= sizeof(uint8_t[kStages][kStageB]), "epilogue alias");
constexpr size_t kSmem = sizeof(Smem);
static_assert(2 * (kSmem + 1024) <= 228 * 1024, "two CTAs per SM");
__device__ __forceinline__ void sync4() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }
}  // namespace win

// The next 32-slot job of a staged tile, claimed by lane 0 for its warp from
// the stage's counter (reset when the stage is refilled): whichever warp is
// free first takes it, so the order in which a unit's partial sums accumulate
// (and the output's last rounding) can differ between launches.
__device__ __forceinline__ int wclaim(int* c, int lane) {
  int j = 0;
  if (lane == 0) j = atomicAdd(c, 1);
  return __shfl_sync(0xffffffffu, j, 0);
}
// kAppend: the launch also appends new_k / new_v (p.new_k non-null), so that
// attention alone carries none of the append code.  kWide: windows of 32
// slots or more, whose job masks are interval arithmetic only (without the
// warp vote that shorter windows take: -0.03 us per launch, -0.06 per ring
// step at W=256, B=32).
template <bool kAppend, bool kWide>
__global__ void __launch_bounds__(win::kThreads, 2)
    window_decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                         const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  grid_launch_dependents();
  // the cache and q may come from the previous kernel of the stream: global
  // memory is read only after the wait below (the barriers are initialised
  // first, which measured faster for attention alone and for append + attend)
  constexpr bool appending = kAppend;
  if (smem_u32(smem_raw) & 1023u) {  // TMA tile destinations need 1024-byte alignment
    if (threadIdx.x == 0) set_error(p.err, NSA_ERR_ALIGN);
    return;
  }
  win::Smem& sm = *reinterpret_cast<win::Smem*>(smem_raw);
  const int ct = threadIdx.x, warp = ct >> 5, lane = ct & 31, g = lane >> 2;
  const int64_t unit = blockIdx.x;
  const int n_tiles = (p.sink + p.window + win::kRows - 1) / win::kRows;
  if (ct == 0) {
    for (int s = 0; s < win::kStages; ++s) {
      mbar_init(smem_u32(&sm.full[s]), 1);
      mbar_init(smem_u32(&sm.empty[s]), win::kWarps);
      sm.job[s] = 0;
    }
    fence_barrier_init();
  }
  __syncthreads();
  // The unit's first tile goes to L2 while the previous grid finishes (a
  // prefetch reads nothing into this CTA, and L2 stays coherent with that
  // grid's writes; its load below then waits on L2).  Only the first: the
  // CTAs that start early would otherwise stream their whole unit during the
  // previous grid's own transfer (W=256, B=32: every tile 7.76 us per launch,
  // the first two 7.20, the first 7.02, none 7.85).
  if (ct == 0 && n_tiles > 0) {
    tma_prefetch_4d(&tmK, 0, 0, 0, static_cast<int>(unit));
    tma_prefetch_4d(&tmV, 0, 0, 0, static_cast<int>(unit));
  }
  // likewise the small inputs loaded right after the wait (query, lengths, ring
  // heads, appended token), so that those loads hit L2
  if (ct == 32) {
    bulk_prefetch_l2(p.q + unit * kGroupHeads * kHeadDim, kGroupHeads * kHeadDim * 2);
    if (p.unit_lens) prefetch_l2(p.unit_lens + unit);
    if (p.seq_lens) prefetch_l2(p.seq_lens + unit / p.n_kv_heads);
    if (p.ring_heads) prefetch_l2(p.ring_heads + unit / p.n_kv_heads);
    if (appending) {
      bulk_prefetch_l2(p.new_k + unit * kHeadDim, kHeadDim * 2);
      bulk_prefetch_l2(p.new_v + unit * kHeadDim, kHeadDim * 2);
    }
  }
  grid_dependency_wait();

  // Tile i uses stage i % kStages; it is issued once warp 0 itself has
  // consumed tile i - kStages (the other warps' release is then waited for).
  const bool leader = ct == 0;
  int issued = 0;
  bool issuing = true;
  auto pump = [&](int consumed) {
    while (issuing && issued < n_tiles && issued < consumed + win::kStages) {
      const uint32_t s = issued % win::kStages, ph = (issued / win::kStages) & 1;
      if (!mbar_wait(smem_u32(&sm.empty[s]), ph ^ 1, p.err)) {
        issuing = false;
        break;
      }
      const uint32_t fb = smem_u32(&sm.full[s]), sd = smem_u32(sm.kv[s]);
      sm.job[s] = 0;
      mbar_arrive_expect_tx(fb, win::kStageB);
      tma_load_4d(sd, &tmK, fb, 0, issued * win::kRows, 0, static_cast<int>(unit));
      tma_load_4d(sd + win::kTile, &tmV, fb, 0, issued * win::kRows, 0, static_cast<int>(unit));
      ++issued;
    }
  };
  const uint4 qv = __ldg(reinterpret_cast<const uint4*>(p.q + (unit * kGroupHeads + (ct >> 4)) * kHeadDim +
                                                       (ct & 15) * 8));
  // one-launch append: position pos = the unit's old length goes to slot
  // `aslot` (tile aslot / kRows); the staged tile's row is patched by the warp
  // whose job holds it, the cache slot and the length are stored at the end
  int64_t pos = 0;
  int aslot = -1;
  __half nk = __float2half_rn(0.f), nv = nk;
  if (appending) {  // the loads go out now; their results are used once the tiles are issued
    pos = p.unit_lens[unit];
    nk = p.new_k[unit * kHeadDim + ct];
    nv = p.new_v[unit * kHeadDim + ct];
  }
  if (leader) {
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    pump(0);
  }
  if (appending) {  // (using them before the issue measured 1.06 us slower per step)
    aslot = pos < p.sink ? static_cast<int>(pos)
                         : (p.window > 0 ? p.sink + static_cast<int>((pos - p.sink) % p.window) : -1);
    sm.newtok[0][ct] = nk;
    sm.newtok[1][ct] = nv;
  }
  const PieceMeta meta = make_meta(p, unit);
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(smem_u32(&sm.qpad[ct >> 4][(ct & 15) * 8])),
               "r"(qv.x), "r"(qv.y), "r"(qv.z), "r"(qv.w));
  win::sync4();

  WarpAttn st;
  st.reset();
  st.load_q(smem_u32(sm.qpad), lane, win::kQPad * 2);
  bool aborted = false;
  for (int ti = 0; ti < n_tiles; ++ti) {
    if (leader) pump(ti);
    __syncwarp();
    const uint32_t s = ti % win::kStages, ph = (ti / win::kStages) & 1;
    if (!aborted && !mbar_wait(smem_u32(&sm.full[s]), ph, p.err)) aborted = true;
    const uint32_t sd = smem_u32(sm.kv[s]);
#pragma unroll 1
    for (int jj = wclaim(&sm.job[s], lane); jj < win::kRows / 32; jj = wclaim(&sm.job[s], lane)) {
      const int r = 32 * jj;
      const int64_t r0 = int64_t(ti) * win::kRows + r;
      // valid rows of the job (bit i: row r + i): uniform arithmetic, or one vote for windows below 32
      const uint32_t vm = kWide ? window_slot_mask(p, static_cast<int>(r0), meta)
                                         : __ballot_sync(0xffffffffu, slot_valid(p, r0 + lane, meta));
      if (!vm) continue;
      bool vl[2], vh[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        vl[h] = ((vm >> (16 * h + g)) & 1u) != 0;
        vh[h] = ((vm >> (16 * h + g + 8)) & 1u) != 0;
      }
      const bool any0 = (vm & 0xffffu) != 0, any1 = (vm >> 16) != 0;
      if (aslot >= r0 && aslot < r0 + 32) {  // the appended token's staged row is stale
        const int row = aslot - ti * win::kRows, kv = lane >> 4, chunk = lane & 15;
        uint4 x = *reinterpret_cast<const uint4*>(&sm.newtok[kv][chunk * 8]);
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sd + kv * win::kTile + (chunk >> 3) * win::kRegion +
                                                                    swz128(row, chunk & 7)),
                     "r"(x.x), "r"(x.y), "r"(x.z), "r"(x.w));
        fence_proxy_async_smem();
        __syncwarp();
      }
      if (any0 && any1) {
        st.consume_rows<2>(sd, sd + win::kTile, win::kRegion, r, vl, vh, p.scale_log2, lane);
      } else {
        // (selects, not vl[h]: a dynamic index would put the flags in local memory)
        const bool l1[1] = {any0 ? vl[0] : vl[1]}, h1[1] = {any0 ? vh[0] : vh[1]};
        st.consume_rows<1>(sd, sd + win::kTile, win::kRegion, r + (any0 ? 0 : 16), l1, h1, p.scale_log2, lane);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&sm.empty[s]));
  }

  // ---- epilogue: merge the 4 warps
  win::sync4();
  warp_publish(st, sm.ep, warp, lane);
  win::sync4();
  const int hh = ct >> 4, d0 = (ct & 15) * 8;  // this thread's head and 8 dims
  float o8[8], lse;
  merge_warps<8>(sm.ep, hh, d0, o8, lse);
  store_half8(p.o + unit * kGroupHeads * kHeadDim + hh * kHeadDim + d0, o8);
  if (appending) {  // every thread read the old length at entry
    const int64_t cap = p.sink + p.window;
    if (aslot >= 0) {
      p.k_w[(unit * cap + aslot) * kHeadDim + ct] = sm.newtok[0][ct];
      p.v_w[(unit * cap + aslot) * kHeadDim + ct] = sm.newtok[1][ct];
    }
    if (ct == 0) p.unit_lens[unit] = pos + 1;
  }
}

// Append without attention (ring cache, any launch shape): one CTA of 128
// threads (thread = channel) per unit stores the token and advances the length.
__global__ void ring_append_kernel(__half* k, __half* v, int64_t* unit_lens, const __half* new_k, const __half* new_v,
                                   int sink, int window) {
  grid_launch_dependents();
  grid_dependency_wait();  // the previous kernel may still read this cache
  const int64_t u = blockIdx.x;
  const int c = threadIdx.x;
  const int64_t pos = unit_lens[u];
  const int64_t cap = sink + window;
  const int64_t slot = pos < sink ? pos : (window > 0 ? sink + (pos - sink) % window : -1);
  if (slot >= 0) {
    k[(u * cap + slot) * kHeadDim + c] = new_k[u * kHeadDim + c];
    v[(u * cap + slot) * kHeadDim + c] = new_v[u * kHeadDim + c];
  }
  __syncthreads();  // every thread has read the length
  if (c == 0) unit_lens[u] = pos + 1;
}

// Whether a sink+window launch uses window_decode_kernel: short caches, at
// any number of units -- with fewer units than SMs too, one CTA per unit beats
// splitting the units over the SMs (W=256: B=8 11.5 -> 5.3 us, B=1 7.8 -> 4.3
// us per launch; a ring step also keeps its append in the launch).
// NSA_SPARSE_KERNEL=persistent forces the other kernel.
bool use_window_kernel(int64_t n_units, int64_t slots) {
  const char* env = getenv("NSA_SPARSE_KERNEL");
  if (env && env[0] == 'p') return false;
  return n_units >= 1 && slots <= win::kMaxSlots && n_units <= 0x7fffffff;
}

int launch_window(Params& p, int64_t n_units, const void* k, const void* v, int64_t cap, cudaStream_t stream) {
  if (n_units == 0) return NSA_OK;
  p.n_units = n_units;
  p.err = device_error_word();
  if (!p.err) return fail(NSA_ERR_CUDA, "device error word unavailable");
  // cache [units][cap][128] viewed as [units][2 halves][cap][64] (dims innermost first)
  CUtensorMap mk, mv;
  const uint64_t dims[4] = {64, static_cast<uint64_t>(cap), 2, static_cast<uint64_t>(n_units)};
  const uint64_t strides[3] = {kHeadDim * 2, 128, static_cast<uint64_t>(cap) * kHeadDim * 2};
  const uint32_t box[4] = {64, win::kRows, 2, 1};
  int rc = encode_tiled(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tiled(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool attr_set[64] = {false};
  const int dev = current_device().device;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaSuccess;
    for (auto kern : {window_decode_kernel<false, false>, window_decode_kernel<true, false>,
                      window_decode_kernel<false, true>, window_decode_kernel<true, true>})
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(win::kSmem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    attr_set[dev] = true;
  }
  const bool wide = p.window >= 32;
  auto kern = p.new_k ? (wide ? window_decode_kernel<true, true> : window_decode_kernel<true, false>)
                      : (wide ? window_decode_kernel<false, true> : window_decode_kernel<false, false>);
  cudaError_t e = launch_kernel(kern, dim3(static_cast<unsigned>(n_units)), dim3(win::kThreads), win::kSmem, stream,
                                mk, mv, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "window_decode_kernel launch");
  return NSA_OK;
}

struct Split {
  int64_t n_units, tiles_per_unit, total_tiles;
  int n_ctas, max_pieces, unit_aligned;
};

// Units of at most this many tiles (1 MiB of K+V) are not split when there
// are at least as many units as CTAs: a short launch is dominated by fixed
// per-piece costs (fence, ticket, cross-SM combine), and one SM can stream
// two such units at well above its fair share of HBM bandwidth.
constexpr int64_t kWholeUnitMaxTiles = 32;

Split plan(int64_t n_units, int64_t range_slots) {
  Split s;
  s.n_units = n_units;
  s.tiles_per_unit = range_slots > 0 ? (range_slots + kTile - 1) / kTile : 1;
  s.total_tiles = n_units * s.tiles_per_unit;
  if (s.total_tiles == 0) {  // empty batch: nothing to split (and nothing is launched)
    s.n_ctas = 1;
    s.max_pieces = 1;
    s.unit_aligned = 1;
    return s;
  }
  const int sms = current_device().sm_count > 0 ? current_device().sm_count : 148;
  s.n_ctas = static_cast<int>(s.total_tiles < sms ? s.total_tiles : sms);
  if (s.n_ctas < 1) s.n_ctas = 1;
  const char* env = getenv("NSA_SPLIT_MODE");  // "stream" / "unit": tuning override
  // Whole units also when the imbalance is mild: the busiest CTA then holds
  // at most 25% more than the mean, which the idle SMs' bandwidth absorbs.
  const int64_t per_cta = (n_units + sms - 1) / sms;
  bool whole = n_units >= sms && (s.tiles_per_unit <= kWholeUnitMaxTiles || per_cta * sms * 4 <= n_units * 5);
  if (env && env[0] == 's') whole = false;
  if (env && env[0] == 'u' && n_units >= sms) whole = true;
  s.unit_aligned = whole ? 1 : 0;
  if (whole) {
    s.n_ctas = sms;
    s.max_pieces = 1;
    return s;
  }
  // a unit spans at most ceil(tpu * ctas / total) + 1 slices
  int64_t mp = (s.tiles_per_unit * s.n_ctas + s.total_tiles - 1) / s.total_tiles + 1;
  if (mp > s.tiles_per_unit) mp = s.tiles_per_unit;
  s.max_pieces = static_cast<int>(mp);
  return s;
}

size_t workspace_bytes(const Split& s) {
  const size_t counters = ((s.n_units * sizeof(int)) + 255) & ~size_t(255);
  const size_t pieces = static_cast<size_t>(s.n_units) * s.max_pieces;
  const size_t lse = ((pieces * kGroupHeads * sizeof(float)) + 255) & ~size_t(255);
  return counters + lse + pieces * kGroupHeads * kHeadDim * sizeof(float);
}

int check_common(const void* q, const void* k, const void* v, const void* o, int64_t batch, int64_t n_heads,
                 int64_t n_kv_heads, int64_t head_dim) {
  if (batch < 0 || n_kv_heads <= 0) return fail(NSA_ERR_INVALID, "batch must be >= 0 and n_kv_heads > 0");
  // an empty batch reads and writes nothing: its (empty) tensors may be NULL
  if (batch > 0 && (!q || !k || !v || !o)) return fail(NSA_ERR_INVALID, "null tensor pointer");
  if (head_dim != kHeadDim) return fail(NSA_ERR_UNSUPPORTED, "head_dim must be 128 (got %lld)", (long long)head_dim);
  if (n_heads != n_kv_heads * kGroupHeads)
    return fail(NSA_ERR_UNSUPPORTED, "n_heads must be 8 * n_kv_heads (got %lld, %lld)", (long long)n_heads,
                (long long)n_kv_heads);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(NSA_ERR_ALIGN, "q, k, v and o must be 16-byte aligned");
  if (batch * n_kv_heads > (int64_t(1) << 31) - 1) return fail(NSA_ERR_UNSUPPORTED, "batch * n_kv_heads too large");
  return NSA_OK;
}

// Whether a launch of plan s over `cap` slots touches the split-K scratch
// (tickets and partials): only the persistent kernel with some unit split
// over several CTAs does; the window kernel and whole-unit plans store every
// output directly.
bool uses_scratch(const Params& p, const Split& s, int64_t cap) {
  if (p.mode == kSparse && use_window_kernel(s.n_units, cap)) return false;
  return s.max_pieces > 1;
}

int launch(Params& p, const Split& s, const void* k, const void* v, int64_t cap, void* ws, size_t ws_bytes,
           cudaStream_t stream) {
  if (s.n_units == 0) return NSA_OK;
  if (p.mode == kSparse && use_window_kernel(s.n_units, cap)) return launch_window(p, s.n_units, k, v, cap, stream);
  if (cap > (int64_t(1) << 31) - kTile) return fail(NSA_ERR_UNSUPPORTED, "cache length too large for TMA coordinates");
  if (uses_scratch(p, s, cap)) {
    const size_t need = workspace_bytes(s);
    if (!ws || ws_bytes < need)
      return fail(NSA_ERR_WORKSPACE, "workspace of %zu bytes required (got %zu)", need, ws ? ws_bytes : size_t(0));
    if (!aligned16(ws)) return fail(NSA_ERR_ALIGN, "workspace must be 16-byte aligned");
    uint8_t* w = static_cast<uint8_t*>(ws);
    const size_t counters = ((s.n_units * sizeof(int)) + 255) & ~size_t(255);
    const size_t pieces = static_cast<size_t>(s.n_units) * s.max_pieces;
    const size_t lse = ((pieces * kGroupHeads * sizeof(float)) + 255) & ~size_t(255);
    p.counters = reinterpret_cast<int*>(w);
    p.part_lse = reinterpret_cast<float*>(w + counters);
    p.part_o = reinterpret_cast<float*>(w + counters + lse);
  } else {  // whole units: every piece stores its output directly
    p.counters = nullptr;
    p.part_lse = nullptr;
    p.part_o = nullptr;
  }
  p.n_units = s.n_units;
  p.tiles_per_unit = s.tiles_per_unit;
  p.total_tiles = s.total_tiles;
  p.n_ctas = s.n_ctas;
  p.max_pieces = s.max_pieces;
  p.unit_aligned = s.unit_aligned;
  p.err = device_error_word();
  if (!p.err) return fail(NSA_ERR_CUDA, "device error word unavailable");

  CUtensorMap mk, mv;
  const uint64_t dims[3] = {static_cast<uint64_t>(kHeadDim), static_cast<uint64_t>(cap),
                            static_cast<uint64_t>(s.n_units)};
  const uint64_t strides[2] = {kHeadDim * 2, static_cast<uint64_t>(cap) * kHeadDim * 2};
  const uint32_t box[3] = {64, kTile, 1};
  int rc = encode_tiled(&mk, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tiled(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  static bool attr_set[64] = {false};
  const int dev = current_device().device;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fp16_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    attr_set[dev] = true;
  }
  cudaError_t e = launch_kernel(fp16_decode_kernel, dim3(s.n_ctas), dim3(kThreads), kSmemBytes, stream, mk, mv, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "fp16_decode_kernel launch");
  return NSA_OK;
}

// Parameters shared by the sink+window entry points.
int sparse_params(const void* q, const void* k, const void* v, const void* o, int64_t batch, int64_t n_heads,
                  int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink, float sm_scale, Params& p) {
  int rc = check_common(q, k, v, o, batch, n_heads, n_kv_heads, head_dim);
  if (rc) return rc;
  if (window < 0 || sink < 0 || window + sink < 1 || window + sink > (int64_t(1) << 30))
    return fail(NSA_ERR_INVALID, "need window, sink >= 0 and 1 <= window + sink <= 2^30");
  p = Params{};
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(const_cast<void*>(o));
  p.n_kv_heads = static_cast<int>(n_kv_heads);
  p.mode = kSparse;
  p.window = static_cast<int>(window);
  p.sink = static_cast<int>(sink);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  return NSA_OK;
}

}  // namespace
}  // namespace nsa

using namespace nsa;

extern "C" {

size_t nsa_dense_workspace_bytes(int64_t batch, int64_t n_kv_heads, int64_t seq_len) {
  if (batch < 0 || n_kv_heads <= 0 || seq_len < 0) return 0;
  return workspace_bytes(plan(batch * n_kv_heads, seq_len));
}

int nsa_dense_decode(const void* q, const void* k, const void* v, void* o, int64_t batch, int64_t n_heads,
                     int64_t n_kv_heads, int64_t head_dim, int64_t cache_len, int64_t seq_len, float sm_scale,
                     void* workspace, size_t workspace_bytes_, nsa_stream_t stream) {
  clear_error();
  int rc = check_common(q, k, v, o, batch, n_heads, n_kv_heads, head_dim);
  if (rc) return rc;
  if (seq_len < 0 || cache_len < 1 || seq_len > cache_len)
    return fail(NSA_ERR_INVALID, "need 0 <= seq_len <= cache_len and cache_len >= 1 (got %lld, %lld)",
                (long long)seq_len, (long long)cache_len);
  Params p{};
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(o);
  p.n_kv_heads = static_cast<int>(n_kv_heads);
  p.mode = kDense;
  p.seq_len = seq_len;
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  const Split s = plan(batch * n_kv_heads, seq_len);
  return launch(p, s, k, v, cache_len, workspace, workspace_bytes_, stream);
}

size_t nsa_sparse_workspace_bytes(int64_t batch, int64_t n_kv_heads, int64_t window, int64_t sink) {
  if (batch < 0 || n_kv_heads <= 0 || window < 0 || sink < 0) return 0;
  return workspace_bytes(plan(batch * n_kv_heads, window + sink));
}

int nsa_sparse_decode(const void* q, const void* k_cache, const void* v_cache, void* o, int64_t batch,
                      int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink,
                      int64_t seq_len, const int64_t* seq_lens, const int32_t* ring_heads, float sm_scale,
                      void* workspace, size_t workspace_bytes_, nsa_stream_t stream) {
  clear_error();
  Params p{};
  int rc = sparse_params(q, k_cache, v_cache, o, batch, n_heads, n_kv_heads, head_dim, window, sink, sm_scale, p);
  if (rc) return rc;
  if (seq_len < 0) return fail(NSA_ERR_INVALID, "seq_len must be >= 0");
  p.seq_len = seq_len;
  p.seq_lens = seq_lens;
  p.ring_heads = ring_heads;
  const Split s = plan(batch * n_kv_heads, window + sink);
  return launch(p, s, k_cache, v_cache, window + sink, workspace, workspace_bytes_, stream);
}

int nsa_ring_append(void* k_cache, void* v_cache, int64_t* unit_lens, const void* new_k, const void* new_v,
                    int64_t batch, int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink,
                    nsa_stream_t stream) {
  clear_error();
  if (batch > 0 && (!k_cache || !v_cache || !unit_lens || !new_k || !new_v))
    return fail(NSA_ERR_INVALID, "null pointer");
  if (head_dim != kHeadDim) return fail(NSA_ERR_UNSUPPORTED, "head_dim must be 128");
  if (batch < 0 || n_kv_heads <= 0 || window < 0 || sink < 0 || window + sink < 1 ||
      window + sink > (int64_t(1) << 30))
    return fail(NSA_ERR_INVALID, "need batch >= 0, n_kv_heads > 0, window, sink >= 0, 1 <= window + sink <= 2^30");
  const int64_t units = batch * n_kv_heads;
  if (units == 0) return NSA_OK;
  if (units > 0x7fffffff) return fail(NSA_ERR_UNSUPPORTED, "too many units");
  cudaError_t e = launch_kernel(ring_append_kernel, dim3(static_cast<unsigned>(units)), dim3(kHeadDim), 0, stream,
                                static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), unit_lens,
                                static_cast<const __half*>(new_k), static_cast<const __half*>(new_v),
                                static_cast<int>(sink), static_cast<int>(window));
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? NSA_OK : cuda_fail(e, "ring_append_kernel launch");
}

int nsa_ring_decode(const void* q, const void* k_cache, const void* v_cache, void* o, int64_t batch, int64_t n_heads,
                    int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink, const int64_t* unit_lens,
                    float sm_scale, void* workspace, size_t workspace_bytes_, nsa_stream_t stream) {
  clear_error();
  if (batch > 0 && !unit_lens) return fail(NSA_ERR_INVALID, "unit_lens must not be NULL");
  Params p{};
  int rc = sparse_params(q, k_cache, v_cache, o, batch, n_heads, n_kv_heads, head_dim, window, sink, sm_scale, p);
  if (rc) return rc;
  p.unit_lens = const_cast<int64_t*>(unit_lens);  // read only without new_k
  const Split s = plan(batch * n_kv_heads, window + sink);
  return launch(p, s, k_cache, v_cache, window + sink, workspace, workspace_bytes_, stream);
}

int nsa_ring_decode_step(const void* q, void* k_cache, void* v_cache, void* o, int64_t batch, int64_t n_heads,
                         int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink, int64_t* unit_lens,
                         const void* new_k, const void* new_v, float sm_scale, void* workspace,
                         size_t workspace_bytes_, nsa_stream_t stream) {
  clear_error();
  if (batch > 0 && (!unit_lens || !new_k || !new_v)) return fail(NSA_ERR_INVALID, "null pointer");
  if (!aligned16(new_k) || !aligned16(new_v)) return fail(NSA_ERR_ALIGN, "new_k and new_v must be 16-byte aligned");
  Params p{};
  int rc = sparse_params(q, k_cache, v_cache, o, batch, n_heads, n_kv_heads, head_dim, window, sink, sm_scale, p);
  if (rc) return rc;
  const Split s = plan(batch * n_kv_heads, window + sink);
  if (use_window_kernel(s.n_units, window + sink)) {  // one launch: the decode CTA of each unit appends
    p.unit_lens = unit_lens;
    p.new_k = static_cast<const __half*>(new_k);
    p.new_v = static_cast<const __half*>(new_v);
    p.k_w = static_cast<__half*>(k_cache);
    p.v_w = static_cast<__half*>(v_cache);
    return launch_window(p, s.n_units, k_cache, v_cache, window + sink, stream);
  }
  rc = nsa_ring_append(k_cache, v_cache, unit_lens, new_k, new_v, batch, n_kv_heads, head_dim, window, sink, stream);
  if (rc) return rc;
  return nsa_ring_decode(q, k_cache, v_cache, o, batch, n_heads, n_kv_heads, head_dim, window, sink, unit_lens,
                         sm_scale, workspace, workspace_bytes_, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Sink + window decode that allocates nothing.
//
// Some callers cannot call cudaMalloc, or allocate through torch, at the point
// where they decode: a host runtime that reserves all device memory up front
// through its own pool and does not let libraries allocate, a plain C caller
// that owns no device allocator, or a decode loop where an allocation (which
// may synchronize the device) is not acceptable.  For them the split-K scratch
// of nsa_sparse_decode (tickets and partial results) lives in the static
// device array below instead of a caller-provided workspace.
//
// Facts a caller must know:
// * The array is kNoAllocScratchBytes (4 MiB) per GPU, held by every GPU that
//   loads this library until the process exits.  Only plans that split a unit
//   over several CTAs use it; among those, shapes whose scratch does not fit
//   are rejected with NSA_ERR_UNSUPPORTED before anything is launched.  Plans
//   that keep units whole (the window kernel, whole-unit persistent plans)
//   never touch it and have no size limit.
// * The first call on a device that uses the array looks up its device
//   address (cudaGetSymbolAddress) and clears it (cudaMemset); make that first
//   call before any stream capture.  Later calls on the device do neither, and
//   an empty batch returns before any CUDA call.
// * Every call on a device shares the one array.  The kernel leaves the parts
//   it used zeroed again, but calls that overlap on the GPU (different streams
//   without ordering) race on it and may return wrong results.  After a call
//   reported NSA_ERR_TIMEOUT through nsa_device_error, the array may hold
//   stale tickets; the next first-use set-up does not run again, so such a
//   process should not keep using this entry point.
// ---------------------------------------------------------------------------
namespace nsa {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_scratch on the current device, set up (address
// lookup + clear) on first use; nullptr (with a message recorded) on failure.
void* noalloc_scratch() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    fail(NSA_ERR_CUDA, "no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
      return nullptr;
    }
    e = cudaMemset(ptr, 0, kNoAllocScratchBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      cuda_fail(e, "clearing g_noalloc_scratch");
      return nullptr;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace nsa

extern "C" {

int nsa_sparse_decode_noalloc(const void* q, const void* k_cache, const void* v_cache, void* o, int64_t batch,
                              int64_t n_heads, int64_t n_kv_heads, int64_t head_dim, int64_t window, int64_t sink,
                              int64_t seq_len, const int64_t* seq_lens, const int32_t* ring_heads, float sm_scale,
                              nsa_stream_t stream) {
  clear_error();
  int rc = check_common(q, k_cache, v_cache, o, batch, n_heads, n_kv_heads, head_dim);
  if (rc) return rc;
  if (window < 0 || sink < 0 || window + sink < 1 || window + sink > (int64_t(1) << 30))
    return fail(NSA_ERR_INVALID, "need window, sink >= 0 and 1 <= window + sink <= 2^30");
  if (seq_len < 0) return fail(NSA_ERR_INVALID, "seq_len must be >= 0");
  if (batch * n_kv_heads == 0) return NSA_OK;  // nothing to do: no set-up, no CUDA call
  const Split s = plan(batch * n_kv_heads, window + sink);
  Params p{};
  p.q = static_cast<const __half*>(q);
  p.o = static_cast<__half*>(o);
  p.n_kv_heads = static_cast<int>(n_kv_heads);
  p.mode = kSparse;
  p.seq_len = seq_len;
  p.seq_lens = seq_lens;
  p.ring_heads = ring_heads;
  p.window = static_cast<int>(window);
  p.sink = static_cast<int>(sink);
  p.scale_log2 = sm_scale * 1.4426950408889634f;
  // Only plans that split a unit over several CTAs use scratch; the others
  // (the window kernel, whole units) need neither the array nor its size limit.
  if (!uses_scratch(p, s, window + sink)) return launch(p, s, k_cache, v_cache, window + sink, nullptr, 0, stream);
  const size_t need = workspace_bytes(s);
  if (need > kNoAllocScratchBytes)
    return fail(NSA_ERR_UNSUPPORTED,
                "this shape needs %zu bytes of split-K scratch; the allocation-free entry point has %zu "
                "(use nsa_sparse_decode with a workspace)",
                need, kNoAllocScratchBytes);
  void* scratch = noalloc_scratch();
  if (!scratch) return NSA_ERR_CUDA;
  return launch(p, s, k_cache, v_cache, window + sink, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
