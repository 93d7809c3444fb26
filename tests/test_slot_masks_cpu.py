"""The warp-uniform slot masks of the decode kernels, restated in Python with
the same integer arithmetic, equal the per-slot validity rules they replace
(CPU only):

* window_slot_mask (csrc/decode_fp16.cu) against the sink+window rule of
  sparse_kernel.py:15-46 plus the ring head (oracle.attention.slot_validity),
  for windows of at least 32 slots (the kernel votes per lane below that);
* res_slot_mask (csrc/kivi_attn.cu) against the streaming KIVI residual
  ring's rule: slot r is attended iff r < res_cap and
  res_skip <= (r - res_head) mod res_cap < n_res.

The GPU parity tests check the kernels themselves; this pins the interval
arithmetic over many more (length, head, window) cases than they reach."""
from oracle.attention import slot_validity


def _bit_range(lo, hi):
    lo, hi = max(lo, 0), min(hi, 32)
    if lo >= hi:
        return 0
    below = 0xFFFFFFFF if hi >= 32 else (1 << hi) - 1
    return below & ~((1 << lo) - 1) & 0xFFFFFFFF


def _window_mask(S, W, length, head, n_inv, r0):
    ns = length if length < S else S
    mk = _bit_range(0, ns - r0)
    i0 = max(S - r0, 0)
    if i0 < 32:
        a = r0 + i0 - S - head
        if a < 0:
            a += W
        wrap = i0 + W - a
        mk |= _bit_range(i0 + n_inv - a, wrap) & _bit_range(i0, 32)
        mk |= _bit_range(wrap + n_inv, 32)
        mk &= _bit_range(0, S + W - r0)
    return mk


def _res_mask(C, head, skip, n_res, r0):
    a = r0 - head
    if a < 0:
        a += C
    mk = _bit_range(skip - a, n_res - a) & _bit_range(0, C - a)
    mk |= _bit_range(skip + C - a, n_res + C - a) & _bit_range(C - a, 32)
    return mk & _bit_range(0, C - r0)


def test_window_slot_mask_matches_slot_rule():
    for S in (0, 1, 4, 7):
        for W in (32, 33, 64, 100, 256, 380 - S):
            for length in list(range(0, S + W + 40, 3)) + [163_840, 163_841]:
                head = (length - S) % W if length > S else 0
                n_inv = min(max(S - (length - W), 0), W)
                ref = slot_validity(length, W, S, head)
                for r0 in range(0, S + W, 32):
                    mk = _window_mask(S, W, length, head, n_inv, r0)
                    for i in range(32):
                        s = r0 + i
                        assert bool((mk >> i) & 1) == (bool(ref[s]) if s < S + W else False), (S, W, length, s)


def test_residual_slot_mask_matches_ring_rule():
    for C in (64, 160, 288, 416):
        for head in range(0, C, 32):
            for n_res in range(0, C + 1, 7):
                for skip in range(0, n_res + 1, 9):
                    for r0 in range(0, C + 40, 16):
                        mk = _res_mask(C, head, skip, n_res, r0)
                        for i in range(32):
                            r = r0 + i
                            d = (r - head) % C
                            want = r < C and skip <= d < n_res
                            assert bool((mk >> i) & 1) == want, (C, head, n_res, skip, r)
