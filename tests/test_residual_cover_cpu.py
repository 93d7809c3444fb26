"""The copy cover of the KIVI streaming cache's residual tiles, restated in
Python with the same integer arithmetic (CPU only).

When the window is shorter than the residual, a launch copies from each
80-slot F-tile only the physical slots [lo, hi) covering the slots it reads:
the attended ring segment -- n_res - res_skip slots from res_head + res_skip,
modulo res_cap -- and, when the launch flushes a group, that group's 32 slots
(attended_cover and Issuer::first_f_sized in csrc/kivi_attn.cu).  These tests
check that the cover holds every slot read and never reaches outside the
tile, for every ring position the streaming geometry produces (its per-length
metadata as make_meta computes it), so that a sized copy can never leave an
attended row unloaded.  The GPU tests check the kernels themselves at W=32
and W=64."""

F_ROWS = 80


def _meta(length, S, W, R):
    """make_meta (streaming layout): res_head, n_res, res_skip of a unit of
    `length` tokens with sink S, window W and residual R."""
    C = R + 32
    n_stream = length - S if length > S else 0
    F = (n_stream - R) >> 5 if n_stream > R else 0
    first = max(length - W, S)
    n_res = n_stream - 32 * F
    res_head = (32 * F) % C
    res_skip = min(max(first - S - 32 * F, 0), n_res)
    return res_head, n_res, res_skip


def _cover(C, head, skip, n_res, a, b):
    """attended_cover: physical slots [lo, hi) within [a, b) covering the
    attended ring segment (lo >= hi: none)."""
    n = n_res - skip
    s0 = head + skip
    if s0 >= C:
        s0 -= C
    lo, hi = b, a
    if n <= 0:
        return lo, hi
    x, y = max(s0, a), min(min(s0 + n, C), b)
    if x < y:
        lo, hi = x, y
    y = min(s0 + n - C, b)
    if a < y:
        lo, hi = min(lo, a), max(hi, y)
    return lo, hi


def _attended(C, head, skip, n_res):
    return {(head + d) % C for d in range(skip, n_res)}


def test_cover_holds_every_attended_slot_and_stays_in_its_tile():
    S = 4
    for R in (32, 64, 128):
        C = R + 32
        for W in (0, 1, 16, 32, 64, 96, R - 32):
            if W < 0 or W >= R:
                continue
            for length in list(range(0, S + R + 5 * 32 + 3)) + [163_840 + j for j in range(40)]:
                head, n_res, skip = _meta(length, S, W, R)
                att = _attended(C, head, skip, n_res)
                assert len(att) == max(n_res - skip, 0) <= W + 1
                for f in range((C + F_ROWS - 1) // F_ROWS):
                    a, b = f * F_ROWS, min(f * F_ROWS + F_ROWS, C)
                    lo, hi = _cover(C, head, skip, n_res, a, b)
                    inside = {x for x in att if a <= x < b}
                    if not inside:
                        assert lo >= hi or (a <= lo and hi <= b), (R, W, length, f)
                        continue
                    assert a <= lo < hi <= b, (R, W, length, f)
                    assert all(lo <= x < hi for x in inside), (R, W, length, f, lo, hi)


def test_cover_is_tight_when_the_segment_does_not_wrap_in_the_tile():
    """A segment that stays in one piece within the tile is covered exactly:
    the copy moves no slot it does not read."""
    C = 160
    for head in range(0, C, 7):
        for n_res in range(0, 64):
            for skip in range(0, n_res + 1, 5):
                att = _attended(C, head, skip, n_res)
                for f in range(2):
                    a, b = f * F_ROWS, f * F_ROWS + F_ROWS
                    inside = sorted(x for x in att if a <= x < b)
                    if not inside or inside[-1] - inside[0] + 1 != len(inside):
                        continue
                    lo, hi = _cover(C, head, skip, n_res, a, b)
                    assert (lo, hi) == (inside[0], inside[-1] + 1), (head, n_res, skip, f)
