"""The attention's tail schedule (lbw_attention_tail_plan / lbw_chunk_attention_tail, csrc/attn.cu) on the host:
the plan the C library picks at the c4 row counts, and the kernel's block -> (window, key range, workspace rows)
decode restated here, checked to cover every key tile of every window exactly once with the cut windows' rows
inside the workspace the plan sizes. No GPU needed: without one the plan uses the B200's 148 SMs."""
import ctypes

import pytest

import lbw_b200._lib as L

SMS = 148
WINDOW_ROWS = 256  # one head's pair of 128-row query tiles


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__
    __graft_entry__.build()
    return L.load()


def plan(lib, q_rows, heads, chunk_rows, pieces=0):
    n = len(chunk_rows)
    rows = (ctypes.c_int * n)(*chunk_rows)
    n_tail, used = ctypes.c_int(-1), ctypes.c_int(-1)
    rc = lib.lbw_attention_tail_plan(q_rows, heads, rows, n, pieces, ctypes.byref(n_tail), ctypes.byref(used))
    return rc, n_tail.value, used.value


def decode(b, n_dp, n_tail, pieces, n_tiles, windows_per_head):
    """The kernel's decode of block b (chunk_attn_kernel, pieces > 0 schedule)."""
    w, g0, g1, part_row0 = b, 0, n_tiles, -1
    if w >= n_dp:
        t, p = (w - n_dp) % n_tail, (w - n_dp) // n_tail
        w = n_dp + t
        g0, g1 = p * n_tiles // pieces, (p + 1) * n_tiles // pieces
        part_row0 = (p * n_tail + t) * WINDOW_ROWS
    return w // windows_per_head, w % windows_per_head, g0, g1, part_row0


@pytest.mark.parametrize("q_rows,heads,chunk_rows,want", [
    (10800, 40, [10800] * 7, (92, 3)),    # 1 GPU at c4: 1,720 windows = 11 waves + 92
    (1350, 40, [10800] * 7, (92, 3)),     # 8 ranks: 240 windows = 148 + 92
    (2700, 40, [10800] * 7, (0, 1)),      # 4 ranks: 440 windows, the last wave 144 of 148 full: nothing cut
    (5400, 40, [10800] * 7, (0, 1)),      # 2 ranks: 880 windows, last wave 140 of 148
    (4680, 12, [4680] * 3, (80, 3)),      # c1: 228 windows = 148 + 80 of 110 key tiles: 2 waves of thirds
])
def test_tail_plan_at_the_configs(lib, q_rows, heads, chunk_rows, want):
    rc, n_tail, used = plan(lib, q_rows, heads, chunk_rows)
    assert rc == L.LBW_OK
    assert (n_tail, used) == want


def test_tail_plan_explicit_pieces_and_errors(lib):
    assert plan(lib, 10800, 40, [10800] * 7, 1) == (L.LBW_OK, 0, 1)       # one piece = whole windows
    assert plan(lib, 10800, 40, [10800] * 7, 8) == (L.LBW_OK, 92, 8)
    assert plan(lib, 300, 75, [200, 77, 500], 7) == (L.LBW_OK, 2, 7)     # 150 windows: 2 past the first wave
    rc, _, _ = plan(lib, 300, 75, [200, 77, 500], 8)                     # 7 key tiles
    assert rc == L.LBW_ERR_SHAPE and "pieces" in L.last_error()
    rc, _, _ = plan(lib, 300, 75, [200, 0, 500], 0)
    assert rc == L.LBW_ERR_SHAPE


@pytest.mark.parametrize("q_rows,heads,chunk_rows,pieces", [
    (10800, 40, [10800] * 7, 0), (1350, 40, [10800] * 7, 0), (1350, 40, [10800] * 7, 16), (300, 75, [200, 77, 500], 7),
    (70, 2, [128, 77], 0), (4680, 12, [4680] * 3, 5), (129, 3, [1000], 0), (1, 1, [1], 0),
])
def test_tail_decode_covers_each_key_tile_once(lib, q_rows, heads, chunk_rows, pieces):
    rc, n_tail, used = plan(lib, q_rows, heads, chunk_rows, pieces)
    assert rc == L.LBW_OK
    n_tiles = sum((r + 127) // 128 for r in chunk_rows)
    per_head = (q_rows + WINDOW_ROWS - 1) // WINDOW_ROWS
    n_windows = per_head * heads
    assert n_tail == (0 if used == 1 else n_windows % SMS)
    n_dp = n_windows - n_tail
    grid = n_dp + n_tail * used
    seen = {}
    rows_used = set()
    for b in range(grid):
        head, pair, g0, g1, part_row0 = decode(b, n_dp, n_tail, used, n_tiles, per_head)
        assert 0 <= head < heads and 0 <= pair < per_head and 0 <= g0 < g1 <= n_tiles
        seen.setdefault((head, pair), []).append((g0, g1))
        if part_row0 >= 0:
            assert 0 <= part_row0 and part_row0 + WINDOW_ROWS <= n_tail * used * WINDOW_ROWS
            assert part_row0 not in rows_used
            rows_used.add(part_row0)
        else:
            assert b < n_dp
    assert len(seen) == n_windows
    for ranges in seen.values():
        ranges.sort()
        assert ranges[0][0] == 0 and ranges[-1][1] == n_tiles
        assert all(a[1] == c[0] for a, c in zip(ranges, ranges[1:]))
    # whole windows come first: the cut pieces are dispatched after every whole window
    assert all(len(seen[divmod(w, per_head)]) == 1 for w in range(n_dp))
