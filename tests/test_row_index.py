"""mod_segments -> per-row modulation-table index (h3b.fuse.row_index), CPU.

The reference builds the index in _row_index (comfyui_nodes/h3-fuse-graph/
h3_fuse_patch.py:32-56): the (start, stop, row) segments are sorted by start,
must tile 0..s with no gap and no overlap, `row` is an int (every row of the
segment) or an integer tensor with one entry per row; anything else returns
None and the patched forward falls back to the original (:107-109).
"""
import pytest
import torch

h3b = pytest.importorskip("h3b")
from h3b.fuse import row_index  # noqa: E402

CPU = torch.device("cpu")


def test_int_rows_tile_in_order():
    r = row_index([(0, 3, 0), (3, 5, 2), (5, 9, 1)], 9, CPU)
    assert r.dtype == torch.int32 and r.tolist() == [0, 0, 0, 2, 2, 1, 1, 1, 1]


def test_unsorted_segments_are_sorted_by_start():
    r = row_index([(5, 9, 1), (0, 3, 0), (3, 5, 2)], 9, CPU)
    assert r.tolist() == [0, 0, 0, 2, 2, 1, 1, 1, 1]


def test_per_row_tensor_entries():
    row = torch.tensor([4, 3, 2], dtype=torch.int64)
    r = row_index([(0, 2, 1), (2, 5, row), (5, 6, 0)], 6, CPU)
    assert r.tolist() == [1, 1, 4, 3, 2, 0]
    assert r.dtype == torch.int32


def test_gap_overlap_and_short_cover_are_rejected():
    assert row_index([(0, 3, 0), (4, 9, 1)], 9, CPU) is None  # gap at row 3
    assert row_index([(0, 4, 0), (3, 9, 1)], 9, CPU) is None  # overlap at row 3
    assert row_index([(0, 3, 0), (3, 8, 1)], 9, CPU) is None  # stops before s
    assert row_index([(0, 3, 0), (3, 10, 1)], 9, CPU) is None  # runs past s
    assert row_index([(1, 9, 0)], 9, CPU) is None  # does not start at 0
    assert row_index([], 9, CPU) is None


def test_backwards_segment_and_wrong_tensor_length_are_rejected():
    assert row_index([(0, 5, 0), (5, 3, 1), (5, 9, 1)], 9, CPU) is None  # stop < start
    assert row_index([(0, 4, torch.tensor([1, 2, 3]))], 4, CPU) is None  # 3 entries for 4 rows


def test_empty_segments_and_empty_sequence():
    # a zero-length segment at the running position is accepted (start == pos, stop == start)
    assert row_index([(0, 2, 0), (2, 2, 5), (2, 4, 1)], 4, CPU).tolist() == [0, 0, 1, 1]
    r = row_index([], 0, CPU)
    assert r is not None and r.numel() == 0


def test_matches_a_literal_restatement_on_random_tilings():
    """Random tilings (int and tensor rows, shuffled order) against a direct
    per-row loop over the sorted segments."""
    g = torch.Generator().manual_seed(3)
    for trial in range(50):
        s = int(torch.randint(1, 300, (1,), generator=g))
        cuts = sorted(set(torch.randint(0, s + 1, (int(torch.randint(0, 8, (1,), generator=g)),),
                                        generator=g).tolist()) | {0, s})
        segs = []
        for a, b in zip(cuts[:-1], cuts[1:]):
            if trial % 2 and b > a:
                segs.append((a, b, torch.randint(0, 6, (b - a,), generator=g)))
            else:
                segs.append((a, b, int(torch.randint(0, 6, (1,), generator=g))))
        perm = torch.randperm(len(segs), generator=g).tolist()
        shuffled = [segs[i] for i in perm]
        expect = []
        for a, b, row in segs:
            expect += row.tolist() if torch.is_tensor(row) else [row] * (b - a)
        r = row_index(shuffled, s, CPU)
        assert r is not None and r.tolist() == expect


def test_modulation_tables_match_the_oracle():
    """The six tables of a7 (h3_fuse_patch.py:111-118): s1 = bf16(1.0 + bf16(scale)),
    shift and gate rounded to bf16, against the C oracle's scalar restatement,
    on values that straddle bf16 rounding boundaries after the 1.0 is added."""
    import numpy as np
    oracle = pytest.importorskip("oracle")
    g = torch.Generator().manual_seed(5)
    D = 4096
    e = torch.randn(6, D, generator=g) * 0.1
    # scale values whose bf16 sum with 1.0 lands on or next to a tie, tiny and large magnitudes, -1
    e[1, :8] = torch.tensor([2 ** -9, -2 ** -9, 3 * 2 ** -9, 2 ** -30, -1.0, 300.0, -2 ** -8, 1e-3])
    e[4, :4] = torch.tensor([2 ** -9 + 2 ** -17, -0.75, 65504.0, -1e-8])
    tabs = h3b.modulation_tables(*(e[i] for i in range(6)))
    bits = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    rne = lambda t: oracle.f32_to_bf16(t.numpy())  # noqa: E731
    s1a, sha, ga, s1m, shm, gm = (bits(t) for t in tabs)
    np.testing.assert_array_equal(s1a, oracle.one_plus(rne(e[1]), oracle.RNE))
    np.testing.assert_array_equal(s1m, oracle.one_plus(rne(e[4]), oracle.RNE))
    for got, i in ((sha, 0), (ga, 2), (shm, 3), (gm, 5)):
        np.testing.assert_array_equal(got, rne(e[i]))
