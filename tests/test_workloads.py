"""CPU tests of the contest-record replay inputs: the committed axes of the
reference's workload records and the two cu_seqlens rewrites of its scripts
(gdn_prefill/scripts/run_local_fast_even.py:31-43, run_local_fast_uneven.py:32-46)."""
import pytest

from gdn_b200 import workloads as W


def test_axes_fixture_shape():
    ax = W.contest_axes()
    assert len(ax["prefill"]) == 100 and len(ax["decode_batch"]) == 54
    assert all(1 <= n <= t for t, n in ax["prefill"])
    assert set(ax["decode_batch"]) <= {1, 4, 8, 16, 32, 48, 64}
    assert max(t for t, _ in ax["prefill"]) == 8192


@pytest.mark.parametrize("total,n", [(6, 1), (134, 1), (100, 7), (8192, 57), (57, 57)])
def test_even_and_uneven_splits(total, n):
    ev = W.even_lengths(total, n)
    assert sum(ev) == total and len(ev) == n and max(ev) - min(ev) <= 1
    assert ev == sorted(ev, reverse=True)  # the longer ones first, as the reference builds them
    un = W.uneven_lengths(total, n)
    assert sum(un) == total and len(un) == n and un[:-1] == [1] * (n - 1)


def test_uneven_rejects_short_totals():
    with pytest.raises(ValueError):
        W.uneven_lengths(3, 4)


def test_record_list_covers_every_record_twice():
    recs = W.contest_prefill_records()
    assert len(recs) == 200
    ax = W.contest_axes()["prefill"]
    for i, split, lengths in recs:
        assert sum(lengths) == ax[i][0] and len(lengths) == ax[i][1]
