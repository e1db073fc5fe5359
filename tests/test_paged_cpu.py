"""Host bookkeeping of the paged KV pools (qwen0.6b_b200/batched.py PagePool):
page mapping per 128-token block, exhaustion, release and reuse."""
import pytest

from batched import PAGE, PagePool


def test_reserve_maps_blocks_in_order_and_only_once():
    pp = PagePool(num_pages=6, num_seqs=2, max_pages=4)
    assert pp.reserve(0, 0) is True and pp.table[0] == [0, -1, -1, -1]
    assert pp.reserve(0, PAGE - 1) is False                      # same block
    assert pp.reserve(0, PAGE) is True and pp.table[0][:2] == [0, 1]
    assert pp.reserve(1, 3 * PAGE + 5) is True and pp.table[1] == [2, 3, 4, 5]
    assert pp.in_use == 6


def test_exhaustion_and_release_reuse():
    pp = PagePool(num_pages=3, num_seqs=2, max_pages=4)
    pp.reserve(0, 2 * PAGE)                                     # 3 pages
    with pytest.raises(RuntimeError, match="exhausted"):
        pp.reserve(1, 0)
    assert pp.table[1] == [-1] * 4                              # nothing half-mapped
    pp.release(0)
    assert pp.in_use == 0 and pp.table[0] == [-1] * 4
    pp.reserve(1, PAGE)
    got = pp.table[1][:2]
    assert len(set(got)) == 2 and set(got) <= {0, 1, 2} and pp.in_use == 2


def test_bounds():
    pp = PagePool(num_pages=4, num_seqs=1, max_pages=2)
    with pytest.raises(ValueError):
        pp.reserve(0, 2 * PAGE)                                 # beyond max_pages
    with pytest.raises(ValueError):
        pp.reserve(1, 0)                                        # no such sequence
