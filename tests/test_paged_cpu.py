"""Host-side page bookkeeping of the paged KV cache (no GPU): allocation, reservation,
exhaustion, freeing and reuse, and the rows that must be synced to the device."""
import numpy as np
import pytest

from leankv_b200.paged import NO_PAGE, PageTable


def test_reserve_allocates_whole_pages_in_order():
    pt = PageTable(num_pages=10, page_size=16, max_seqs=4, max_pages_per_seq=5)
    a, b = pt.add_sequence(), pt.add_sequence()
    assert (a, b) == (0, 1)
    pt.reserve([a, b], 17)               # 2 pages each
    assert pt.n_pages[a] == 2 and pt.n_pages[b] == 2
    assert list(pt.table[a, :2]) == [0, 1] and list(pt.table[b, :2]) == [2, 3]
    assert pt.table[a, 2] == NO_PAGE
    assert pt.free_pages == 6
    assert pt.dirty == {a, b}
    pt.commit([a, b], 17)
    pt.dirty.clear()
    pt.reserve([a], 15)                  # 32 tokens fit the 2 pages held: no new page
    assert pt.n_pages[a] == 2 and not pt.dirty
    pt.reserve([a], 16)                  # 33 tokens: a third page
    assert pt.n_pages[a] == 3 and pt.table[a, 2] == 4 and pt.dirty == {a}


def test_exhaustion_is_all_or_nothing():
    pt = PageTable(num_pages=3, page_size=16, max_seqs=2, max_pages_per_seq=4)
    a, b = pt.add_sequence(), pt.add_sequence()
    with pytest.raises(MemoryError):
        pt.reserve([a, b], 32)           # 4 pages needed, 3 free
    assert pt.free_pages == 3 and pt.n_pages[a] == 0 and pt.n_pages[b] == 0
    with pytest.raises(ValueError):
        pt.reserve([a], 65)              # over one sequence's 64-token limit


def test_free_returns_pages_and_slot_for_reuse():
    pt = PageTable(num_pages=6, page_size=32, max_seqs=2, max_pages_per_seq=3)
    a, b = pt.add_sequence(), pt.add_sequence()
    pt.reserve([a, b], 40)
    pt.commit([a, b], 40)
    held = set(pt.table[a, :2])
    pt.free_sequence(a)
    assert pt.free_pages == 4 and (pt.table[a] == NO_PAGE).all() and not pt.active[a]
    c = pt.add_sequence()                # the freed slot
    assert c == a and pt.lens[c] == 0
    with pytest.raises(RuntimeError):
        pt.add_sequence()                # no slot is idle
    pt.reserve([c], 64)
    assert set(pt.table[c, :2]) == held  # the freed pages come back first


def test_commit_and_inactive_checks():
    pt = PageTable(num_pages=4, page_size=16, max_seqs=2, max_pages_per_seq=4)
    a = pt.add_sequence()
    with pytest.raises(ValueError):
        pt.commit([a], 1)                # nothing reserved
    with pytest.raises(ValueError):
        pt.reserve([1], 1)               # inactive slot
    pt.reserve([a], 5)
    pt.commit([a], 5)
    assert pt.lens[a] == 5


@pytest.mark.parametrize("page_size", [0, 8, 24])
def test_bad_page_size(page_size):
    with pytest.raises(ValueError):
        PageTable(num_pages=4, page_size=page_size, max_seqs=1, max_pages_per_seq=1)


def test_random_workload_invariants():
    """Random joins, steps and leaves: pages are never shared and none is lost."""
    rng = np.random.default_rng(0)
    pt = PageTable(num_pages=64, page_size=16, max_seqs=8, max_pages_per_seq=16)
    for _ in range(400):
        act = list(np.flatnonzero(pt.active))
        r = rng.random()
        if r < 0.2 and len(act) < 8:
            pt.add_sequence()
        elif r < 0.3 and act:
            pt.free_sequence(int(rng.choice(act)))
        elif act:
            seqs = [int(s) for s in rng.choice(act, size=rng.integers(1, len(act) + 1), replace=False)]
            n = int(rng.integers(1, 20))
            try:
                pt.reserve(seqs, n)
            except (MemoryError, ValueError):
                continue
            pt.commit(seqs, n)
        held = pt.table[pt.table != NO_PAGE]
        assert len(set(held.tolist())) == held.size
        assert held.size + pt.free_pages == 64
        for s in np.flatnonzero(pt.active):
            assert pt.lens[s] <= pt.n_pages[s] * 16
