"""Page manager host logic (molot_pager_*, n_layers = 0: no device memory):
allocation order, reuse, capacity errors, block tables."""
import numpy as np
import pytest


@pytest.fixture()
def mbl():
    import molot_b200
    return molot_b200


def test_tables_and_lengths(mbl):
    p = mbl.Pager(0, 8, 128, 16, num_pages=20, max_seqs=4, max_pages_per_seq=6)
    try:
        a = p.add(40)   # 3 pages: 0, 1, 2
        b = p.add(16)   # 1 page: 3
        assert (a, b) == (0, 1)
        bt, lens = p.tables([a, b])
        assert bt.shape == (2, 6)
        assert list(bt[0, :3]) == [0, 1, 2] and list(bt[1, :1]) == [3]
        assert list(lens) == [40, 16]
        p.grow(a, 8)    # 48 slots: still 3 pages
        p.grow(b, 1)    # 17 slots: a second page (4)
        bt, lens = p.tables([b, a])
        assert list(lens) == [17, 48] and list(bt[0, :2]) == [3, 4]
        assert p.free_pages() == 20 - 5
    finally:
        p.close()


def test_free_reuses_pages_first(mbl):
    p = mbl.Pager(0, 2, 64, 16, num_pages=8, max_seqs=3, max_pages_per_seq=8)
    try:
        a = p.add(33)  # pages 0, 1, 2
        b = p.add(16)  # page 3
        p.free(a)
        c = p.add(20)  # a's first pages come back first: 0, 1
        assert c == a  # the sequence slot is reused too
        bt, _ = p.tables([c, b])
        assert list(bt[0, :2]) == [0, 1] and bt[1, 0] == 3
        with pytest.raises(mbl.MolotError):
            p.length(2)  # never added
    finally:
        p.close()


def test_capacity_errors(mbl):
    p = mbl.Pager(0, 2, 64, 16, num_pages=4, max_seqs=2, max_pages_per_seq=3)
    try:
        a = p.add(48)  # 3 pages
        with pytest.raises(mbl.MolotError) as ei:
            p.grow(a, 1)  # a 4th page exceeds max_pages_per_seq
        assert ei.value.status == mbl.ERR_CACHE_FULL
        assert p.length(a) == 48
        with pytest.raises(mbl.MolotError) as ei:
            p.add(32)  # 2 pages, 1 left
        assert ei.value.status == mbl.ERR_CACHE_FULL
        assert p.free_pages() == 1  # the failed add returned what it took
        b = p.add(1)
        with pytest.raises(mbl.MolotError):
            p.add(1)  # no sequence slot left
        p.free(a)
        p.free(b)
        assert p.free_pages() == 4
        with pytest.raises(mbl.MolotError):
            p.free(a)  # already free
    finally:
        p.close()


def test_rejects_bad_page_size(mbl):
    with pytest.raises(mbl.MolotError):
        mbl.Pager(0, 2, 64, 10, 4, 2, 3)


def test_storage_types(mbl):
    """Pools of each storage type are accepted (tables-only here: no device
    memory); an unknown type and Q8 rows that do not split into 32-value
    blocks of both halves are refused."""
    for dtype in ("f32", "bf16", "q8"):
        p = mbl.Pager(0, 2, 128, 16, 4, 2, 3, dtype=dtype)
        assert p.dtype == dtype and p.free_pages() == 4
        p.close()
    with pytest.raises(ValueError):
        mbl.Pager(0, 2, 128, 16, 4, 2, 3, dtype="fp8")
    with pytest.raises(mbl.MolotError) as e:
        mbl.Pager(0, 2, 96, 16, 4, 2, 3, dtype="q8")
    assert e.value.status == mbl.ERR_INVALID
    h = mbl.ctypes.c_void_p()
    assert mbl._lib.molot_pager_create_ex(0, 2, 128, 16, 4, 2, 3, 7, mbl.ctypes.byref(h)) == mbl.ERR_INVALID
