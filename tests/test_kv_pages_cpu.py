"""The paged KV cache's host bookkeeping under random reserve / release
sequences: page tables stay disjoint, tables plus the free list are exactly
the pool, a request's table only grows while it lives, and a reservation
that does not fit raises without taking any page."""
import pytest

from arc_chain_b200.runtime.kv_paged import PAGE, PagedKV

hyp = pytest.importorskip("hypothesis")
st = hyp.strategies

OPS = st.lists(st.tuples(st.sampled_from(["reserve", "release"]), st.integers(0, 5), st.integers(0, 6 * PAGE)),
               max_size=60)


@hyp.settings(max_examples=300, deadline=None, derandomize=True)
@hyp.given(st.integers(1, 24), st.integers(1, 8), OPS)
def test_page_tables_partition_the_pool(n_pages, max_per_seq, ops):
    kv = PagedKV(1, n_pages, 1, 1, "cpu", max_per_seq)
    for op, rid, n_tok in ops:
        before = {r: list(t) for r, t in kv.tables.items()}
        free_before = list(kv.pool.free)
        if op == "reserve":
            need = (n_tok + PAGE - 1) // PAGE
            try:
                t = kv.reserve(rid, n_tok)
            except ValueError:
                assert need > max_per_seq
            except MemoryError:
                assert need - len(before.get(rid, [])) > len(free_before)
                assert kv.pool.free == free_before
                assert all(kv.tables.get(r, []) == p for r, p in before.items())
            else:
                assert len(t) >= need and t[:len(before.get(rid, []))] == before.get(rid, [])
        else:
            kv.release(rid)
            assert rid not in kv.tables
        owned = [p for t in kv.tables.values() for p in t]
        assert len(owned) == len(set(owned))
        assert sorted(owned + kv.pool.free) == list(range(n_pages))
        assert kv.pool.used == len(owned)
        for r in kv.tables:
            row = kv.table_row(r)
            assert len(row) == max_per_seq and row[:len(kv.tables[r])] == kv.tables[r]


def test_requests_that_can_never_fit_are_refused():
    from arc_chain_b200.runtime.scheduler import check_fits

    kv = PagedKV(1, 8, 1, 1, "cpu", 8)  # 8 pages, a sequence may hold all 8
    check_fits(kv, 1, 100, 11)  # 112 positions = 7 pages: fits beside the scratch page
    with pytest.raises(ValueError, match="besides"):
        check_fits(kv, 1, 100, 12)  # 113 positions = 8 pages, only 7 outside the scratch page
    kv = PagedKV(1, 64, 1, 1, "cpu", 4)
    check_fits(kv, 1, 30, 33)  # 64 positions = 4 pages
    with pytest.raises(ValueError, match="at most 4"):
        check_fits(kv, 1, 30, 34)
