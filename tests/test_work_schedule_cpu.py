"""The fused GEMM's work list (csrc/kernels/fgemm_dev.cuh, struct Work),
restated in Python: over every CTA the items cover each (tile, chunk) of
the GEMM exactly once, the round-robin part hands out whole tiles, each
CTA's item sequence is what its loops walk (item / next / seg_end), and the
stream-K tail keeps the per-CTA load within one tile of even.  The TMA
producer's segment walk (csrc/kernels/gemm_fused.cu: chunk index stepped
with wrap inside a segment) gives the same chunks as kc(it).  Fixed shapes
plus a random-shape sweep."""
import itertools

import pytest


class Work:
    def __init__(self, Mt, nch, ntu, grid, c, multi):
        self.Mt, self.nch, self.ntu, self.G, self.c = Mt, nch, ntu, grid, c
        self.dpn = self.dp_end = self.sk0 = self.per = self.rot = 0
        T = ntu * Mt
        if multi and ntu > 1 and T < 2 * grid and grid >= ntu:
            Gg = grid // ntu
            self.per = Mt * nch
            if c >= Gg * ntu:
                self.it0 = self.it1 = self.sk0 = 0
                return
            g, r = c % ntu, c // ntu
            self.it0 = self.sk0 = g * self.per + self.per * r // Gg
            self.it1 = g * self.per + self.per * (r + 1) // Gg
            return
        waves = max(0, T // grid - 1) if multi and ntu > 1 else 0
        self.dpn = waves * nch
        self.dp_end = waves * grid * nch
        self.rot = ((c % ntu) * max(1, nch // ntu) + (c // ntu) * 3) % nch
        total = (T - waves * grid) * nch
        self.sk0 = self.dp_end + total * c // grid
        self.it1 = self.dp_end + total * (c + 1) // grid
        self.it0 = c * self.dpn if self.dpn else self.sk0

    def count(self):
        return self.dpn + (self.it1 - self.sk0)

    def item(self, i):
        return self.it0 + i if i < self.dpn else self.sk0 + (i - self.dpn)

    def next(self, se):
        return self.sk0 if (self.dpn and se == self.it0 + self.dpn) else se

    def tile(self, it):
        if self.per:
            return ((it % self.per) // self.nch) * self.ntu + it // self.per
        if it < self.dp_end:
            return self.c + ((it - self.it0) // self.nch) * self.G
        return it // self.nch

    def kc(self, it):
        k = it % self.nch
        return (k + self.rot) % self.nch if it < self.dp_end else k

    def seg_end(self, it):
        e = (it // self.nch + 1) * self.nch
        return e if it < self.dp_end else min(self.it1, e)


@pytest.mark.parametrize("Mt,nch,ntu,grid", [(448, 64, 8, 148), (80, 64, 2, 148), (448, 64, 2, 148),
                                             (3, 5, 4, 7), (250, 64, 32, 148), (32, 16, 1, 148), (172, 32, 1, 148),
                                             (9, 3, 3, 4), (1, 1, 2, 5), (64, 64, 2, 148), (10, 16, 8, 148),
                                             (5, 7, 3, 8), (2, 4, 8, 3)])
@pytest.mark.parametrize("multi", [False, True])
def test_items_cover_each_tile_chunk_once(Mt, nch, ntu, grid, multi):
    check_cover(Mt, nch, ntu, grid, multi)


def test_cover_property_random_shapes():
    hyp = pytest.importorskip("hypothesis")
    st = hyp.strategies

    @hyp.settings(max_examples=400, deadline=None, derandomize=True)
    @hyp.given(st.integers(1, 200), st.integers(1, 64), st.integers(1, 40), st.integers(1, 300), st.booleans())
    def prop(Mt, nch, ntu, grid, multi):
        hyp.assume(Mt * ntu * nch <= 40000)
        check_cover(Mt, nch, ntu, grid, multi)

    prop()


def check_cover(Mt, nch, ntu, grid, multi):
    seen = {}
    loads = []
    for c in range(grid):
        W = Work(Mt, nch, ntu, grid, c, multi)
        items = [W.item(i) for i in range(W.count())]
        # the segment walk visits the same items in the same order
        walk, it = [], W.item(0)
        while it < W.it1:
            se = W.seg_end(it)
            t = W.tile(it)
            assert all(W.tile(j) == t for j in range(it, se))
            if it < W.dp_end:
                assert it % nch == 0 and se - it == nch  # round-robin tiles are whole
            # the producer steps the chunk index inside a segment (kc + 1, wrapping)
            kc = W.kc(it)
            for j in range(it, se):
                assert kc == W.kc(j)
                kc = 0 if kc + 1 == nch else kc + 1
            walk.extend(range(it, se))
            it = W.next(se)
        assert walk == items
        for it in items:
            key = (W.tile(it), W.kc(it))
            assert key not in seen, (key, c, seen.get(key))
            seen[key] = c
        loads.append(len(items))
    assert set(seen) == set(itertools.product(range(Mt * ntu), range(nch)))
    busy = [x for x in loads if x] if Work(Mt, nch, ntu, grid, 0, multi).per else loads
    assert max(busy) - min(busy) <= nch + 1


def test_round_robin_keeps_concurrent_tiles_on_few_weight_tiles():
    # 70B gate/up at B = 256: 448 weight tiles x 8 n-tiles over 148 CTAs
    Mt, nch, ntu, G = 448, 64, 8, 148
    Ws = [Work(Mt, nch, ntu, G, c, True) for c in range(G)]
    for j in (0, 5, 20):  # the j-th tile of every CTA runs at about the same time
        mts = {Ws[c].tile(Ws[c].item(j * nch)) // ntu for c in range(G)}
        assert len(mts) <= G // ntu + 2
        # ... but no chunk of a weight tile or of an n-tile is read by many CTAs at one moment
        for p in (0, 17, 63):
            a_reads, b_reads = {}, {}
            for c in range(G):
                it = Ws[c].item(j * nch + p)
                t, k = Ws[c].tile(it), Ws[c].kc(it)
                a_reads[(t // ntu, k)] = a_reads.get((t // ntu, k), 0) + 1
                b_reads[(t % ntu, k)] = b_reads.get((t % ntu, k), 0) + 1
            assert max(a_reads.values()) <= 2 and max(b_reads.values()) <= 3


def test_grouped_ctas_walk_the_same_weight_tiles_in_step():
    # 70B qkv at B = 64: 80 weight tiles x 2 n-tiles over 148 CTAs
    Mt, nch, ntu, G = 80, 64, 2, 148
    Ws = [Work(Mt, nch, ntu, G, c, True) for c in range(G)]
    assert all(W.per for W in Ws)
    for r in range(G // ntu):
        a, b = Ws[r * ntu], Ws[r * ntu + 1]
        assert a.count() == b.count()
        for i in range(a.count()):
            ia, ib = a.item(i), b.item(i)
            assert a.tile(ia) // ntu == b.tile(ib) // ntu and a.kc(ia) == b.kc(ib)  # same weight tile, same chunk
            assert a.tile(ia) % ntu == 0 and b.tile(ib) % ntu == 1
