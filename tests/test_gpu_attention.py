"""Paged decode attention kernels against a numpy restatement of the
reference's integer attention (spec.softmax; scores ((q.k >> 16) * scale)
>> 16 with wrapping dots; per-term (w * v) >> 16): the TMA-fed page-ring
form per query head and the per-thread-load form, every cluster size, GQA with
1, 2, 4 and 8 query heads per KV head, several slots of different lengths
over a shuffled page table, and magnitudes that wrap."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200 import spec

pytestmark = pytest.mark.gpu
PAGE = 16


def _reference(q, K, V, pt, pos, n_heads, n_kv, dh, scale):
    B = q.shape[0]
    out = np.zeros((B, n_heads * dh), dtype=np.int64)
    with np.errstate(over="ignore"):
        for b in range(B):
            T = int(pos[b]) + 1
            pages = pt[b, :(T + PAGE - 1) // PAGE]
            for hq in range(n_heads):
                kvh = hq * n_kv // n_heads
                Kh = K[pages, kvh].reshape(-1, dh)[:T]
                Vh = V[pages, kvh].reshape(-1, dh)[:T]
                qh = q[b, hq * dh:(hq + 1) * dh]
                dots = (Kh * qh).sum(axis=1, dtype=np.int64)
                sc = ((dots >> 16) * scale) >> 16
                w = spec.softmax(sc)
                out[b, hq * dh:(hq + 1) * dh] = ((w[:, None] * Vh) >> 16).sum(axis=0, dtype=np.int64)
    return out


@pytest.mark.parametrize("form", ["paged", "plain"])
@pytest.mark.parametrize("cluster", [1, 2, 4, 8])
@pytest.mark.parametrize("dh,n_heads,n_kv,lens,mag", [
    (128, 4, 4, [386], 1 << 18),
    (128, 8, 2, [1, 17, 130, 255], 1 << 20),
    (64, 4, 4, [33, 64, 200], 1 << 18),
    (128, 2, 1, [100, 300], 1 << 40),  # dots wrap
    (128, 16, 2, [5, 70, 301, 1, 17, 33, 64, 129, 200], 1 << 19),  # 8 query heads per KV head, 9 slots
    (128, 8, 2, [40, 3, 300, 16, 15, 90, 7, 250], 1 << 40),  # 4 per KV head, 8 slots, wrapping dots
])
def test_attention_matches_reference(form, cluster, dh, n_heads, n_kv, lens, mag):
    from arc_chain_b200.ops import int_ops as ops

    rng = np.random.default_rng(len(lens) * 7 + dh + n_kv)
    B = len(lens)
    max_T = (max(lens) + PAGE - 1) // PAGE * PAGE + 32
    ppb = max_T // PAGE
    n_pages = B * ppb + 3
    K = rng.integers(-mag, mag, size=(n_pages, n_kv, PAGE, dh), dtype=np.int64)
    V = rng.integers(-mag, mag, size=(n_pages, n_kv, PAGE, dh), dtype=np.int64)
    q = rng.integers(-mag, mag, size=(B, n_heads * dh), dtype=np.int64)
    pt = rng.permutation(n_pages)[:B * ppb].reshape(B, ppb).astype(np.int32)
    pos = np.array([t - 1 for t in lens], dtype=np.int32)
    scale = 5793 if dh == 128 else 8192
    ref = _reference(q, K, V, pt, pos, n_heads, n_kv, dh, scale)
    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    X = torch.zeros(ops.limb_rows(B), n_heads * dh, dtype=torch.int8, device=dev)
    lm = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    o = torch.zeros(B, n_heads * dh, dtype=torch.int64, device=dev)
    ops.set_attn_paged(form != "plain")
    try:
        ops.attn(t(q), t(K), t(V), t(pt), t(pos), n_heads, n_kv, dh, scale, B, X, lm, max_T, err, o_out=o,
                 cluster=cluster)
        torch.cuda.synchronize()
    finally:
        ops.set_attn_paged(True)
    assert int(err.item()) == 0
    np.testing.assert_array_equal(o.cpu().numpy(), ref)
    planes, need = ops.limb_planes(ref)
    np.testing.assert_array_equal(X.cpu().numpy()[:planes.shape[0]], planes)
    assert int(lm.item()) == need
