"""The allocation-free fused-GEMM entry point (arcb_fgemm_noalloc).

It serves callers that cannot allocate device memory themselves: its
partial-sum buffer and tile counters live in a fixed device array inside the
library instead of buffers the caller passes.  This test calls it through
its exported C symbol, twice in a row with different inputs, and requires
each result to equal the regular entry point's (which gets torch-allocated
scratch) exactly, the same tolerance the other kernel tests use.  It also
checks that an oversized problem, the partial-only mode and the push /
peer-target modes are refused.  The file is named so pytest collects it
last.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _entry():
    from arc_chain_b200.ops import _lib

    f = _lib.lib().arcb_fgemm_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    return f


def _limb_planes(x, rows):
    B, K = x.shape
    planes = np.zeros((8, B, K), dtype=np.int8)
    r = x.astype(np.int64).copy()
    for l in range(8):
        d = (r & 0xFF).astype(np.uint8).view(np.int8)
        planes[l] = d
        r = (r - d.astype(np.int64)) >> 8
    p = planes.reshape(8 * B, K)
    if p.shape[0] < rows:
        p = np.concatenate([p, np.zeros((rows - p.shape[0], K), np.int8)])
    return p


def test_noalloc_matches_regular_entry_twice():
    from arc_chain_b200.ops import int_ops as ops

    f = _entry()
    dev = torch.device("cuda")
    M, K, B = 1000, 688, 3
    rng = np.random.default_rng(7)
    W = torch.from_numpy(rng.integers(-127, 128, size=(M, K), dtype=np.int64).astype(np.int8)).to(dev)
    S = torch.from_numpy(rng.integers(1, 5000, size=M).astype(np.int64)).to(dev)
    wm = ops.TensorMap(ops.tile_weight(W), 128)
    bn = ops.fgemm_bn(B)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lmax = torch.tensor([8], dtype=torch.int32, device=dev)
    for call in range(2):
        x = rng.integers(-(1 << 40), 1 << 40, size=(B, K), dtype=np.int64)
        X = torch.from_numpy(_limb_planes(x, bn)).to(dev)
        xm = ops.TensorMap(X, bn)
        ref = torch.zeros(B, M, dtype=torch.int64, device=dev)
        P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
        tiles = torch.zeros((M + 127) // 128 + 1, dtype=torch.int32, device=dev)
        ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, ops.epi(ops.STORE, S, err, out=ref, ldo=M))
        out = torch.full((B, M), -1, dtype=torch.int64, device=dev)
        e = ops.epi(ops.STORE, S, err, out=out, ldo=M)
        rc = f(wm.addr, xm.addr, M, K, B, bn, lmax.data_ptr(), C.addressof(e),
               torch.cuda.current_stream().cuda_stream)
        assert rc == 0, f"call {call}: rc={rc}"
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out, ref), f"call {call}: no-alloc result differs"


def test_noalloc_rejects_oversized_and_partial_mode():
    from arc_chain_b200.ops import int_ops as ops

    f = _entry()
    dev = torch.device("cuda")
    W = torch.zeros(128, 128, dtype=torch.int8, device=dev)
    wm = ops.TensorMap(W, 128)
    X = torch.zeros(256, 128, dtype=torch.int8, device=dev)
    xm = ops.TensorMap(X, 256)
    lmax = torch.tensor([1], dtype=torch.int32, device=dev)
    S = torch.ones(128, dtype=torch.int64, device=dev)
    out = torch.zeros(64, 128, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream().cuda_stream
    e = ops.epi(ops.STORE, S, err, out=out, ldo=128)
    # 8 * 64 * 32000 partials exceed the 4 MiB scratch: refused, nothing launched
    assert f(wm.addr, xm.addr, 32000, 128, 64, 256, lmax.data_ptr(), C.addressof(e), st) == -21
    # more than 4093 tiles of 128 rows
    assert f(wm.addr, xm.addr, 4094 * 128 + 1, 128, 1, 16, lmax.data_ptr(), C.addressof(e), st) == -20
    p = ops.epi(ops.PARTIAL, S, err)
    assert f(wm.addr, xm.addr, 128, 128, 1, 16, lmax.data_ptr(), C.addressof(p), st) == -22
    # push and peer-target modes write other GPUs' caller-allocated buffers: refused
    # on the host before any launch (the pointers below are never dereferenced)
    for field in ("rp", "peer_h", "peer_sig"):
        q = ops.epi(ops.STORE, S, err, out=out, ldo=128)
        setattr(q, field, 1 if field == "rp" else out.data_ptr())
        assert f(wm.addr, xm.addr, 128, 128, 1, 16, lmax.data_ptr(), C.addressof(q), st) == -22, field
