"""On the GPU, waits that can never be satisfied end with an error status
instead of hanging: the fused GEMM's cross-rank arrival wait is given a
"peer" counter that nothing fills, runs out after its ~2 s bound, sets
ARCB_ERR_COMM_TIMEOUT and returns; the context stays usable.  Out-of-range
positions are reported (ARCB_ERR_SEQ_OVERFLOW) and skipped, never accessed."""
import time

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ERR_COMM_TIMEOUT = 16
ERR_SEQ_OVERFLOW = 32


def test_cross_rank_wait_times_out_cleanly():
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    M, K, B = 128, 256, 1
    W = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev)
    wm = ops.TensorMap(ops.tile_weight(W), 128)
    bn = ops.fgemm_bn(B)
    X = torch.randint(-3, 4, (max(8 * B, bn), K), dtype=torch.int8, device=dev)
    xm = ops.TensorMap(X, bn)
    lmax = torch.tensor([1], dtype=torch.int32, device=dev)
    S = torch.ones(M, dtype=torch.int64, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    h = torch.zeros(B, M, dtype=torch.int64, device=dev)
    P = torch.zeros(8 * B * M, dtype=torch.int32, device=dev)
    R = torch.zeros(2 * B * M, dtype=torch.int64, device=dev)
    cnt = torch.zeros(4, dtype=torch.int32, device=dev)
    R_lost = torch.zeros_like(R)
    cnt_lost = torch.zeros_like(cnt)  # a "peer" that never reports back
    tiles = torch.zeros(4, dtype=torch.int32, device=dev)
    peerR = torch.tensor([R.data_ptr(), R_lost.data_ptr()], dtype=torch.int64, device=dev)
    peerC = torch.tensor([cnt.data_ptr(), cnt_lost.data_ptr()], dtype=torch.int64, device=dev)
    e = ops.epi(ops.RESID, S, err, out=h, ldo=M)
    e.rp, e.npeers, e.rank = 1, 2, 0
    e.peer_R, e.peer_cnt, e.cnt_local = peerR.data_ptr(), peerC.data_ptr(), cnt.data_ptr()
    # the local counter only ever sees this rank's own arrival, never the peer's
    t0 = time.time()
    ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, e)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(err.item()) & ERR_COMM_TIMEOUT
    assert dt < 30
    # the context is still healthy: an ordinary GEMM runs and is correct
    err.zero_()
    out = torch.zeros(B, M, dtype=torch.int64, device=dev)
    P.zero_()
    ops.fgemm(wm, xm, M, K, B, lmax, P, tiles, ops.epi(ops.STORE, S, err, out=out, ldo=M))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    x = X[:B].long().cpu()
    ref = (W.long().cpu() @ x.T).T
    assert torch.equal(out.cpu(), (ref * 1) >> 16)


def test_position_overflow_is_reported_not_accessed():
    from arc_chain_b200.ops import int_ops as ops

    dev = torch.device("cuda")
    nh, dh, B, T = 2, 64, 1, 32
    K = torch.zeros(2, nh, 16, dh, dtype=torch.int64, device=dev)
    V = torch.zeros_like(K)
    q = torch.zeros(B, nh * dh, dtype=torch.int64, device=dev)
    pt = torch.zeros(B, 2, dtype=torch.int32, device=dev)
    pos = torch.tensor([10_000], dtype=torch.int32, device=dev)  # far past max_T
    X = torch.zeros(8 * B, nh * dh, dtype=torch.int8, device=dev)
    lm = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.attn(q, K, V, pt, pos, nh, nh, dh, 5793, B, X, lm, T, err)
    torch.cuda.synchronize()
    assert int(err.item()) & ERR_SEQ_OVERFLOW
