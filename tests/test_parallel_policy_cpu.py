"""Host-side policy of the fused multi-GPU paths (no GPU): when the tensor-
parallel GEMM reduce switches to reduce-scatter + all-gather, and the guard
that keeps the continuous-batching scheduler away from the token-dispatch
expert-parallel communicator."""
import pytest

from arc_chain_b200.parallel.fused import FusedComm
from arc_chain_b200.runtime.scheduler import Scheduler


def _comm(size, mode):
    c = FusedComm.__new__(FusedComm)  # policy only: no process group
    c.size = size
    c.rs_ag = mode
    return c


@pytest.mark.parametrize("size,B,want", [(2, 1, False), (2, 64, False), (4, 8, False), (4, 16, True),
                                         (8, 1, False), (8, 128, True)])
def test_rs_ag_auto_policy(size, B, want):
    assert _comm(size, "auto").use_rs_ag(B) == want


def test_rs_ag_forced():
    assert _comm(2, "on").use_rs_ag(1) and not _comm(8, "off").use_rs_ag(128)


def test_scheduler_refuses_token_dispatch():
    class Eng:
        dispatch = True

    with pytest.raises(ValueError, match="replicated-token"):
        Scheduler(Eng())


@pytest.mark.parametrize("N,B", [(2, 1), (2, 16), (4, 8), (8, 4), (8, 16)])
def test_token_dispatch_layout(N, B):
    """The expert-parallel dispatch places row limb_row(l, b, B) of rank r's
    limb planes at row limb_row(l, r * B + b, N * B) of every gathered
    buffer (csrc/kernels/ep_ops.cu: k_ep_dispatch).  Assembled that way, the
    gathered buffer is exactly the limb operand of all N * B slots, and the
    combine's owner of gathered slot g (g // B, row g % B) is the rank that
    sent it."""
    import numpy as np

    from arc_chain_b200.ops import int_ops as ops

    rng = np.random.default_rng(N * 100 + B)
    K = 64
    xs = [rng.integers(-(1 << 40), 1 << 40, size=(B, K), dtype=np.int64) for _ in range(N)]
    NB = N * B
    want, _ = ops.limb_planes(np.concatenate(xs), ops.limb_rows(NB))
    got = np.zeros_like(want)
    for r, x in enumerate(xs):
        local, _ = ops.limb_planes(x, ops.limb_rows(B))
        for l in range(8):
            for b in range(B):
                got[ops.limb_row(l, r * B + b, NB)] = local[ops.limb_row(l, b, B)]
    np.testing.assert_array_equal(got, want)
    for g in range(NB):
        owner, row = g // B, g % B
        assert owner * B + row == g and np.array_equal(xs[owner][row], np.concatenate(xs)[g])
