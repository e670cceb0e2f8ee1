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
