"""Tensor parallelism for the dense decoder: 2-rank (and, where the box has
them, 4- and 8-rank) runs with the NCCL all-reduce, with the fused in-GEMM reduce
over NVLink peer memory (push to every rank, and the reduce-scatter +
all-gather form) with the LM head's fused all-gather, and with the logits
gathered over NCCL instead, every token checked against the oracle."""
import json
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpu():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("comm", ["nccl", "fused", "fused-nccl-logits", "fused-rsag"])
def test_tp_matches_oracle(comm, world):
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    port = 29300 + (os.getpid() % 200) + {"nccl": 0, "fused": 7, "fused-nccl-logits": 13, "fused-rsag": 23}[comm] + world
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "tp_worker.py"), "--comm", comm]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["ok_all_ranks"] and res["kernel_errors"] == 0 and res["checks"] == 52
