"""Expert parallelism for the MLA + MoE decoder: the device generator with
expert shards, and 2-, 4- and 8-rank runs (as the box allows) against the oracle: replicated tokens (NCCL
and fused peer-push combine) and token dispatch (each rank decodes its own
prompts; tokens are sent to the experts' ranks and combined on their
owner)."""
import json
import os
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")

from arc_chain_b200.formats import gen
from arc_chain_b200.models.config import preset

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("ep_size", [1, 2, 3])
def test_device_generator_matches_host_shards(ep_size):
    from arc_chain_b200.models import mla_moe_engine as me

    cfg = preset("micro_moe")
    host = gen.random_model(cfg, 2)
    for rank in range(ep_size):
        a = me.from_host(host, "cuda", rank, ep_size)
        b = me.random_device(cfg, "cuda", 2, rank, ep_size)
        assert torch.equal(a.emb, b.emb) and torch.equal(a.lm.w, b.lm.w) and torch.equal(a.final_norm, b.final_norm)
        for la, lb in zip(a.layers, b.layers):
            for n in ("q", "kva", "wo", "gu", "down", "router", "egu", "edown"):
                x, y = getattr(la, n), getattr(lb, n)
                assert (x is None) == (y is None), n
                if x is not None:
                    assert torch.equal(x.w, y.w) and torch.equal(x.s, y.s), n
            for n in ("kv_norm", "uk", "uk_s", "uv", "uv_s", "attn_norm", "ffn_norm"):
                assert torch.equal(getattr(la, n), getattr(lb, n)), n


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("comm", ["nccl", "fused", "dispatch"])
def test_ep_matches_oracle(comm, world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    port = 29600 + (os.getpid() % 200) + {"nccl": 0, "fused": 7, "dispatch": 13}[comm] + 20 * world
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "ep_worker.py"), "--comm", comm]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("{")][-1]
    res = json.loads(line)
    assert res["ok_all_ranks"] and res["kernel_errors"] == 0
    assert res["checks"] == (5 if comm == "dispatch" else 12)
