"""Small launches of single hot kernels, sized for profiler captures: each
target holds at most a few GB on the device and launches its kernel a
handful of times (a warm-up, then the launches to capture).

    python -m arc_chain_b200.bench.profile_targets <target>

targets (kernel name to select, launches before the first timed one):
  attn        k_attn_paged     7B decode attention, T = 386, 32 heads    (3)
  gemm_b1     k_gemm_fused     7B gate/up 22016 x 4096 at B = 1          (5)
  gemm_b256   k_gemm_fused     70B gate/up 57344 x 8192 at B = 256       (5)
  commit      k_batch_commit   BLAKE3 derive-key commit, 1M x 256 B      (1)
  ed25519     k_verify         Ed25519 verify_strict, 65,536 signatures  (1)
"""
from __future__ import annotations

import json
import sys

import torch


def attn():
    from arc_chain_b200.bench.kernels import bench_attn

    print(json.dumps(bench_attn(386, iters=2)))


def gemm_b1():
    from arc_chain_b200.bench.kernels import bench_fgemm

    print(json.dumps(bench_fgemm(22016, 4096, 1, iters=2)))


def gemm_b256():
    from arc_chain_b200.bench.kernels import bench_fgemm

    print(json.dumps(bench_fgemm(57344, 8192, 256, iters=2, limbs=4)))


def commit():
    from arc_chain_b200.bench.crypto import bench_commit

    print(json.dumps(bench_commit(1 << 20, reps=2)))


def ed25519():
    from arc_chain_b200.bench.crypto import bench_ed25519

    print(json.dumps(bench_ed25519(1 << 16, reps=2)))


TARGETS = {"attn": attn, "gemm_b1": gemm_b1, "gemm_b256": gemm_b256, "commit": commit, "ed25519": ed25519}


def main():
    torch.cuda.set_device(0)
    TARGETS[sys.argv[1]]()


if __name__ == "__main__":
    main()
