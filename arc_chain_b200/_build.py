"""Builds the native libraries in-tree (``arc_chain_b200/_lib``).

* ``libarcref.so``  — C++ CPU oracle + BLAKE3 (g++).
* ``libarcb_cuda.so`` — every sm_100a kernel (nvcc, ``-gencode
  arch=compute_100a,code=sm_100a``), plus its C ABI launchers.

Objects are rebuilt only when a source or header is newer than the object.
``python -m arc_chain_b200._build`` builds everything.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "csrc")
LIBDIR = os.path.join(ROOT, "arc_chain_b200", "_lib")
OBJDIR = os.path.join(ROOT, "build", "obj")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                     "-Xptxas", "-warn-spills", "-I" + CSRC]
# no floating-point contraction: the host float paths restate Rust, which rounds
# every product and sum separately
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-pthread", "-ffp-contract=off", "-I" + CSRC]


def _headers():
    return glob.glob(os.path.join(CSRC, "**", "*.h"), recursive=True) + \
        glob.glob(os.path.join(CSRC, "**", "*.cuh"), recursive=True)


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    # a sanitizer runtime preloaded into the Python process is not the
    # compiler's business
    env = {k: v for k, v in os.environ.items() if k != "LD_PRELOAD"}
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


# ARCB_HOST_SANITIZE=1 builds and loads ``libarcref_san.so`` instead: the host
# library under AddressSanitizer and UndefinedBehaviorSanitizer.  Python itself
# is not instrumented, so the runtimes must be preloaded:
#   ARCB_HOST_SANITIZE=1 ASAN_OPTIONS=detect_leaks=0 \
#   LD_PRELOAD="$(gcc -print-file-name=libasan.so) $(gcc -print-file-name=libubsan.so)" \
#   python -m pytest tests -m "not gpu"
SANITIZE_FLAGS = ["-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=address,undefined"]


def build_arcref(verbose=False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = [os.path.join(CSRC, "ref", f) for f in ("arcref.cpp", "blake3.cpp", "toy_engine.cpp", "wgsl_forward.cpp", "neuralnet.cpp")]
    san = os.environ.get("ARCB_HOST_SANITIZE", "0") not in ("", "0")
    out = os.path.join(LIBDIR, "libarcref_san.so" if san else "libarcref.so")
    if _stale(out, srcs + _headers()):
        flags = CXX_FLAGS + (SANITIZE_FLAGS if san else [])
        # the sanitized build uses the g++ on PATH: the one whose runtimes
        # `gcc -print-file-name` names for the preload
        _run(["g++" if san else CXX, *flags, "-shared", "-o", out + ".tmp", *srcs])
        os.replace(out + ".tmp", out)
        if verbose:
            print("built", out)
    return out


def cuda_sources():
    return sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")) + glob.glob(os.path.join(CSRC, "aux", "*.cu")))


def build_cuda(verbose=False, ptxas_verbose=False) -> str:
    os.makedirs(LIBDIR, exist_ok=True)
    os.makedirs(OBJDIR, exist_ok=True)
    hdrs = _headers()
    srcs = cuda_sources()
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(OBJDIR, os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, [s] + hdrs) or ptxas_verbose:
            flags = list(NVCC_FLAGS)
            if ptxas_verbose:
                flags += ["-Xptxas", "-v"]
            jobs.append((s, [NVCC, *flags, "-c", s, "-o", o]))
    logs = {}
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = {ex.submit(_run, cmd): s for s, cmd in jobs}
        for f, s in futs.items():
            logs[s] = f.result()
            if verbose:
                print("compiled", os.path.relpath(s, ROOT))
    out = os.path.join(LIBDIR, "libarcb_cuda.so")
    if _stale(out, objs):
        _run([NVCC, *ARCH, "-shared", "-o", out + ".tmp", *objs, "-lcuda"])
        os.replace(out + ".tmp", out)
        if verbose:
            print("linked", out)
    if ptxas_verbose:
        for s, log in logs.items():
            print(f"== {os.path.relpath(s, ROOT)}\n{log}")
    return out


def build_all(verbose=False):
    a = build_arcref(verbose)
    c = build_cuda(verbose) if shutil.which(NVCC) or os.path.exists(NVCC) else None
    return a, c


if __name__ == "__main__":
    build_all(verbose=True) if "-v" not in sys.argv else build_cuda(verbose=True, ptxas_verbose=True)
