"""Loader for the in-tree sm_100a kernel library (``libarcb_cuda.so``).

There is no fallback: on a machine with a GPU, a missing or unloadable
library raises.  Kernels launch on the caller's current torch CUDA stream, so
they compose with torch ops and are captured by CUDA graphs.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_LIB = None
_LOCK = threading.Lock()

vp, i32, i64, u64 = C.c_void_p, C.c_int, C.c_int64, C.c_uint64

_SIGS = {
    "arcb_tmap_i8": (i32, [vp, vp, i64, i64, i32]),
    "arcb_gemm_bn": (i32, [i32]),
    "arcb_gemm_i8": (i32, [vp, vp, i32, i32, i32, i32, i32, vp, vp, vp, vp]),
    "arcb_embed": (i32, [vp, vp, vp, i32, i32, i32, vp, vp, i32, vp, i32, vp]),
    "arcb_norm_limbs": (i32, [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp]),
    "arcb_rmsnorm_limbs": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, vp]),
    "arcb_finalize": (i32, [vp, i32, i32, vp, vp, vp, i32, i32, vp, vp]),
    "arcb_sample": (i32, [vp, i32, i32, vp, i32, vp, vp, vp, i32, vp, vp, vp, vp, i32, vp]),
    "arcb_rng_i8": (i32, [u64, u64, vp, i64, vp]),
    "arcb_attn_cluster": (i32, [vp, vp, vp, vp, i32, vp, i32, i32, i32, i64, i32, i32, i32, vp, vp, vp, vp, vp]),
    "arcb_fgemm_bn": (i32, [i32]),
    "arcb_fgemm": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, i32, vp]),
    "arcb_fgemm_epi_size": (i32, []),
    "arcb_fgemm_q4": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp, vp, i32, vp]),
    "arcb_verify_sample": (i32, [vp, i32, i32, i32, i32, vp, vp, vp, vp, vp]),
    "arcb_blake3_chunk_cvs": (i32, [vp, vp, i32, i64, i64, vp, vp]),
    "arcb_blake3_parents": (i32, [vp, i64, vp, vp]),
    "arcb_blake3_batch_commit": (i32, [vp, i64, vp, i64, vp, vp, i64, vp, vp]),
    "arcb_merkle_root": (i32, [vp, i64, vp, vp, vp, vp]),
    "arcb_ep_wait_apply": (i32, [vp, vp, C.c_uint64, vp, vp, i64, vp, vp, vp]),
    "arcb_check_udiv": (i32, [i64, i64, i32, vp, vp]),
    "arcb_ep_dispatch": (i32, [vp, i32, i32, vp, i32, vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, i32, vp, vp]),
    "arcb_attn_prefill": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i64, i32, i32, vp, vp, vp, vp]),
    "arcb_attn_prefill_max_T": (i32, [i32, i32]),
    "arcb_attn_gqa_block": (i32, [vp, vp, vp, vp, i32, vp, i32, i32, i32, i64, i32, i32, i32, vp, vp, vp, vp]),
    "arcb_ed25519_init": (i32, [vp, vp, vp, vp, vp, vp]),
    "arcb_ed25519_verify": (i32, [vp, vp, vp, vp, i64, vp, vp]),
    "arcb_ed25519_verify_prehashed": (i32, [vp, i64, vp, vp]),
    "arcb_ed25519_selftest": (i32, [i32, vp, i64, vp, vp, vp]),
    "arcb_mla_kv": (i32, [vp, i32, i32, vp, i32, vp, vp, i32, vp, vp, vp, i32, i32, vp, vp]),
    "arcb_mla_q": (i32, [vp, i32, i32, i32, i32, vp, vp, vp, vp, vp, i32, i32, vp, vp]),
    "arcb_mla_out": (i32, [vp, i32, i32, i32, vp, vp, i32, vp, vp, vp, vp]),
    "arcb_attn_mla": (i32, [vp, vp, vp, i32, vp, i32, i32, i32, i64, i32, i32, i32, vp, vp, vp]),
    "arcb_moe_route": (i32, [vp, i32, i32, i32, i32, i32, vp, vp]),
    "arcb_set_pdl": (None, [i32]),
    "arcb_set_attn_paged": (None, [i32]),
    "arcb_wg_layernorm": (i32, [vp, i64, vp, i64, vp, i64, i32, vp]),
    "arcb_wg_quantize": (i32, [vp, i64, vp, i64, vp, vp]),
    "arcb_wg_matmul": (i32, [vp, i64, vp, i64, vp, i64, i32, i32, vp, i64, vp]),
    "arcb_wg_rope": (i32, [vp, i64, vp, vp, i64, i32, i32, i32, vp]),
    "arcb_wg_attention": (i32, [vp, i64, vp, vp, i64, vp, vp, i64, vp, i64, i32, i32, i32, i32, i32, i32, vp]),
    "arcb_wg_silu": (i32, [vp, vp, i64, vp]),
    "arcb_wg_residual": (i32, [vp, vp, i64, vp]),
    "arcb_wg_argmax": (i32, [vp, i64, vp, vp]),
    "arcb_get_pdl": (i32, []),
}


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            from arc_chain_b200 import _build

            path = os.path.join(_build.LIBDIR, "libarcb_cuda.so")
            if not os.path.exists(path) or _build._stale(path, _build.cuda_sources() + _build._headers()):
                path = _build.build_cuda()
            L = C.CDLL(path)
            for name, (res, args) in _SIGS.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _LIB = L
    return _LIB


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with CUDA error {rc}")


def loaded_path() -> str:
    from arc_chain_b200 import _build

    return os.path.join(_build.LIBDIR, "libarcb_cuda.so")
