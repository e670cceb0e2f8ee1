"""ctypes binding of the C++ CPU oracle (``csrc/ref/arcref.cpp``).

The oracle is the bit-exact restatement of the reference engine's
``CachedIntegerModel`` (crates/arc-inference/src/cached_integer_model.rs).
It is loaded from the in-tree ``libarcref.so``; :func:`lib` builds it on first
use when the shared object is missing or stale.
"""
from __future__ import annotations

import ctypes as C
import threading
from typing import List, Optional, Sequence, Tuple

import numpy as np

_LIB = None
_LOCK = threading.Lock()


class Config(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("n_layers", "d_model", "n_heads", "n_kv_heads", "d_ff",
                                          "d_head", "d_kv", "vocab", "max_seq", "attn_scale")]


def lib():
    global _LIB
    with _LOCK:
        if _LIB is None:
            from arc_chain_b200 import _build

            path = _build.build_arcref()
            L = C.CDLL(path)
            vp, i64, u64 = C.c_void_p, C.c_int64, C.c_uint64
            sig = {
                "arcref_load_file": (vp, [C.c_char_p, C.c_char_p, C.c_int]),
                "arcref_from_arrays": (vp, [C.POINTER(Config), C.POINTER(vp), C.POINTER(i64)]),
                "arcref_free": (None, [vp]),
                "arcref_get_config": (None, [vp, C.POINTER(Config)]),
                "arcref_enable_q4": (None, [vp]),
                "arcref_generate": (i64, [vp, vp, i64, i64, vp, i64, vp, vp]),
                "arcref_cache_new": (vp, [vp]),
                "arcref_cache_free": (None, [vp]),
                "arcref_cache_len": (i64, [vp]),
                "arcref_cache_overflow": (C.c_int, [vp]),
                "arcref_cache_truncate": (None, [vp, i64]),
                "arcref_forward": (None, [vp, vp, C.c_uint32, vp]),
                "arcref_last_hidden": (None, [vp, vp]),
                "arcref_weight_hash": (None, [vp, vp]),
                "arcref_integer_exp": (i64, [i64]),
                "arcref_integer_isqrt": (i64, [i64]),
                "arcref_silu": (i64, [i64]),
                "arcref_softmax": (None, [vp, i64, vp]),
                "arcref_rmsnorm": (None, [vp, i64, vp, i64, vp]),
                "arcref_matmul_i8": (None, [vp, vp, vp, i64, i64, vp]),
                "arcref_blake3": (None, [vp, C.c_size_t, vp]),
                "arcref_blake3_new": (vp, []),
                "arcref_blake3_update": (None, [vp, vp, C.c_size_t]),
                "arcref_blake3_push_chunk_cv": (None, [vp, vp, u64]),
                "arcref_blake3_finalize": (None, [vp, vp]),
                "arcref_blake3_push_subtree_cv": (None, [vp, vp, C.c_int, u64]),
                "arcref_blake3_free": (None, [vp]),
                "arcref_blake3_new_derive": (vp, [C.c_char_p, C.c_size_t]),
                "arcref_set_embedding_q16": (None, [vp, vp]),
                "arcref_blake3_new_keyed": (vp, [vp]),
                "arcref_blake3_context_key": (None, [C.c_char_p, C.c_size_t, vp]),
                "arcref_blake3_batch_commit": (None, [vp, vp, C.c_int64, vp, C.c_char_p, C.c_size_t, vp]),
                "arcref_merkle_root": (None, [vp, C.c_int64, C.c_char_p, C.c_size_t, vp]),
                "arcref_rng_fill_i8": (None, [u64, u64, vp, i64]),
                "arcref_rng_u64": (None, [u64, u64, vp, i64]),
                "arcwg_new": (vp, [C.c_int] * 7 + [C.c_int32]),
                "arcwg_free": (None, [vp]),
                "arcwg_set_layer": (C.c_int, [vp, C.c_int, C.POINTER(vp), C.POINTER(vp), vp, vp]),
                "arcwg_set_head": (C.c_int, [vp, vp, vp, vp, vp, vp, C.c_int]),
                "arcwg_forward": (C.c_int, [vp, vp, C.c_int, vp]),
                "arcref_save_file": (C.c_int, [vp, C.c_char_p, C.c_char_p, i64, C.c_char_p, C.c_int]),
                "arcnn_parse": (vp, [C.c_char_p, C.c_size_t, C.c_char_p, C.c_int]),
                "arcnn_new": (vp, []),
                "arcnn_add_layer": (C.c_int, [vp, C.c_int, i64, i64, vp, vp, C.c_float]),
                "arcnn_free": (None, [vp]),
                "arcnn_tag_base": (C.c_int, [vp]),
                "arcnn_num_layers": (i64, [vp]),
                "arcnn_layer": (C.c_int, [vp, i64, C.POINTER(i64), C.POINTER(i64), C.POINTER(C.c_float)]),
                "arcnn_layer_data": (i64, [vp, i64, C.c_int, vp, i64]),
                "arcnn_input_size": (i64, [vp]),
                "arcnn_output_size": (i64, [vp]),
                "arcnn_serialize": (i64, [vp, C.c_int, vp, i64]),
                "arcnn_output_len": (i64, [vp, i64]),
                "arcnn_forward_f32": (i64, [vp, vp, i64, vp, i64]),
                "arcnn_forward_q16": (i64, [vp, vp, i64, vp, i64]),
                "arcnn_softmax_f32": (None, [vp, i64, vp]),
                "arcref_num_threads": (C.c_int, []),
                "arcref_set_threads": (None, [C.c_int]),
            }
            for name, (res, args) in sig.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _LIB = L
    return _LIB


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def integer_exp(x: int) -> int:
    return lib().arcref_integer_exp(int(x))


def integer_isqrt(x: int) -> int:
    return lib().arcref_integer_isqrt(int(x))


def silu(x: int) -> int:
    return lib().arcref_silu(int(x))


def softmax(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int64)
    out = np.empty_like(x)
    lib().arcref_softmax(_p(x), x.size, _p(out))
    return out


def rmsnorm(x: np.ndarray, gamma: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int64)
    g = np.ascontiguousarray(gamma, dtype=np.int64)
    out = np.empty_like(x)
    lib().arcref_rmsnorm(_p(x), x.size, _p(g), g.size, _p(out))
    return out


def matmul_i8(w: np.ndarray, s: np.ndarray, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.int64)
    x = np.ascontiguousarray(x, dtype=np.int64)
    out = np.empty(w.shape[0], dtype=np.int64)
    lib().arcref_matmul_i8(_p(w), _p(s), _p(x), w.shape[0], w.shape[1], _p(out))
    return out


def blake3(data) -> bytes:
    b = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else np.ascontiguousarray(data).view(np.uint8)
    out = np.zeros(32, dtype=np.uint8)
    lib().arcref_blake3(_p(b) if b.size else None, b.size, _p(out))
    return out.tobytes()


def rng_fill_i8(seed: int, stream: int, out: np.ndarray) -> None:
    assert out.dtype == np.int8 and out.flags.c_contiguous
    lib().arcref_rng_fill_i8(seed, stream, _p(out), out.size)


class Model:
    """An oracle model over an :class:`Int8Model` (arrays are referenced, not copied)."""

    def __init__(self, model=None, path: Optional[str] = None):
        L = lib()
        self._keep = []
        if path is not None:
            err = C.create_string_buffer(512)
            self.h = L.arcref_load_file(path.encode(), err, 512)
            if not self.h:
                raise ValueError(err.value.decode())
        else:
            c = model.cfg
            cfg = Config(c.n_layers, c.d_model, c.n_heads, c.n_kv_heads, c.d_ff, c.d_head, c.d_kv,
                         c.vocab, c.max_seq, int(model.attn_scale))
            arrs = []

            def add(a, dt):
                a = np.ascontiguousarray(a, dtype=dt)
                self._keep.append(a)
                arrs.append(a.ctypes.data)

            add(model.emb, np.int8); add(model.emb_s, np.int64)
            add(model.out, np.int8); add(model.out_s, np.int64)
            add(model.final_norm, np.int64)
            add(model.rope_cos, np.int64); add(model.rope_sin, np.int64)
            lens = [len(model.final_norm), len(model.rope_cos)]
            for Ly in model.layers:
                for n in ("wq", "wk", "wv", "wo", "gate", "up", "down"):
                    add(Ly[n], np.int8); add(Ly[n + "_s"], np.int64)
                add(Ly["attn_norm"], np.int64); add(Ly["ffn_norm"], np.int64)
                lens += [len(Ly["attn_norm"]), len(Ly["ffn_norm"])]
            ptrs = (C.c_void_p * len(arrs))(*arrs)
            ln = (C.c_int64 * len(lens))(*lens)
            self._keep += [ptrs, ln, cfg]
            self.h = L.arcref_from_arrays(C.byref(cfg), ptrs, ln)
            q16 = getattr(model, "emb_q16", None)
            if q16 is not None:
                q16 = np.ascontiguousarray(q16, dtype=np.int64)
                assert q16.shape == (c.vocab, c.d_model)
                self._keep.append(q16)
                L.arcref_set_embedding_q16(self.h, q16.ctypes.data)
        c = Config()
        L.arcref_get_config(self.h, C.byref(c))
        self.cfg = c

    def __del__(self):
        h = getattr(self, "h", None)
        if h and _LIB is not None:
            _LIB.arcref_free(h)
            self.h = None

    def enable_q4(self):
        lib().arcref_enable_q4(self.h)

    def save(self, path: str, vocab: Optional[List[str]] = None) -> None:
        """Write the model as an ARC-INT8 v2 file (the reference's
        ``save_weights`` bytes).  ``vocab`` None keeps the vocab of the file
        the model was loaded from (an empty list for array-built models)."""
        import json

        vj = None if vocab is None else json.dumps(vocab, ensure_ascii=False, separators=(",", ":")).encode()
        err = C.create_string_buffer(512)
        rc = lib().arcref_save_file(self.h, path.encode(), vj, 0 if vj is None else len(vj), err, 512)
        if rc != 0:
            raise OSError(err.value.decode())

    def generate(self, prompt: Sequence[int], max_tokens: int, eos: Sequence[int] = ()) -> Tuple[List[int], bytes]:
        p = np.asarray(list(prompt), dtype=np.uint32)
        e = np.asarray(list(eos), dtype=np.uint32)
        out = np.zeros(max(1, max_tokens), dtype=np.uint32)
        h = np.zeros(32, dtype=np.uint8)
        n = lib().arcref_generate(self.h, _p(p) if p.size else None, p.size, max_tokens,
                                  _p(e) if e.size else None, e.size, _p(out), _p(h))
        if n < 0:
            raise ValueError(f"{1 + len(p)} + {max_tokens} positions run past the model's RoPE tables (max_seq)")
        return [int(t) for t in out[:n]], h.tobytes()

    def weight_hash(self) -> bytes:
        h = np.zeros(32, dtype=np.uint8)
        lib().arcref_weight_hash(self.h, _p(h))
        return h.tobytes()

    def new_cache(self) -> "Cache":
        return Cache(self)


class Cache:
    def __init__(self, model: Model):
        self.model = model
        self.h = lib().arcref_cache_new(model.h)

    def __del__(self):
        if getattr(self, "h", None) and _LIB is not None:
            _LIB.arcref_cache_free(self.h)
            self.h = None

    def __len__(self):
        return lib().arcref_cache_len(self.h)

    def truncate(self, n: int):
        lib().arcref_cache_truncate(self.h, n)

    def forward(self, token: int) -> np.ndarray:
        out = np.empty(self.model.cfg.vocab, dtype=np.int64)
        lib().arcref_forward(self.model.h, self.h, int(token), _p(out))
        if lib().arcref_cache_overflow(self.h):
            raise ValueError("position past the model's RoPE tables (max_seq)")
        return out

    def last_hidden(self) -> np.ndarray:
        out = np.empty(self.model.cfg.d_model, dtype=np.int64)
        lib().arcref_last_hidden(self.h, _p(out))
        return out
