"""Float -> per-row INT8 quantisation, as the reference does it when it
imports float weights (``I8Weights::quantize_f32``,
crates/arc-inference/src/cached_integer_model.rs:36-62).

Per row: abs_max = max |w| (at least 1e-10); data = round(w * (127 / abs_max))
clamped to [-127, 127], computed in f32 with Rust's round-half-away-from-zero;
scale = ((abs_max as i64) * ONE + 126) / 127, at least 1.  ``abs_max as i64``
truncates, so every row whose largest magnitude is below 1.0 gets scale 1
(a reference quirk kept on purpose: outputs must match its files).
"""
from __future__ import annotations

import numpy as np

ONE = 1 << 16


def round_half_away_f32(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float32)
    t = np.trunc(v)
    f = v - t
    return t + (f >= np.float32(0.5)).astype(np.float32) - (f <= np.float32(-0.5)).astype(np.float32)


def quantize_f32(values: np.ndarray, n_rows: int, n_cols: int):
    """Returns (int8 [n_rows, n_cols], int64 scales [n_rows])."""
    w = np.asarray(values, dtype=np.float32).reshape(n_rows, n_cols)
    abs_max = np.maximum(np.abs(w).max(axis=1), np.float32(1e-10)).astype(np.float32)
    inv = (np.float32(127.0) / abs_max).astype(np.float32)
    data = np.clip(round_half_away_f32(w * inv[:, None]), -127, 127).astype(np.int8)
    am_i = np.trunc(abs_max).astype(np.int64)
    scales = np.maximum((am_i * ONE + 126) // 127, 1).astype(np.int64)
    return data, scales


def dequantize(data: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Approximate float view (value ~= data * scale / ONE), for inspection."""
    return data.astype(np.float64) * scales[:, None] / ONE
