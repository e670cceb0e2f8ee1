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
    """Returns (int8 [n_rows, n_cols], int64 scales [n_rows]).  NaN entries
    are skipped by the row maximum (f32::max) and quantise to 0; an infinite
    maximum saturates ``abs_max as i64``; the scale division truncates."""
    w = np.asarray(values, dtype=np.float32).reshape(n_rows, n_cols)
    # fold from 0.0 with a NaN-ignoring max, as the reference does; an empty
    # row has abs_max 0 (then 1e-10)
    abs_max = np.fmax.reduce(np.abs(w), axis=1, initial=np.float32(0)).astype(np.float32)
    abs_max = np.maximum(abs_max, np.float32(1e-10)).astype(np.float32)
    inv = (np.float32(127.0) / abs_max).astype(np.float32)
    with np.errstate(invalid="ignore"):
        r = np.clip(round_half_away_f32(w * inv[:, None]), -127, 127)
    data = np.where(np.isnan(r), 0, r).astype(np.int8)
    am = np.trunc(abs_max.astype(np.float64))
    hi = am >= 2.0 ** 63
    am_i = np.where(hi, 0.0, am).astype(np.int64)  # every value kept here is below 2^63
    am_i[hi] = np.iinfo(np.int64).max
    with np.errstate(over="ignore"):
        num = am_i * ONE + 126  # wrapping, as the reference's release build
    q = np.abs(num) // 127
    scales = np.maximum(np.where(num >= 0, q, -q), 1).astype(np.int64)
    return data, scales


def dequantize(data: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """Approximate float view (value ~= data * scale / ONE), for inspection."""
    return data.astype(np.float64) * scales[:, None] / ONE


def q4_engine_from_i8(data: np.ndarray, scales: np.ndarray):
    """The reference's second Q4 format (crates/arc-inference/src/q4_engine.rs:
    27-62, ``Q4Weights::from_i8``): per row q = ceil(absmax / 7), values
    trunc(w / q) clamped to [-7, 7], packed two per byte (low nibble = even
    column, stored biased by 8), scale s * max(q, 1).

    Returns (packed uint8 [rows, cols / 2], scales int64).  Since
    |trunc(w / ceil(absmax / 7))| <= 7 for every w of the row, the values
    equal those of the per-row Q4 that the engine runs (``enable_q4``, clamp
    [-8, 7]): the two formats differ only in the container."""
    w = np.asarray(data, dtype=np.int8)
    rows, cols = w.shape
    if cols % 2:
        raise ValueError("Q4 requires an even column count")
    amax = np.maximum(np.abs(w.astype(np.int16)).max(axis=1), 1).astype(np.int64)
    qpu = (amax + 6) // 7
    v = w.astype(np.int64)
    q = np.clip(np.sign(v) * (np.abs(v) // qpu[:, None]), -7, 7)
    nib = (q + 8).astype(np.uint8)
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    return packed, np.asarray(scales, dtype=np.int64) * np.maximum(qpu, 1)


def q4_engine_values(packed: np.ndarray) -> np.ndarray:
    """Signed values [rows, 2 * packed cols] of a ``q4_engine_from_i8`` matrix."""
    p = np.asarray(packed, dtype=np.uint8)
    out = np.empty((p.shape[0], 2 * p.shape[1]), dtype=np.int8)
    out[:, 0::2] = (p & 0x0F).astype(np.int8) - 8
    out[:, 1::2] = (p >> 4).astype(np.int8) - 8
    return out


def matmul_q4_engine(packed: np.ndarray, scales: np.ndarray, x: np.ndarray) -> np.ndarray:
    """``matmul_q4`` (q4_engine.rs:71-97): (sum_j q_j x_j) * s >> 16 with
    wrapping i64 arithmetic."""
    q = q4_engine_values(packed).astype(np.int64)
    with np.errstate(over="ignore"):
        acc = (q * np.asarray(x, dtype=np.int64)[None, :]).sum(axis=1, dtype=np.int64)
        return (acc * np.asarray(scales, dtype=np.int64)) >> 16
