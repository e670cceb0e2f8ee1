"""Device-resident dense INT8 decoder weights (Llama-style MHA/GQA).

Fusions done once at load time (exact: they only concatenate output rows):
* ``wqkv`` = [wq; wk; wv] rows, one GEMM for the three projections
  (cached_integer_model.rs:1425-1427 runs them on the same normed input);
* ``wgu``  = [gate; up] rows (1491-1492);
Each matrix keeps its own per-row i64 scales, so every output element is
computed exactly as the reference's ``matmul_i8_into`` computes it.

Tensor-parallel sharding (``tp_rank``/``tp_size``) is Megatron-style: q/k/v
and gate/up are split by output rows (whole heads / whole FFN rows), wo and
down by input columns, the LM head by vocab rows.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from arc_chain_b200.formats import gen
from arc_chain_b200.formats.arc_int8 import Int8Model, LAYER_MATS
from arc_chain_b200.models.config import ModelConfig
from arc_chain_b200.ops import int_ops as ops


@dataclass
class Linear:
    """One INT8 matrix with per-row Q16 scales.  ``build_map`` converts the
    row-major [M, K] weight into the tiled layout the fused GEMM streams
    (128x128-byte tiles, each contiguous) and encodes its TMA map."""

    w: torch.Tensor          # int8 [M, K] row-major; tiled after build_map()
    s: torch.Tensor          # int64 [M]
    tmap: ops.TensorMap = None
    M: int = 0
    K: int = 0

    def build_map(self):
        self.M, self.K = self.w.shape
        self.w = ops.tile_weight(self.w)
        self.tmap = ops.TensorMap(self.w, ops.BM)
        return self

    q4: Optional[torch.Tensor] = None  # packed Q4 tiles (ops.pack_q4) when quantised

    def row_major(self) -> torch.Tensor:
        return ops.untile_weight(self.w, self.M, self.K)

    def to_q4(self, mode: str = "group") -> "Linear":
        """Quantise to Q4 in place.  mode "group": group-32 4-bit weights
        with 4-bit group multipliers (row scale kept); mode "values": the
        int8 data already holds Q4 values in [-8, 7] (reference per-row Q4
        prepared on the host), multipliers 1."""
        w = self.row_major()
        if mode == "group":
            q, mult = ops.q4_group_quantize(w)
        elif mode == "values":
            q = w
            mult = torch.ones(self.M, (self.K + 31) // 32, dtype=torch.uint8, device=w.device)
        else:
            raise ValueError(mode)
        self.q4 = ops.pack_q4(q, mult)
        self.w, self.tmap = None, None
        return self


@dataclass
class DenseLayer:
    qkv: Linear
    wo: Linear
    gu: Linear
    down: Linear
    attn_norm: torch.Tensor
    ffn_norm: torch.Tensor


@dataclass
class DenseModel:
    cfg: ModelConfig
    attn_scale: int
    emb: torch.Tensor
    emb_s: torch.Tensor
    lm: Linear
    final_norm: torch.Tensor
    rope_cos: torch.Tensor
    rope_sin: torch.Tensor
    layers: List[DenseLayer]
    tp_rank: int = 0
    tp_size: int = 1
    vocab_offset: int = 0
    weight_hash: Optional[bytes] = None
    emb_q16: Optional[torch.Tensor] = None  # full-precision Q16 embedding (GGUF imports)

    @property
    def n_heads_local(self):
        return self.cfg.n_heads // self.tp_size

    @property
    def n_kv_local(self):
        return self.cfg.n_kv_heads // self.tp_size

    @property
    def d_ff_local(self):
        return self.cfg.d_ff // self.tp_size

    @property
    def vocab_local(self):
        return self.lm.M


def _swap12(a):
    return a.transpose(1, 2) if isinstance(a, torch.Tensor) else np.swapaxes(a, 1, 2)


def interleave_heads(a, n_heads: int, dh: int):
    """Reorder the rows of each head from (0..half-1, half..dh-1) to
    (0, half, 1, half+1, ...): the two rows of one RoPE rotation pair become
    adjacent, so the fused GEMM epilogue rotates them with one lane shuffle.
    Works on [n_heads*dh, K] weights and [n_heads*dh] scales."""
    half = dh // 2
    tail = tuple(a.shape[1:])
    r = _swap12(a.reshape(n_heads, 2, half, *tail))
    return r.reshape(n_heads * dh, *tail)


def interleave_pairs(g, u):
    """Rows g0, u0, g1, u1, ...: gate and up of one FFN unit adjacent."""
    st = torch.stack if isinstance(g, torch.Tensor) else np.stack
    r = st([g, u], 1)
    return r.reshape(2 * g.shape[0], *tuple(g.shape[1:]))


def _contig(a):
    return a.contiguous() if isinstance(a, torch.Tensor) else np.ascontiguousarray(a)


def _shard_rows(a, rank, size):
    n = a.shape[0] // size
    return a[rank * n:(rank + 1) * n]


def _shard_cols(a, rank, size):
    n = a.shape[1] // size
    return a[:, rank * n:(rank + 1) * n]


def _vocab_range(V, rank, size):
    per = (V + size - 1) // size
    lo = min(V, rank * per)
    return lo, min(V, lo + per)


def check_tp(cfg: ModelConfig, tp: int):
    if cfg.n_heads % tp or cfg.n_kv_heads % tp or cfg.d_ff % tp:
        raise ValueError(f"{cfg.name}: heads {cfg.n_heads}/{cfg.n_kv_heads} and d_ff {cfg.d_ff} must divide by tp={tp}")
    if (cfg.d_ff // tp) % 16 or (cfg.d_model // tp) % 16:
        raise ValueError("sharded K must stay a multiple of 16 bytes (TMA row stride)")


def linears(model: "DenseModel"):
    for Ly in model.layers:
        yield from (Ly.qkv, Ly.wo, Ly.gu, Ly.down)
    yield model.lm


def to_q4(model: "DenseModel", mode: str = "group") -> "DenseModel":
    """Quantise every matrix of a device model to Q4 (see Linear.to_q4)."""
    if mode == "group" and model.tp_size > 1:
        for k in (model.cfg.d_model, model.cfg.d_ff):
            if (k // model.tp_size) % 32:
                raise ValueError("group-32 Q4 with TP needs K shards that are multiples of 32")
    for lin in linears(model):
        lin.to_q4(mode)
    torch.cuda.synchronize()
    return model


def q4_row_host(m: Int8Model) -> Int8Model:
    """The reference's per-row Q4 applied on the host before sharding
    (absmax over the whole row): data becomes the Q4 values, scales s * qpu."""
    from arc_chain_b200 import spec
    import copy

    out = copy.copy(m)
    out.out, out.out_s = spec.q4_from_i8(m.out, m.out_s)
    out.layers = []
    for L in m.layers:
        L2 = dict(L)
        for n in LAYER_MATS:
            L2[n], L2[n + "_s"] = spec.q4_from_i8(L[n], L[n + "_s"])
        out.layers.append(L2)
    return out


def from_host(m: Int8Model, device, tp_rank: int = 0, tp_size: int = 1, q4: Optional[str] = None,
              presharded: bool = False) -> DenseModel:
    """Upload an Int8Model (numpy) to the device, sharded for TP.

    q4=None keeps INT8; "row" applies the reference's per-row Q4 (every
    matrix including the LM head, as enable_q4 does); "group" the group-32
    Q4 extension.  presharded: `m` already holds rank tp_rank's slices
    (formats/sharded.py), so nothing is sliced again."""
    if q4 == "row":
        if presharded:
            raise ValueError("per-row Q4 is applied before sharding: shard a q4_row_host model instead")
        dm = from_host(q4_row_host(m), device, tp_rank, tp_size)
        return to_q4(dm, "values")
    if q4 == "group":
        return to_q4(from_host(m, device, tp_rank, tp_size, presharded=presharded), "group")
    c = m.cfg
    check_tp(c, tp_size)
    dev = torch.device(device)
    T = lambda a, dt=None: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dh = c.d_head
    layers = []
    for L in m.layers:
        r, s_ = (0, 1) if presharded else (tp_rank, tp_size)
        nhl, nkl = c.n_heads // tp_size, c.n_kv_heads // tp_size
        wq, wk, wv = (_shard_rows(L[n], r, s_) for n in ("wq", "wk", "wv"))
        sq, sk, sv = (_shard_rows(L[n + "_s"], r, s_) for n in ("wq", "wk", "wv"))
        qkv = Linear(T(np.concatenate([interleave_heads(wq, nhl, dh), interleave_heads(wk, nkl, dh), wv])),
                     T(np.concatenate([interleave_heads(sq, nhl, dh), interleave_heads(sk, nkl, dh), sv])))
        wo = Linear(T(_shard_cols(L["wo"], r, s_)), T(L["wo_s"]))
        gu = Linear(T(interleave_pairs(_shard_rows(L["gate"], r, s_), _shard_rows(L["up"], r, s_))),
                    T(interleave_pairs(_shard_rows(L["gate_s"], r, s_), _shard_rows(L["up_s"], r, s_))))
        down = Linear(T(_shard_cols(L["down"], r, s_)), T(L["down_s"]))
        layers.append(DenseLayer(qkv.build_map(), wo.build_map(), gu.build_map(), down.build_map(),
                                 T(L["attn_norm"]), T(L["ffn_norm"])))
    lo, hi = _vocab_range(c.vocab, tp_rank, tp_size)
    lm = Linear(T(m.out if presharded else m.out[lo:hi]), T(m.out_s if presharded else m.out_s[lo:hi])).build_map()
    q16 = getattr(m, "emb_q16", None)
    return DenseModel(c, int(m.attn_scale), T(m.emb), T(m.emb_s), lm, T(m.final_norm), T(m.rope_cos),
                      T(m.rope_sin), layers, tp_rank, tp_size, lo, emb_q16=None if q16 is None else T(q16))


def random_device(cfg: ModelConfig, device, seed: int = 0, tp_rank: int = 0, tp_size: int = 1) -> DenseModel:
    """Seeded random-init model generated directly on the device (identical
    values to :func:`arc_chain_b200.formats.gen.random_model`)."""
    check_tp(cfg, tp_size)
    dev = torch.device(device)
    d, dkv, dff, V = cfg.d_model, cfg.d_kv, cfg.d_ff, cfg.vocab
    r, s_ = tp_rank, tp_size

    def mat_rows(tid, rows, cols, lo, hi, out=None):
        """rows [lo, hi) of the seeded matrix `tid` (data, scales)."""
        full = torch.empty(rows * cols, dtype=torch.int8, device=dev) if out is None else out
        ops.rng_i8(seed, tid << 2, full)
        full = full.view(rows, cols)
        sc = gen.row_scales(seed, (tid << 2) | 1, rows, gen.scale_base(cols))
        return full[lo:hi], torch.from_numpy(sc[lo:hi]).to(dev)

    def rows_of(tid, rows, cols):
        n = rows // s_
        w, sc = mat_rows(tid, rows, cols, r * n, (r + 1) * n)
        return w.contiguous(), sc

    def cols_of(tid, rows, cols):
        w, sc = mat_rows(tid, rows, cols, 0, rows)
        n = cols // s_
        return w[:, r * n:(r + 1) * n].contiguous(), sc

    layers = []
    for l in range(cfg.n_layers):
        tid = lambda j: gen.layer_tensor_id(l, j)
        wq, sq = rows_of(tid(0), d, d)
        wk, sk = rows_of(tid(1), dkv, d)
        wv, sv = rows_of(tid(2), dkv, d)
        nhl, nkl = cfg.n_heads // s_, cfg.n_kv_heads // s_
        dh = cfg.d_head
        qkv = Linear(torch.cat([interleave_heads(wq, nhl, dh), interleave_heads(wk, nkl, dh), wv]).contiguous(),
                     torch.cat([interleave_heads(sq, nhl, dh), interleave_heads(sk, nkl, dh), sv]).contiguous())
        del wq, wk, wv
        wo, so = cols_of(tid(3), d, d)
        wg, sg = rows_of(tid(4), dff, d)
        wu, su = rows_of(tid(5), dff, d)
        gu = Linear(interleave_pairs(wg, wu).contiguous(), interleave_pairs(sg, su).contiguous())
        del wg, wu
        wd, sd = cols_of(tid(6), d, dff)
        an = torch.from_numpy(gen.gamma(seed, (tid(7) << 2) | 1, d)).to(dev)
        fn = torch.from_numpy(gen.gamma(seed, (tid(8) << 2) | 1, d)).to(dev)
        layers.append(DenseLayer(qkv.build_map(), Linear(wo, so).build_map(), gu.build_map(),
                                 Linear(wd, sd).build_map(), an, fn))
    emb = torch.empty(V * d, dtype=torch.int8, device=dev)
    ops.rng_i8(seed, 0 << 2, emb)
    emb = emb.view(V, d)
    emb_s = torch.from_numpy(gen.row_scales(seed, (0 << 2) | 1, V, gen.EMB_SCALE_BASE)).to(dev)
    lo, hi = _vocab_range(V, r, s_)
    lw, ls = mat_rows(1, V, d, lo, hi)
    lm = Linear(lw.contiguous(), ls).build_map()
    fnorm = torch.from_numpy(gen.gamma(seed, (2 << 2) | 1, d)).to(dev)
    rc, rs = gen.rope_tables(cfg.d_head, cfg.max_seq, cfg.rope_theta)
    torch.cuda.synchronize(dev)
    return DenseModel(cfg, cfg.resolved_attn_scale(), emb, emb_s, lm, fnorm, torch.from_numpy(rc).to(dev),
                      torch.from_numpy(rs).to(dev), layers, tp_rank, tp_size, lo)


def weight_hash_seeded(cfg: ModelConfig, seed: int, device) -> bytes:
    """The reference weight hash (BLAKE3 over each matrix's i8 bytes then its
    LE i64 row scales: embedding, output, then per layer wq wk wv wo gate up
    down; cached_integer_model.rs:1598-1617) of the seeded random model,
    regenerating each matrix row-major on the device and hashing it there."""
    from arc_chain_b200.utils.hashing import DeviceBlake3

    dev = torch.device(device)
    h = DeviceBlake3(dev)
    d, dkv, dff, V = cfg.d_model, cfg.d_kv, cfg.d_ff, cfg.vocab

    def mat(tid, rows, cols, base=None):
        w = torch.empty(rows * cols, dtype=torch.int8, device=dev)
        ops.rng_i8(seed, tid << 2, w)
        s = gen.row_scales(seed, (tid << 2) | 1, rows, gen.scale_base(cols) if base is None else base)
        h.update(w, torch.from_numpy(s.astype("<i8")).to(dev))

    mat(0, V, d, gen.EMB_SCALE_BASE)
    mat(1, V, d)
    shapes = ((d, d), (dkv, d), (dkv, d), (d, d), (dff, d), (dff, d), (d, dff))
    for l in range(cfg.n_layers):
        for j, (r, c) in enumerate(shapes):
            mat(gen.layer_tensor_id(l, j), r, c)
    return h.digest()
