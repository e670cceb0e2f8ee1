"""torch-facing wrappers of the sm_100a kernels (one call = one kernel launch).

Every wrapper launches on ``torch.cuda.current_stream()`` and counts its
launch in :data:`LAUNCHES` so benchmarks can report how many of this
library's kernels ran in a timed region.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import torch

from arc_chain_b200.ops._lib import check, lib

LAUNCHES = [0]
BM, BK = 128, 128


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _s():
    return torch.cuda.current_stream().cuda_stream


def _count():
    LAUNCHES[0] += 1


class TensorMap:
    """A CUtensorMap (128 bytes, 64-byte aligned host memory) over a 2-D int8
    tensor [rows, cols], box = {128 bytes of K, box_rows}, 128-byte swizzle.

    For a limb operand, ``enc_rows`` < ``box_rows`` encodes a shorter box: the
    fused GEMM then loads a BN = box_rows tile as box_rows / enc_rows boxes and
    skips those past the live rows."""

    def __init__(self, t: torch.Tensor, box_rows: int, enc_rows: Optional[int] = None):
        assert t.dtype == torch.int8 and t.dim() == 2 and t.is_contiguous()
        self._raw = C.create_string_buffer(128 + 64)
        self.addr = (C.addressof(self._raw) + 63) & ~63
        self.tensor = t
        self.rows, self.cols = t.shape
        self.box_rows = box_rows
        self.enc_rows = enc_rows or box_rows
        assert box_rows % self.enc_rows == 0
        rc = lib().arcb_tmap_i8(self.addr, t.data_ptr(), self.rows, self.cols, self.enc_rows)
        if rc != 0:
            raise RuntimeError(f"cuTensorMapEncodeTiled failed ({rc}) for {tuple(t.shape)} box {box_rows}")


def gemm_bn(B: int) -> int:
    return lib().arcb_gemm_bn(B)


_SMS = [None]


def num_sms() -> int:
    if _SMS[0] is None:
        _SMS[0] = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return _SMS[0]


def gemm_i8(wmap: TensorMap, xmap: TensorMap, M: int, K: int, B: int, ksplit: int, lmax: torch.Tensor,
            P: torch.Tensor, err: torch.Tensor) -> None:
    _count()
    check(lib().arcb_gemm_i8(wmap.addr, xmap.addr, M, K, B, xmap.box_rows, ksplit, _p(lmax), _p(P), _p(err), _s()),
          "gemm_i8")


def embed(tokens, emb, emb_s, V, d, B, h, counters, ss):
    """h = embedding rows; ss[0] = first norm's sum of squares; zeroes
    counters and ss[1:] (ss is [n_norms, B] int64 viewed as u64)."""
    _count()
    check(lib().arcb_embed(_p(tokens), _p(emb), _p(emb_s), V, d, B, _p(h), _p(counters), counters.numel(), _p(ss),
                           ss.shape[0], _s()), "embed")


def norm_limbs(h, ss_row, gamma, d, B, X, lmax, y_out=None):
    _count()
    check(lib().arcb_norm_limbs(_p(h), _p(ss_row), _p(gamma), gamma.numel(), d, B, _p(X), _p(lmax), _p(y_out),
                                _s()), "norm_limbs")


def rmsnorm_limbs(h, gamma, d, B, X, lmax, y_out=None):
    _count()
    check(lib().arcb_rmsnorm_limbs(_p(h), _p(gamma), gamma.numel(), d, B, _p(X), _p(lmax), _p(y_out), _s()),
          "rmsnorm_limbs")


def finalize(P, M, B, lmax, scales, out, ldo, mode, ss_out=None):
    _count()
    check(lib().arcb_finalize(_p(P), M, B, _p(lmax), _p(scales), _p(out), ldo, mode, _p(ss_out), _s()), "finalize")


def sample(logits, V, n, hist, count, gen, tokens_next, pos_inc=None, done=None, eos=None, lrow=None):
    _count()
    n_eos = 0 if eos is None else eos.numel()
    check(lib().arcb_sample(_p(logits), logits.shape[1], V, _p(lrow), n, _p(hist), _p(count), _p(gen),
                            gen.shape[1], _p(tokens_next), _p(pos_inc), _p(done), _p(eos), n_eos, _s()),
          "sample")


def rng_i8(seed: int, stream: int, out: torch.Tensor) -> None:
    _count()
    check(lib().arcb_rng_i8(seed, stream, _p(out), out.numel(), _s()), "rng_i8")


# --------------------------------------------------------------- fused GEMM
class Epi(C.Structure):
    """Mirror of fg::Epi (csrc/kernels/gemm_fused.cu)."""

    _fields_ = [("mode", C.c_int), ("scales", C.c_void_p), ("out", C.c_void_p), ("ldo", C.c_int),
                ("ss_out", C.c_void_p), ("n_heads", C.c_int), ("n_kv", C.c_int), ("dh", C.c_int),
                ("q_out", C.c_void_p), ("Kc", C.c_void_p), ("Vc", C.c_void_p), ("pt", C.c_void_p),
                ("pt_stride", C.c_int), ("pos", C.c_void_p), ("rcos", C.c_void_p), ("rsin", C.c_void_p),
                ("max_seq", C.c_int), ("X", C.c_void_p), ("ldx", C.c_int), ("lmax_out", C.c_void_p),
                ("err", C.c_void_p), ("B", C.c_int),
                ("rp", C.c_int), ("npeers", C.c_int), ("rank", C.c_int), ("peer_R", C.c_void_p),
                ("peer_cnt", C.c_void_p), ("cnt_local", C.c_void_p), ("prof", C.c_void_p),
                ("grp_rows", C.c_int), ("grp_koff", C.c_int), ("route", C.c_void_p), ("route_ld", C.c_int),
                ("max_ctas", C.c_int), ("b_box", C.c_int), ("route_gs", C.c_int), ("peer_h", C.c_void_p),
                ("peer_sig", C.c_void_p), ("sched", C.c_int), ("rs_ag", C.c_int), ("rs_cnt_off", C.c_int),
                ("ep_rows", C.c_int)]


PARTIAL, STORE, RESID, QKV, SWIGLU, MOE_COMBINE, STORE_PEERS = 0, 1, 2, 3, 4, 5, 6


def fgemm_bn(B: int) -> int:
    return lib().arcb_fgemm_bn(B)


def fgemm(wmap: TensorMap, xmap: TensorMap, M: int, K: int, B: int, lmax, P, tile_cnt, epi: Epi,
          pdl: bool = True) -> None:
    """Persistent stream-K limb GEMM with the finalize fused in (mode in epi)."""
    _count()
    epi.b_box = xmap.enc_rows if xmap.enc_rows < xmap.box_rows else 0
    check(lib().arcb_fgemm(wmap.addr, xmap.addr, M, K, B, xmap.box_rows, _p(lmax), _p(P), _p(tile_cnt),
                           C.addressof(epi), int(pdl), _s()), "fgemm")


def epi(mode, scales, err, **kw) -> Epi:
    e = Epi()
    e.mode = mode
    e.scales = _p(scales)
    e.err = _p(err)
    for k, v in kw.items():
        setattr(e, k, _p(v) if isinstance(v, torch.Tensor) else v)
    return e


def set_pdl(on: bool) -> None:
    lib().arcb_set_pdl(int(on))


def set_attn_paged(on: bool) -> None:
    """Decode attention for standard heads: TMA-fed page ring (True, the
    default) or per-thread loads (False); identical results."""
    lib().arcb_set_attn_paged(int(on))


def tile_weight(w: torch.Tensor) -> torch.Tensor:
    """[M, K] int8 -> tiled [Mt*nch*128, 128]: tile (m, k) (128 rows x 128
    bytes, zero padded at the M and K edges) is contiguous at row
    (m*nch + k)*128, the order the fused GEMM streams it."""
    M, K = w.shape
    Mt, nch = (M + BM - 1) // BM, (K + BK - 1) // BK
    if M % BM or K % BK:
        wp = torch.zeros(Mt * BM, nch * BK, dtype=torch.int8, device=w.device)
        wp[:M, :K] = w
    else:
        wp = w
    return wp.view(Mt, BM, nch, BK).permute(0, 2, 1, 3).contiguous().view(Mt * nch * BM, BK)


def untile_weight(t: torch.Tensor, M: int, K: int) -> torch.Tensor:
    Mt, nch = (M + BM - 1) // BM, (K + BK - 1) // BK
    return t.view(Mt, nch, BM, BK).permute(0, 2, 1, 3).reshape(Mt * BM, nch * BK)[:M, :K].contiguous()


def attn_cluster_size(B: int, n_heads: int) -> int:
    """CTAs per (slot, head): spread few heads over many SMs, keep one CTA
    per head when the batch already fills the GPU."""
    n = B * n_heads
    return 8 if n <= 64 else (4 if n <= 128 else (2 if n <= 512 else 1))


def attn(q, Kc, Vc, pt, pos, n_heads, n_kv, dh, attn_scale, B, X, lmax, max_T, err, o_out=None, cluster=None):
    """Exact paged decode attention, one launch (thread-block clusters)."""
    _count()
    cs = cluster or attn_cluster_size(B, n_heads)
    check(lib().arcb_attn_cluster(_p(q), _p(Kc), _p(Vc), _p(pt), pt.shape[1], _p(pos), n_heads, n_kv, dh,
                                  int(attn_scale), max_T, B, cs, _p(X), _p(lmax), _p(o_out), _p(err), _s()),
          "attn_cluster")


def attn_prefill(q, Kc, Vc, pt_row, nq, p0, n_heads, n_kv, dh, attn_scale, B, X, lmax, max_T, err) -> bool:
    """Causal attention of a prefill chunk (slots [0, nq) = positions p0 ..
    p0 + nq - 1 of one sequence, page-table row `pt_row`; slots [nq, B)
    padding): every K/V page is read once per 16 positions.  False when the
    chunk's scores do not fit in shared memory (nothing was launched)."""
    rc = lib().arcb_attn_prefill(_p(q), _p(Kc), _p(Vc), _p(pt_row), nq, p0, n_heads, n_kv, dh, int(attn_scale), max_T,
                                 B, _p(X), _p(lmax), _p(err), _s())
    if rc == -3:
        return False
    _count()
    check(rc, "attn_prefill")
    return True


def attn_gqa_block(q, Kc, Vc, pt, pos, n_heads, n_kv, dh, attn_scale, B, X, lmax, max_T, t_lim, err) -> bool:
    """Grouped-query decode attention, one CTA per (slot, KV head) serving
    that KV head's query heads (each page read once for all of them).
    t_lim bounds every slot's position + 1.  False when the scores do not
    fit in shared memory (nothing was launched)."""
    rc = lib().arcb_attn_gqa_block(_p(q), _p(Kc), _p(Vc), _p(pt), pt.shape[1], _p(pos), n_heads, n_kv, dh,
                                   int(attn_scale), max_T, t_lim, B, _p(X), _p(lmax), _p(err), _s())
    if rc == -3:
        return False
    _count()
    check(rc, "attn_gqa_block")
    return True


# --------------------------------------------------------------- Q4 weights
Q4_TILE = 128 * 64 + 128 * 2


def pack_q4(q: torch.Tensor, mult: torch.Tensor) -> torch.Tensor:
    """Pack Q4 weights into the tiles the Q4 GEMM streams.

    q: int [M, K] values in [-8, 7]; mult: int [M, ceil(K/32)] group
    multipliers in [1, 15].  Tile (m, k) (128 rows x 128 columns) is
    Q4_TILE contiguous bytes: 128 rows x 64 bytes of bias-8 nibbles (low
    nibble = even column) then 128 rows x 2 bytes of multipliers (group g
    of the chunk in bits 4g..4g+3).  Padding is q = 0, multiplier 1."""
    M, K = q.shape
    Mt, nch = (M + BM - 1) // BM, (K + BK - 1) // BK
    dev = q.device
    qp = torch.zeros(Mt * BM, nch * BK, dtype=torch.int16, device=dev)
    qp[:M, :K] = q.to(torch.int16)
    nib = (qp + 8).to(torch.uint8)
    packed = nib[:, 0::2] | (nib[:, 1::2] << 4)
    ng = (K + 31) // 32
    mp = torch.ones(Mt * BM, nch * 4, dtype=torch.int32, device=dev)
    mp[:M, :ng] = mult.to(torch.int32)
    mm = mp.view(Mt * BM, nch, 4)
    m16 = (mm[..., 0] | (mm[..., 1] << 4) | (mm[..., 2] << 8) | (mm[..., 3] << 12))
    mb = torch.stack([(m16 & 0xFF), (m16 >> 8) & 0xFF], -1).to(torch.uint8)  # [Mt*128, nch, 2]
    nibt = packed.view(Mt, BM, nch, 64).permute(0, 2, 1, 3).reshape(Mt * nch, BM * 64)
    mbt = mb.view(Mt, BM, nch, 2).permute(0, 2, 1, 3).reshape(Mt * nch, BM * 2)
    return torch.cat([nibt, mbt], 1).contiguous().view(-1)


def q4_group_quantize(w: torch.Tensor):
    """Group-32 Q4 of an int8 matrix (the extension format): per 32-column
    group m = clamp(ceil(absmax / 7), 1, 15), q = clamp(trunc(w / m), -8, 7);
    the effective int8 weight is m * q and the row scale is unchanged."""
    M, K = w.shape
    ng = (K + 31) // 32
    wp = torch.zeros(M, ng * 32, dtype=torch.int32, device=w.device)
    wp[:, :K] = w.to(torch.int32)
    g = wp.view(M, ng, 32)
    am = g.abs().amax(-1).clamp(min=1)
    m = ((am + 6) // 7).clamp(1, 15)
    q = torch.div(g, m.unsqueeze(-1), rounding_mode="trunc").clamp(-8, 7).view(M, ng * 32)[:, :K]
    return q.to(torch.int8), m.to(torch.uint8)


def fgemm_q4(packed: torch.Tensor, xmap: TensorMap, M: int, K: int, B: int, lmax, P, tile_cnt, epi: Epi,
             pdl: bool = True) -> None:
    """K2: the fused GEMM over Q4 tiles (dequantised to int8 in shared memory)."""
    _count()
    epi.b_box = xmap.enc_rows if xmap.enc_rows < xmap.box_rows else 0
    check(lib().arcb_fgemm_q4(_p(packed), xmap.addr, M, K, B, xmap.box_rows, _p(lmax), _p(P), _p(tile_cnt),
                              C.addressof(epi), int(pdl), _s()), "fgemm_q4")


# (max batch, CTAs per tile) pairs for split_ctas; the last entry covers all
# larger batches.
SPLIT_TABLE = [(2, 64), (8, 4), (32, 2), (1 << 30, 1)]


def limb_slots(B: int) -> int:
    """Slots per block of the limb-operand layout (csrc/kernels/common.cuh limb_row)."""
    return min(B, 32)


def n_tiles(B: int) -> int:
    """N tiles of the fused GEMM for B slots (one per 32-slot block)."""
    S = limb_slots(B)
    return (B + S - 1) // S


def limb_rows(B: int, bn: Optional[int] = None) -> int:
    """Rows of a limb operand of B slots (every block's 8 planes, at least one TMA box)."""
    return max(8 * n_tiles(B) * limb_slots(B), bn or fgemm_bn(B))


def tile_counters(M: int, B: int) -> int:
    """Entries of the fused GEMM's per-(M tile, N tile) arrival counters."""
    return ((M + BM - 1) // BM) * n_tiles(B) + 1


def limb_row(l: int, b: int, B: int) -> int:
    S = limb_slots(B)
    return (b // S) * 8 * S + l * S + b % S


def limb_planes(x, rows: Optional[int] = None):
    """Host limb operand of int64 values x [B, K]: (int8 [rows, K] in the
    limb_row layout, limb count); signed radix-256 digits."""
    import numpy as np

    x = np.asarray(x, dtype=np.int64)
    B, K = x.shape
    rows = rows or limb_rows(B)
    out = np.zeros((rows, K), dtype=np.int8)
    r = x.copy()
    need = 0
    for l in range(8):
        d = (r & 0xFF).astype(np.uint8).view(np.int8)
        for b in range(B):
            out[limb_row(l, b, B)] = d[b]
        r = (r - d.astype(np.int64)) >> 8
        if np.any(d != 0):
            need = l + 1
    return out, max(need, 1)


def split_ctas(M: int, B: int, bn: int) -> int:
    """CTA budget of the stream-K GEMM: at decode batch 1-2 every SM streams
    (tiles split many ways; the partials are few); as the batch grows each
    split adds B x limbs partials per row, so tiles are shared by fewer CTAs."""
    splits = next(s for b, s in SPLIT_TABLE if B <= b)
    mt = (M + BM - 1) // BM
    return max(1, mt * n_tiles(B) * splits)


def linear_gemm(lin, xmap: TensorMap, B: int, lmax, P, tile_cnt, epi: Epi) -> None:
    """Dispatch a Linear (int8 tiles or Q4 tiles) to its fused GEMM."""
    if not epi.peer_sig:  # expert-parallel arrival counts assume the full grid
        epi.max_ctas = min(num_sms(), split_ctas(lin.M, B, xmap.box_rows))
    if getattr(lin, "q4", None) is not None:
        fgemm_q4(lin.q4, xmap, lin.M, lin.K, B, lmax, P, tile_cnt, epi)
    else:
        fgemm(lin.tmap, xmap, lin.M, lin.K, B, lmax, P, tile_cnt, epi)


def verify_sample(logits, V: int, lanes: int, k: int, drafts, hist, count, y) -> None:
    """Speculative verify: penalty + argmax at each of the k+1 positions of
    every lane, with history = confirmed tokens + the preceding drafts."""
    _count()
    check(lib().arcb_verify_sample(_p(logits), logits.shape[1], V, lanes, k, _p(drafts), _p(hist), _p(count),
                                   _p(y), _s()), "verify_sample")


# --------------------------------------------------------------- MLA / MoE
def mla_kv(kva, r, dr, gamma, cache, pt, pos, rcos, rsin, max_seq, B, err):
    _count()
    check(lib().arcb_mla_kv(_p(kva), r, dr, _p(gamma), gamma.numel(), _p(cache), _p(pt), pt.shape[1], _p(pos),
                            _p(rcos), _p(rsin), max_seq, B, _p(err), _s()), "mla_kv")


def mla_q(q, H, dn, dr, r, Wuk, suk, pos, rcos, rsin, max_seq, B, Q):
    _count()
    check(lib().arcb_mla_q(_p(q), H, dn, dr, r, _p(Wuk), _p(suk), _p(pos), _p(rcos), _p(rsin), max_seq, B, _p(Q),
                           _s()), "mla_q")


def mla_out(oc, H, r, dv, Wuv, suv, B, X, lmax, o_out=None):
    _count()
    check(lib().arcb_mla_out(_p(oc), H, r, dv, _p(Wuv), _p(suv), B, _p(X), _p(lmax), _p(o_out), _s()), "mla_out")


def attn_mla(Q, cache, pt, pos, H, dk, dv, attn_scale, max_T, B, oc, err, cluster=None):
    """MLA latent attention (per-(slot, head) cluster kernel).  Clusters of 8
    CTAs at every batch: with 576-wide latent rows the per-thread loads are
    latency bound, and more CTAs per head keep more of them in flight
    (16 heads, T = 512: 154 vs 187 us at 16 slots, 297 vs 335 us at 32,
    against clusters of 2)."""
    _count()
    cs = cluster or 8
    check(lib().arcb_attn_mla(_p(Q), _p(cache), _p(pt), pt.shape[1], _p(pos), H, dk, dv, int(attn_scale), max_T, B,
                              cs, _p(oc), _p(err), _s()), "attn_mla")


def moe_route(logits, E, S, top_k, B, route):
    _count()
    check(lib().arcb_moe_route(_p(logits), logits.shape[1], E, S, top_k, B, _p(route), _s()), "moe_route")


def ep_wait_apply(cnt, epoch, per_call: int, h, delta, done, err) -> None:
    """Expert-parallel combine: bounded wait for this call's arrivals, then
    h += delta (wrapping) and delta = 0 (csrc/kernels/ep_ops.cu)."""
    _count()
    check(lib().arcb_ep_wait_apply(_p(cnt), _p(epoch), per_call, _p(h), _p(delta), 0 if h is None else h.numel(),
                                   _p(done), _p(err), _s()), "ep_wait_apply")


def ep_dispatch(X, B: int, ldx: int, route, G: int, lcnt, rank: int, npeers: int, peer_X, peer_route, peer_counts,
                peer_sig, cnt, epoch, gcnt, zero_cnt, blocks: int, err) -> None:
    """Expert-parallel token dispatch: this rank's limb planes and routing
    weights into every rank's gathered buffers, then a bounded wait for all
    ranks' (csrc/kernels/ep_ops.cu)."""
    _count()
    check(lib().arcb_ep_dispatch(_p(X), B, ldx, _p(route), G, _p(lcnt), rank, npeers, _p(peer_X), _p(peer_route),
                                 _p(peer_counts), _p(peer_sig), _p(cnt), _p(epoch), _p(gcnt), _p(zero_cnt), blocks,
                                 _p(err), _s()), "ep_dispatch")


def check_udiv(den0: int, den1: int, n_rand: int) -> int:
    """Mismatches of the kernels' small-quotient division against the
    compiler's 64-bit division (csrc/kernels/decode_ops.cu: k_check_udiv)."""
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    check(lib().arcb_check_udiv(den0, den1, n_rand, _p(bad), _s()), "check_udiv")
    return int(bad.item())
