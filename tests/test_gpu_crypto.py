"""GPU crypto kernels against the CPU implementations and independent
libraries: BLAKE3 batch commitments / Merkle roots."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
blake3 = pytest.importorskip("blake3")

from arc_chain_b200.crypto import commit

pytestmark = pytest.mark.gpu

LENS = [0, 1, 3, 4, 63, 64, 65, 127, 255, 256, 1023, 1024, 1025, 2048, 3071, 5000, 70001]


@pytest.mark.parametrize("with_domain", [False, True])
def test_batch_commit_gpu_matches_cpu(with_domain):
    rng = np.random.default_rng(1)
    items = [os.urandom(n) for n in LENS] + [os.urandom(int(x)) for x in rng.integers(0, 300, 3000)]
    doms = [int(x) for x in rng.integers(0, 256, len(items))] if with_domain else None
    got = commit.batch_commit(items, doms)
    assert got == commit.batch_commit_cpu(items, doms)
    h = blake3.blake3(derive_key_context=commit.TX_CONTEXT)
    if with_domain:
        h.update(bytes([doms[-1]]))
    h.update(items[-1])
    assert got[-1] == h.digest()


@pytest.mark.parametrize("n", [0, 1, 2, 3, 5, 8, 1000, 4097])
def test_merkle_root_gpu_matches_cpu(n):
    leaves = [blake3.blake3(i.to_bytes(4, "little")).digest() for i in range(n)]
    assert commit.merkle_root(leaves) == commit.merkle_root_cpu(leaves)


# ---------------------------------------------------------------- Ed25519
from arc_chain_b200.crypto import ed25519_ref as E  # noqa: E402

P = E.P


def _rec(a: int, b: int = 0, nb: int = 32) -> bytes:
    return a.to_bytes(32, "little") + b.to_bytes(32, "little")


def _vals(rng, n):
    edge = [0, 1, 2, 19, P - 1, P, P + 1, P + 18, 2 ** 255 - 1, 2 ** 254, 2 ** 26 - 1, 2 ** 51]
    return edge + [int.from_bytes(rng.bytes(32), "little") & (2 ** 255 - 1) for _ in range(n)]


def _run(op, recs):
    from arc_chain_b200.crypto import ed25519 as G

    arr = np.frombuffer(b"".join(recs), dtype=np.uint8).reshape(len(recs), 64)
    out, code = G.selftest(op, arr)
    return [bytes(o) for o in out], list(code)


def test_field_ops():
    rng = np.random.default_rng(5)
    a, b = _vals(rng, 300), _vals(rng, 300)[::-1]
    cases = {0: lambda x, y: x * y % P, 1: lambda x, y: x * x % P, 2: lambda x, y: pow(x, P - 2, P),
             3: lambda x, y: pow(x, (P - 5) // 8, P)}
    for op, f in cases.items():
        got, _ = _run(op, [_rec(x, y) for x, y in zip(a, b)])
        want = [f(x % P, y % P).to_bytes(32, "little") for x, y in zip(a, b)]
        assert got == want, op


def test_mod_l():
    rng = np.random.default_rng(6)
    L = E.L
    xs = [0, 1, L - 1, L, L + 1, 2 * L, 3 * L - 1, 2 ** 512 - 1, 2 ** 256, 2 ** 511] + \
        [int.from_bytes(rng.bytes(64), "little") for _ in range(500)]
    got, _ = _run(4, [x.to_bytes(64, "little") for x in xs])
    assert got == [(x % L).to_bytes(32, "little") for x in xs]


def test_scalar_mults_and_decompress():
    rng = np.random.default_rng(7)
    L = E.L
    ss = [0, 1, 2, 15, 16, L - 1, L - 2] + [int.from_bytes(rng.bytes(32), "little") % L for _ in range(60)]
    got, _ = _run(5, [_rec(s) for s in ss])
    assert got == [E.encode(E.mul(s, E.B)) for s in ss]
    pts = [E.encode(E.mul(int.from_bytes(rng.bytes(32), "little") % L, E.B)) for _ in range(len(ss))]
    got, code = _run(6, [s.to_bytes(32, "little") + p for s, p in zip(ss, pts)])
    assert list(code) == [0] * len(ss)
    assert got == [E.encode(E.mul(s, E.decode(p))) for s, p in zip(ss, pts)]
    # decompression: valid points, random (mostly invalid) encodings, x = 0 with the sign bit
    encs = pts + [rng.bytes(32) for _ in range(100)] + [(1).to_bytes(32, "little"),
                                                        (1 | (1 << 255)).to_bytes(32, "little")]
    got, code = _run(7, [e + bytes(32) for e in encs])
    for e, g, c in zip(encs, got, code):
        d = E.decode(e)
        assert (c == 0) == (d is not None)
        if d is not None:
            assert g == E.encode(d)


def _sigs(n, rng):
    nacl = pytest.importorskip("nacl.signing")
    msgs, sigs, pks = [], [], []
    for i in range(n):
        sk = nacl.SigningKey(rng.bytes(32))
        m = rng.bytes(int(rng.integers(0, 400)))
        msgs.append(m)
        sigs.append(sk.sign(m).signature)
        pks.append(bytes(sk.verify_key))
    return msgs, sigs, pks


def test_ed25519_verify_matches_oracle():
    from arc_chain_b200.crypto import ed25519 as G

    rng = np.random.default_rng(8)
    msgs, sigs, pks = _sigs(400, rng)
    # corruptions: flipped bits in R / S / A / message, S + L, small-order keys and R
    small = [E.encode(E.IDENT), (2 ** 255 - 20).to_bytes(32, "little"), bytes(32)]
    for i in range(0, 400, 5):
        kind = (i // 5) % 7
        s, a, m = bytearray(sigs[i]), bytearray(pks[i]), bytearray(msgs[i])
        if kind == 0:
            s[int(rng.integers(0, 32))] ^= 1 << int(rng.integers(0, 8))
        elif kind == 1:
            s[32 + int(rng.integers(0, 31))] ^= 1 << int(rng.integers(0, 8))
        elif kind == 2:
            a[int(rng.integers(0, 32))] ^= 1 << int(rng.integers(0, 8))
        elif kind == 3:
            m = bytearray(m + b"x")
        elif kind == 4:
            S = int.from_bytes(bytes(s[32:]), "little") + E.L
            s[32:] = S.to_bytes(32, "little")
        elif kind == 5:
            a = bytearray(small[(i // 35) % 3])
        else:
            s[:32] = small[(i // 35) % 3]
        sigs[i], pks[i], msgs[i] = bytes(s), bytes(a), bytes(m)
    codes = G.verify_codes(msgs, sigs, pks)
    want = [E.verify_strict(a, m, s) for m, s, a in zip(msgs, sigs, pks)]
    assert [c == 0 for c in codes] == want
    assert sum(want) > 300 and not all(want)
    # the prehashed record layout gives the same answers
    recs = torch.from_numpy(G.prehash_records(msgs, sigs, pks)).cuda()
    assert list(G.verify_prehashed_device(recs).cpu().numpy()) == list(codes)
