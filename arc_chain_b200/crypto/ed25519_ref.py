"""Ed25519 in plain Python integers: the oracle of the GPU batch verifier and
the source of every constant it uses.

Written from the curve's definition (RFC 8032 section 5.1: the twisted
Edwards curve -x^2 + y^2 = 1 + d x^2 y^2 over GF(2^255 - 19),
d = -121665/121666, base point y = 4/5 with even x, group order L) and
FIPS 180-4 (SHA-512).  Constants are computed here from those definitions,
not transcribed: d, sqrt(-1) and the base point from field arithmetic, the
SHA-512 round constants and initial hash words from the fractional parts of
cube and square roots of the first primes.

Verification follows the strict rule of the reference's batch verifier
(``VerifyingKey::verify_strict`` in crates/arc-gpu/src/lib.rs:470-495;
GPU kernel crates/arc-gpu/src/cuda/ed25519_verify.cu:432-494):
  * S must be canonical (S < L);
  * A and R must decompress (y is taken mod p; the square root must exist;
    x = 0 with the sign bit set is accepted as x = 0) and must not be of
    small order ([8]P != identity);
  * k = SHA-512(R || A || M) mod L;
  * accept iff encode([S]B - [k]A) == R (byte equality; cofactorless).
"""
from __future__ import annotations

import hashlib
from typing import List, Optional, Sequence, Tuple

P = 2 ** 255 - 19
L = 2 ** 252 + 27742317777372353535851937790883648493


def inv(x: int) -> int:
    return pow(x, P - 2, P)


D = (-121665 * inv(121666)) % P
D2 = (2 * D) % P
SQRT_M1 = pow(2, (P - 1) // 4, P)
assert SQRT_M1 * SQRT_M1 % P == P - 1


def recover_x(y: int, sign: int) -> Optional[int]:
    """x with x^2 = (y^2 - 1) / (d y^2 + 1) and parity `sign`; None if none."""
    y %= P
    u = (y * y - 1) % P
    v = (D * y * y + 1) % P
    x2 = u * inv(v) % P
    if x2 == 0:
        return 0  # x = 0 (the sign bit is ignored, as the strict verifier does)
    x = pow(x2, (P + 3) // 8, P)
    if (x * x - x2) % P != 0:
        x = x * SQRT_M1 % P
    if (x * x - x2) % P != 0:
        return None
    if (x & 1) != sign:
        x = P - x
    return x


BY = 4 * inv(5) % P
BX = recover_x(BY, 0)
# extended coordinates (X, Y, Z, T), x = X/Z, y = Y/Z, x y = T/Z
Point = Tuple[int, int, int, int]
B: Point = (BX, BY, 1, BX * BY % P)
IDENT: Point = (0, 1, 1, 0)


def add(p: Point, q: Point) -> Point:
    """Unified addition in extended coordinates for a = -1 (complete, since
    d is not a square mod p)."""
    X1, Y1, Z1, T1 = p
    X2, Y2, Z2, T2 = q
    a = (Y1 - X1) * (Y2 - X2) % P
    b = (Y1 + X1) * (Y2 + X2) % P
    c = T1 * D2 * T2 % P
    dd = Z1 * 2 * Z2 % P
    e, f, g, h = b - a, dd - c, dd + c, b + a
    return (e * f % P, g * h % P, f * g % P, e * h % P)


def neg(p: Point) -> Point:
    X, Y, Z, T = p
    return ((-X) % P, Y, Z, (-T) % P)


def mul(s: int, p: Point) -> Point:
    q = IDENT
    while s > 0:
        if s & 1:
            q = add(q, p)
        p = add(p, p)
        s >>= 1
    return q


def affine(p: Point) -> Tuple[int, int]:
    zi = inv(p[2])
    return p[0] * zi % P, p[1] * zi % P


def encode(p: Point) -> bytes:
    x, y = affine(p)
    return (y | ((x & 1) << 255)).to_bytes(32, "little")


def decode(b: bytes) -> Optional[Point]:
    v = int.from_bytes(b, "little")
    y, sign = v & ((1 << 255) - 1), v >> 255
    x = recover_x(y, sign)
    if x is None:
        return None
    y %= P
    return (x, y, 1, x * y % P)


def is_small_order(p: Point) -> bool:
    q = mul(8, p)
    return q[0] % P == 0 and (q[1] - q[2]) % P == 0


def h_scalar(R: bytes, A: bytes, msg: bytes) -> int:
    return int.from_bytes(hashlib.sha512(R + A + msg).digest(), "little") % L


# ---------------------------------------------------------------- keys and signatures (test vectors)
def secret_expand(seed: bytes) -> Tuple[int, bytes]:
    h = hashlib.sha512(seed).digest()
    a = int.from_bytes(h[:32], "little")
    a &= (1 << 254) - 8
    a |= 1 << 254
    return a, h[32:]


def public_key(seed: bytes) -> bytes:
    a, _ = secret_expand(seed)
    return encode(mul(a, B))


def sign(seed: bytes, msg: bytes) -> bytes:
    a, prefix = secret_expand(seed)
    A = encode(mul(a, B))
    r = int.from_bytes(hashlib.sha512(prefix + msg).digest(), "little") % L
    R = encode(mul(r, B))
    k = h_scalar(R, A, msg)
    S = (r + k * a) % L
    return R + S.to_bytes(32, "little")


def verify_strict(pk: bytes, msg: bytes, sig: bytes) -> bool:
    if len(sig) != 64 or len(pk) != 32:
        return False
    Rb, Sb = sig[:32], sig[32:]
    S = int.from_bytes(Sb, "little")
    if S >= L:
        return False
    A = decode(pk)
    R = decode(Rb)
    if A is None or R is None or is_small_order(A) or is_small_order(R):
        return False
    k = h_scalar(Rb, pk, msg)
    return encode(add(mul(S, B), neg(mul(k, A)))) == Rb


# ---------------------------------------------------------------- device constants
def fe_limbs(x: int) -> List[int]:
    """Radix 2^25.5 limbs (26, 25, 26, ... bits) of a canonical field value."""
    x %= P
    out, pos = [], 0
    for i in range(10):
        b = 26 if i % 2 == 0 else 25
        out.append((x >> pos) & ((1 << b) - 1))
        pos += b
    return out


def base_table() -> List[List[int]]:
    """T[i][j-1] = j * 16^i * B for i < 64, j = 1..8, as (y+x, y-x, 2d x y)
    limb triples (30 int32 per entry)."""
    rows = []
    base = B
    for i in range(64):
        q = IDENT
        for j in range(1, 9):
            q = add(q, base)
            x, y = affine(q)
            rows.append(fe_limbs(y + x) + fe_limbs(y - x) + fe_limbs(D2 * x * y))
        for _ in range(4):
            base = add(base, base)
    return rows


def _primes(n: int) -> List[int]:
    out, c = [], 2
    while len(out) < n:
        if all(c % q for q in out if q * q <= c):
            out.append(c)
        c += 1
    return out


def _iroot(v: int, k: int) -> int:
    """floor(v ** (1/k)) for integers."""
    lo, hi = 0, 1 << (v.bit_length() // k + 1)
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if mid ** k <= v:
            lo = mid
        else:
            hi = mid - 1
    return lo


def sha512_constants() -> Tuple[List[int], List[int]]:
    """(K[80], H0[8]) of FIPS 180-4: the first 64 bits of the fractional parts
    of the cube roots of the first 80 primes / square roots of the first 8."""
    ps = _primes(80)
    K = [_iroot(q << 192, 3) & ((1 << 64) - 1) for q in ps]
    H = [_iroot(q << 128, 2) & ((1 << 64) - 1) for q in ps[:8]]
    return K, H


def curve_constants() -> List[int]:
    """d, 2d and sqrt(-1) as limbs (30 int32)."""
    return fe_limbs(D) + fe_limbs(D2) + fe_limbs(SQRT_M1)


def barrett_mu() -> int:
    """floor(2^512 / L) for the Barrett reduction of 512-bit hashes mod L."""
    return (1 << 512) // L


def scalars_ok(xs: Sequence[int]) -> bool:
    return all(0 <= x < L for x in xs)
