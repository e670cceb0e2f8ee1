"""BLAKE3 modes, batch commitments and Merkle roots on the CPU, against the
independent ``blake3`` package."""
import os

import pytest

blake3 = pytest.importorskip("blake3")

from arc_chain_b200.crypto import commit

CTX = commit.TX_CONTEXT
LENS = [0, 1, 3, 4, 63, 64, 65, 127, 1023, 1024, 1025, 2048, 3071, 5000, 70001]


def _ref_commit(data: bytes, domain=None) -> bytes:
    h = blake3.blake3(derive_key_context=CTX)
    if domain is not None:
        h.update(bytes([domain]))
    h.update(data)
    return h.digest()


def _ref_merkle(leaves):
    if not leaves:
        return bytes(32)
    cur = list(leaves)
    if len(cur) == 1:
        return cur[0]
    if len(cur) % 2:
        cur.append(bytes(32))
    while len(cur) > 1:
        cur = [_ref_commit(cur[i] + cur[i + 1]) for i in range(0, len(cur), 2)]
        if len(cur) > 1 and len(cur) % 2:
            cur.append(bytes(32))
    return cur[0]


@pytest.mark.parametrize("n", LENS)
def test_derive_and_keyed_modes(n):
    data = os.urandom(n)
    assert commit.derive_key(CTX, data) == blake3.blake3(data, derive_key_context=CTX).digest()
    key = bytes(range(32))
    assert commit.keyed_hash(key, data) == blake3.blake3(data, key=key).digest()


def test_batch_commit_with_and_without_domain():
    items = [os.urandom(n) for n in LENS * 3]
    doms = [i % 256 for i in range(len(items))]
    assert commit.batch_commit_cpu(items) == [_ref_commit(x) for x in items]
    assert commit.batch_commit_cpu(items, doms) == [_ref_commit(x, d) for x, d in zip(items, doms)]


@pytest.mark.parametrize("n", [0, 1, 2, 3, 4, 5, 7, 8, 33, 100])
def test_merkle_root(n):
    leaves = [blake3.blake3(i.to_bytes(4, "little")).digest() for i in range(n)]
    assert commit.merkle_root_cpu(leaves) == _ref_merkle(leaves)
