"""Greedy longest-match tokenizer over the vocab stored in ARC-INT8 files
(``CachedIntegerModel::encode/decode``, crates/arc-inference/src/
cached_integer_model.rs:1331-1374).

encode: the text becomes "▁" + text with spaces replaced by "▁"; at each byte
position the longest vocab entry (up to 32 bytes, valid UTF-8) wins; an
unmatched byte becomes its "<0xNN>" token when the vocab has one, otherwise
it is dropped.  decode: ids map to their strings with "▁" -> " ", ids
outside the vocab to "[id]".
"""
from __future__ import annotations

from typing import Dict, List, Sequence


class Tokenizer:
    def __init__(self, vocab: Sequence[str]):
        self.vocab = list(vocab)
        # first occurrence wins, as a linear position() search does
        self.index: Dict[bytes, int] = {}
        for i, s in enumerate(self.vocab):
            self.index.setdefault(s.encode(), i)

    def encode(self, text: str) -> List[int]:
        if not self.vocab:
            return []
        b = ("▁" + text.replace(" ", "▁")).encode()
        out, pos = [], 0
        while pos < len(b):
            best = None
            for n in range(min(32, len(b) - pos), 0, -1):
                piece = b[pos:pos + n]
                try:
                    piece.decode()
                except UnicodeDecodeError:
                    continue
                i = self.index.get(piece)
                if i is not None:
                    best = (n, i)
                    break
            if best is not None:
                out.append(best[1])
                pos += best[0]
            else:
                i = self.index.get(f"<0x{b[pos]:02X}>".encode())
                if i is not None:
                    out.append(i)
                pos += 1
        return out

    def decode(self, ids: Sequence[int]) -> str:
        return "".join(self.vocab[i].replace("▁", " ") if 0 <= i < len(self.vocab) else f"[{i}]"
                       for i in map(int, ids))
