"""Token ids to text, as the Parakeet tokenizer decodes them with skip_special_tokens=True:
SentencePiece pieces joined, "▁" read as a space, byte-fallback pieces "<0xNN>" collected
and decoded as UTF-8, special tokens skipped (tinybark/text.py:1-34).

`Tokenizer.decode` does it on the host for one list of ids. For a batch the GPU joins each
lane's bytes from the piece table of `Tokenizer.table` (tb_text_offsets / tb_text_bytes)
and `finish` turns a lane's bytes into its text: decoding the joined bytes once equals
decoding each run of byte pieces on its own, because a run always ends at a whole piece,
whose first byte closes any sequence the run left open."""

from __future__ import annotations

import json
import re

import numpy as np

_BYTE = re.compile(r"<0x([0-9A-Fa-f]{2})>")


class Tokenizer:
    def __init__(self, path: str):
        with open(path) as f:
            spec = json.load(f)
        self.pieces = {i: p for p, i in spec["model"]["vocab"].items()}
        self.special = set()
        for tok in spec.get("added_tokens", []):
            self.pieces[tok["id"]] = tok["content"]
            if tok.get("special"):
                self.special.add(tok["id"])

    def decode(self, ids: list[int]) -> str:
        parts: list[str] = []
        raw = bytearray()
        for i in ids:
            if i in self.special:
                continue
            piece = self.pieces[i]
            m = _BYTE.fullmatch(piece)
            if m:
                raw.append(int(m.group(1), 16))
                continue
            if raw:
                parts.append(raw.decode("utf-8", "replace"))
                raw.clear()
            parts.append(piece)
        if raw:
            parts.append(raw.decode("utf-8", "replace"))
        return "".join(parts).replace("▁", " ").strip()

    def table(self) -> tuple[np.ndarray, np.ndarray]:
        """The piece table of the GPU join: offsets [vocab + 1] (int32) into the bytes
        (uint8) of every id, vocab = the largest id + 1. A special token has no bytes, a
        byte-fallback piece is its byte, any other piece is its UTF-8 with "▁" as a space.

        The join equals `decode` only if no other piece is empty (an empty piece between
        two byte runs would merge them into one UTF-8 sequence) and every id below vocab has
        a piece (decode raises KeyError on one without; the GPU join cannot tell it from a
        special token): a tokenizer breaking either rule raises ValueError here. Ids at or
        above vocab are flagged by the GPU join (TB_DEV_TEXT_TOKEN)."""
        vocab = max(self.pieces) + 1
        missing = [i for i in range(vocab) if i not in self.pieces]
        if missing:
            raise ValueError(f"tokenizer has no piece for ids {missing[:8]}: the GPU join needs one for every id")
        parts = []
        for i in range(vocab):
            piece = self.pieces[i]
            if i in self.special:
                parts.append(b"")
            elif piece == "":
                raise ValueError(f"tokenizer piece {i} is empty: the GPU join needs non-empty pieces")
            elif m := _BYTE.fullmatch(piece):
                parts.append(bytes([int(m.group(1), 16)]))
            else:
                parts.append(piece.replace("▁", " ").encode("utf-8"))
        off = np.zeros(vocab + 1, np.int32)
        off[1:] = np.cumsum([len(b) for b in parts])
        return off, np.frombuffer(b"".join(parts), np.uint8).copy()


def finish(raw: bytes) -> str:
    """A lane's joined piece bytes as text: UTF-8 (invalid sequences replaced), "▁" from
    byte pieces as a space, the ends stripped (tinybark/text.py:29-34)."""
    return raw.decode("utf-8", "replace").replace("▁", " ").strip()
