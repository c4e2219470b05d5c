"""Token ids to text, as the Parakeet tokenizer decodes them with skip_special_tokens=True:
SentencePiece pieces joined, "▁" read as a space, byte-fallback pieces "<0xNN>" collected
and decoded as UTF-8, special tokens skipped (tinybark/text.py:1-34). Host-side: it runs
once per transcript on a few dozen ids."""

from __future__ import annotations

import json
import re

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
