"""Host-side logic of the cuda backend, without a GPU: batch planning, the weight
repacking rules, the detokeniser and the backend registry."""

import json

import numpy as np
import pytest

from tinybark_b200 import backends, lengths
from tinybark_b200.engine import MIN_PART_SAMPLES, part_edges, plan_arrays, token_list
from tinybark_b200.text import Tokenizer


def test_plan_offsets_and_tiles():
    frames = [2, 100, 1000, 3, 257]
    p = plan_arrays(frames, 2, 32)
    t3 = [lengths.subsampled(f) for f in frames]
    assert p["t3"].tolist() == t3
    assert p["frame_off"].tolist() == [0, 2, 102, 1102, 1105, 1362]
    assert p["t3_off"][-1] == sum(t3)
    assert p["t3_clip"].tolist() == sum(([i] * n for i, n in enumerate(t3)), [])
    assert p["caps"].tolist() == [lengths.decode_cap(f) for f in frames]
    # Every attention row covered exactly once, longest clip first.
    att = p["attn_tiles"].reshape(-1, 2)
    assert att[0, 0] == int(np.argmax(t3))
    covered = {(c, r + k) for c, r in att for k in range(32) if r + k < t3[c]}
    assert covered == {(c, r) for c in range(len(frames)) for r in range(t3[c])}
    t2 = [lengths.subsampled(f, 2) for f in frames]
    sub = p["sub_tiles"].reshape(-1, 2)
    covered = {(c, r + k) for c, r in sub for k in range(2) if r + k < t2[c]}
    assert covered == {(c, r) for c in range(len(frames)) for r in range(t2[c])}


def test_upload_parts_are_never_shorter_than_the_minimum():
    """tokens_batch's upload parts: contiguous clip ranges covering the batch, cut near the
    fractions, none shorter than MIN_PART_SAMPLES unless the batch itself is (so a batch of
    more than 256 encoder rows never runs a part through the small-batch GEMMs whose K
    split makes the last bits vary between calls)."""
    rng = np.random.default_rng(3)
    fractions = (1 / 64, 1 / 16, 1 / 4, 1 / 2)
    for n, lo, hi in [(9, 0.5, 12.0), (40, 1.0, 30.0), (4096, 2.0, 30.0), (1, 5.0, 5.0), (3, 0.02, 60.0)]:
        sizes = (rng.uniform(lo, hi, n) * 16000).astype(np.int64)
        off = np.concatenate([[0], np.cumsum(sizes)])
        edges = part_edges(off, fractions)
        assert edges[0] == 0 and edges[-1] == n and all(a < b for a, b in zip(edges, edges[1:]))
        lens = [int(off[b] - off[a]) for a, b in zip(edges, edges[1:])]
        assert len(lens) == 1 or min(lens) >= MIN_PART_SAMPLES
    # The bench's set keeps every cut, each at the first clip boundary past its fraction.
    sizes = (rng.uniform(2.0, 30.0, 4096) * 16000).astype(np.int64)
    off = np.concatenate([[0], np.cumsum(sizes)])
    edges = part_edges(off, fractions)
    assert edges[1:-1] == np.searchsorted(off, [f * off[-1] for f in fractions]).tolist()
    # A batch of 56 s in all is one part.
    assert part_edges(np.array([0, 56 * 16000]), fractions) == [0, 1]


def test_token_lists_share_int_objects_and_equal_tolist():
    """Token rows become lists of the same Python ints as tolist() gives, taken from one
    shared table (no int created per token); the multi-GPU gather does the same for rows
    of token ids and converts anything else as it is."""
    from tinybark_b200 import dp

    rng = np.random.default_rng(1)
    row = rng.integers(0, 8193, 3700).astype(np.int32)
    got = token_list(row)
    assert got == row.tolist() and all(type(t) is int for t in got)
    assert got[0] is token_list(row[:1])[0]
    assert token_list(row[:0]) == []
    assert dp._id_list(row) == row.tolist()
    odd = np.array([5, -1, 9000], np.int64)
    assert dp._id_list(odd) == [5, -1, 9000] and dp._id_list(odd[:0]) == []


def test_plan_rejects_short_clips():
    with pytest.raises(ValueError):
        plan_arrays([5, 1], 2, 32)


def test_lstm_gate_interleave():
    """Row 4u+g of the repacked LSTM weight is gate g of unit u (PyTorch order i, f, g, o)."""
    w = np.arange(4 * 640 * 3, dtype=np.float32).reshape(4 * 640, 3)
    packed = w.reshape(4, 640, 3).transpose(1, 0, 2).reshape(4 * 640, 3)
    for u in (0, 5, 639):
        for g in range(4):
            np.testing.assert_array_equal(packed[4 * u + g], w[g * 640 + u])


def test_glu_pair_interleave():
    w = np.arange(2048 * 2, dtype=np.float32).reshape(2048, 2)
    packed = np.stack([w[:1024], w[1024:]], 1).reshape(2048, 2)
    for c in (0, 7, 1023):
        np.testing.assert_array_equal(packed[2 * c], w[c])
        np.testing.assert_array_equal(packed[2 * c + 1], w[1024 + c])


def test_subsampling_linear_permutation():
    """Linear input columns go from (channel, frequency) to (frequency, channel), so the
    kernels' [time][frequency][channel] activations multiply the same weights."""
    rng = np.random.default_rng(0)
    w = rng.standard_normal((8, 256 * 16)).astype(np.float32)
    x = rng.standard_normal((256, 16)).astype(np.float32)  # (channel, frequency)
    perm = w.reshape(8, 256, 16).transpose(0, 2, 1).reshape(8, -1)
    np.testing.assert_allclose(perm @ x.T.reshape(-1), w @ x.reshape(-1), rtol=1e-5, atol=1e-4)


def test_tokenizer_decodes_pieces_bytes_and_specials(tmp_path):
    spec = {
        "model": {"vocab": {"<unk>": 0, "▁Hel": 1, "lo": 2, "▁w": 3, "<0xC3>": 4, "<0xA9>": 5, "rld": 6}},
        "added_tokens": [{"id": 7, "content": "<|endoftext|>", "special": True}],
    }
    path = tmp_path / "tokenizer.json"
    path.write_text(json.dumps(spec))
    tok = Tokenizer(str(path))
    assert tok.decode([1, 2, 3, 4, 5, 6, 7]) == "Hello wérld"
    assert tok.decode([7]) == ""


def test_joined_piece_bytes_are_the_tokenizers_text(tmp_path):
    """The GPU's join, restated: every id's bytes from Tokenizer.table joined and finished
    once give Tokenizer.decode's text, over random id lists heavy in byte-fallback runs
    (invalid UTF-8 included) and special tokens between them."""
    import random

    from conftest import synthetic_tokenizer
    from tinybark_b200.text import finish

    tok = Tokenizer(synthetic_tokenizer(tmp_path / "tokenizer.json", vocab=600))
    off, data = tok.table()
    assert len(off) == 601 and off[0] == 0 and off[-1] == len(data)
    assert bytes(data[off[3 + 0xC3] : off[4 + 0xC3]]) == b"\xc3" and off[1] == off[0]  # a byte piece; a special
    rng = random.Random(1)
    for _ in range(20000):
        ids = []
        for _ in range(rng.randint(0, 12)):
            r = rng.random()
            ids.append(rng.randrange(3, 259) if r < 0.5 else (rng.choice([0, 1, 2, 599]) if r < 0.6 else rng.randrange(259, 599)))
        joined = b"".join(bytes(data[off[i] : off[i + 1]]) for i in ids)
        assert finish(joined) == tok.decode(ids), ids


def test_piece_table_refuses_what_the_join_cannot_match(tmp_path):
    """An empty ordinary piece or an id without a piece below the largest id: the GPU
    join would not equal decode (merged byte runs; no KeyError), so table() refuses."""
    for vocab in ({"a": 0, "": 1, "b": 2}, {"a": 0, "b": 2}):
        path = tmp_path / "tokenizer.json"
        path.write_text(json.dumps({"model": {"vocab": vocab}, "added_tokens": []}))
        with pytest.raises(ValueError):
            Tokenizer(str(path)).table()


def test_detokeniser_matches_reference_tokenizer(tmp_path):
    """tinybark.text.Tokenizer.decode's texts (tests/golden/text.json) on 300 seeded id
    lists under the seeded 8193-id tokenizer: this module's decode, and the GPU join
    restated (the piece table's bytes joined, then finish), give the same texts."""
    from conftest import golden_json, synthetic_tokenizer
    from golden.make_golden import text_cases
    from tinybark_b200.text import finish

    want = golden_json("text.json")["texts"]
    tok = Tokenizer(synthetic_tokenizer(tmp_path / "tokenizer.json"))
    off, data = tok.table()
    cases = text_cases()
    assert len(cases) == len(want)
    for ids, text in zip(cases, want):
        assert tok.decode(ids) == text
        assert finish(b"".join(bytes(data[off[i] : off[i + 1]]) for i in ids)) == text


def test_cache_file_is_the_references(tmp_path):
    """convert + save of the 2-layer synthetic weights write the same bytes, tensor order
    and header included, as tinybark's _convert + _save (tests/golden/cache_file.json)."""
    import hashlib

    from conftest import golden_json, state_dict
    from tinybark_b200 import synthetic, weights

    want = golden_json("cache_file.json")
    conv = weights.convert(state_dict(2), synthetic.config(2))
    assert list(conv) == want["order"]
    path = tmp_path / "bark.safetensors"
    weights.save(conv, path)
    assert hashlib.sha256(path.read_bytes()).hexdigest() == want["sha256"]


def test_registry_has_cuda_backend():
    b = backends.BACKENDS["cuda"]
    assert b.name == "cuda" and set(b.descriptions) <= set(backends.DEVICES)
    assert "gpu" in b.descriptions and b.env("gpu") == {}


def test_public_entry_points_take_the_ffn_option():
    import inspect

    import tinybark_b200
    from tinybark_b200.engine import Engine

    for fn in (tinybark_b200.load, tinybark_b200.Bark.__init__, Engine.__init__):
        assert inspect.signature(fn).parameters["ffn"].default == "bf16"


def test_cpu_device_is_refused():
    import tinybark_b200

    with pytest.raises(RuntimeError):
        tinybark_b200.Bark("cpu", weights=({}, {}))


def _csource_constant(name: str) -> int:
    import re

    from conftest import ROOT

    text = (ROOT / "tinybark_b200" / "csrc" / "common.cuh").read_text()
    return int(re.search(rf"constexpr int {name} = (0x[0-9A-Fa-f]+);", text).group(1), 16)


def test_reciprocal_seed_is_minimax_and_newton_bound():
    """rcp_newton's seed constant minimises max |1 - y r0| over every float mantissa (its
    neighbours do worse), and the seed refined by two Newton steps, restated in float32
    with numpy, is within 8e-6 of 1/y for every mantissa at several exponents."""
    seed = _csource_constant("RCP_SEED")
    m = np.arange(1 << 23, dtype=np.int64)
    bits = (127 << 23) | m
    y = bits.astype(np.uint32).view(np.float32)

    def worst(c):
        r0 = (np.int64(c) - bits).astype(np.uint32).view(np.float32).astype(np.float64)
        return np.abs(1 - y.astype(np.float64) * r0).max()

    e = worst(seed)
    assert e < 0.0506 and e <= worst(seed - 1) and e <= worst(seed + 1)
    for shift in (0, 5, 40, 110):
        yb = bits + (shift << 23)
        ys = yb.astype(np.uint32).view(np.float32)
        r = (np.int64(seed) - yb).astype(np.uint32).view(np.float32)
        two = np.float32(2)
        for _ in range(2):
            r = r * (two - ys * r)
        rel = np.abs(r.astype(np.float64) * ys.astype(np.float64) - 1)
        assert rel.max() < 8e-6, shift
