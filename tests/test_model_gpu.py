"""The whole path on the GPU against the oracle: encoder outputs within max-rel 1e-4
(fp32) and 2e-2 (bf16), greedy TDT tokens identical in fp32 on the reference loop's
golden cases, and end-to-end transcription tokens identical to the oracle pipeline."""

import numpy as np
import pytest
import torch

from conftest import golden_json, max_rel, state_dict

pytestmark = pytest.mark.gpu


def make_engine(layers, dtype, sd=None):
    from tinybark_b200 import synthetic, weights
    from tinybark_b200.engine import Engine

    sd = state_dict(layers) if sd is None else sd
    return Engine(weights.convert(sd, synthetic.config(layers)), synthetic.config(layers), dtype=dtype)


def oracle_encode(layers, clip):
    from oracle import encoder, frontend

    return encoder.encode(state_dict(layers), frontend.features(clip), hidden=True)


def gpu_encode(eng, clips):
    plan = eng.plan([len(c) // 160 for c in clips])
    samples, off = eng.upload(clips)
    enc = eng.encode(eng.features(samples, off, plan), plan)
    eng.check()
    o = plan.t3_off.cpu().numpy()
    e = enc.cpu().numpy()
    return [e[o[i] : o[i + 1]] for i in range(len(clips))]


def clips_of(seconds, seed=50):
    from tinybark_b200 import synthetic

    return [synthetic.to_float(synthetic.clip(s, seed + i)) for i, s in enumerate(seconds)]


@pytest.mark.parametrize("dtype,tol", [("fp32", 1e-4), ("bf16", 2e-2)])
def test_encoder_two_layers_packed_batch(dtype, tol):
    eng = make_engine(2, dtype)
    clips = clips_of((0.5, 1.0, 3.33, 0.02))
    got = gpu_encode(eng, clips)
    for c, g in zip(clips, got):
        ref, _ = oracle_encode(2, c)
        assert g.shape == ref.shape
        assert max_rel(g, ref) < tol


@pytest.mark.parametrize("dtype,tol", [("fp32", 1e-4), ("bf16", 2e-2)])
def test_encoder_24_layers_10s(dtype, tol):
    from tinybark_b200 import synthetic

    eng = make_engine(24, dtype)
    clip = synthetic.to_float(synthetic.clip(10.0, 0))
    (got,) = gpu_encode(eng, [clip])
    ref, _ = oracle_encode(24, clip)
    assert got.shape == (125, 640)
    err = max_rel(got, ref)
    print(f"encoder 24 layers {dtype}: max-rel {err:.2e}")
    assert err < tol


def run_decode(eng, frames_list, feature_frames, groups=None):
    plan = eng.plan(feature_frames)
    enc = torch.from_numpy(np.concatenate(frames_list)).cuda()
    tokens, counts = eng.decode(enc, plan, groups=groups)
    eng.check()
    t, c = tokens.cpu().numpy(), counts.cpu().numpy()
    return [t[i, : c[i]].tolist() for i in range(len(frames_list))]


@pytest.mark.parametrize("case", ["mixed", "eos", "cap", "single"])
def test_decode_matches_reference_loop(case):
    from golden.make_golden import decode_frames, decode_weights

    g = golden_json("decode.json")[case]
    eng = make_engine(2, "fp32", decode_weights(g["case"]))
    (tokens,) = run_decode(eng, [decode_frames(g["case"])], [g["case"]["feature_frames"]])
    assert tokens == g["tokens"]


@pytest.mark.parametrize("groups", [1, 2, 4])
def test_decode_lanes_are_independent(groups):
    """The four golden cases' encoder frames as four lanes of one batch, under the
    'mixed' weights, each equal to the oracle's single-clip loop, with the lanes
    decoded as 1, 2 or 4 concurrent groups."""
    from golden.make_golden import DECODE_CASES, decode_frames, decode_weights
    from oracle import decoder

    sd = decode_weights(DECODE_CASES["mixed"])
    eng = make_engine(2, "fp32", sd)
    cases = list(DECODE_CASES.values())
    frames = [decode_frames(c) for c in cases]
    ff = [c["feature_frames"] for c in cases]
    got = run_decode(eng, frames, ff, groups)
    dec = decoder.Decoder(sd)
    for fr, f, g in zip(frames, ff, got):
        assert g == dec.greedy(fr, f)


@pytest.mark.parametrize("lanes", [300, 1000])
def test_decode_bf16_persistent_matches_graph_decoder(lanes):
    """bf16, lanes of seeded encoder frames with lengths 1..60 (lanes finishing at
    different iterations): the persistent decoder (one kernel, grid barriers) and the
    graph-replayed one (one kernel per GEMM) compute the same products and epilogues;
    only fp32 summation orders differ (the persistent kernel takes layer 0 as
    E[token] + W_hh0.h0, and at 300 lanes layer 1's h1 half one phase ahead of its h0
    half; at 1000 lanes layer 1's tiles outnumber the SMs and it runs unsplit), and
    every lane's tokens come out identical."""
    from golden.make_golden import DECODE_CASES, decode_weights

    sd = decode_weights(DECODE_CASES["mixed"])
    eng = make_engine(2, "bf16", sd)
    rng = np.random.default_rng(7)
    t3 = rng.integers(1, 61, lanes)
    t3[:5] = 60  # longest first, as the engine orders a batch
    t3 = np.sort(t3)[::-1]
    feature_frames = [int(8 * t - 4) for t in t3]  # 8x subsampling: feature frames giving t3 frames
    frames = [rng.standard_normal((int(t), 640)).astype(np.float32) for t in t3]
    plan = eng.plan(feature_frames)
    assert list(plan.t3) == list(t3)
    enc = torch.from_numpy(np.concatenate(frames)).cuda()
    results = []
    for groups in (0, 1):
        tokens, counts = eng.decode(enc, plan, groups=groups)
        eng.check()
        t, c = tokens.cpu().numpy(), counts.cpu().numpy()
        results.append([t[i, : c[i]].tolist() for i in range(len(frames))])
    assert sum(len(r) for r in results[0]) > 0
    assert results[0] == results[1]


def test_end_to_end_fp32_tokens_match_oracle():
    import tinybark_b200
    from oracle import decoder
    from tinybark_b200 import synthetic, weights

    sd = state_dict(24)
    bark = tinybark_b200.load("gpu", dtype="fp32", weights=(weights.convert(sd, synthetic.config(24)), synthetic.config(24)))
    clip = synthetic.to_float(synthetic.clip(10.0, 0))
    got = bark.tokens(clip)
    enc, _ = oracle_encode(24, clip)
    ref = decoder.Decoder(sd).greedy(enc, len(clip) // 160)
    assert got == ref
    assert bark.tokens(np.zeros(100, np.float32)) == []  # fewer than 2 frames
    batch = bark.tokens_batch([clip[:16000], clip, np.zeros(10, np.float32)])
    assert batch[1] == got and batch[2] == [] and batch[0] == bark.tokens(clip[:16000])


def test_end_to_end_bf16_batch_consistent():
    import tinybark_b200
    from tinybark_b200 import synthetic, weights

    sd = state_dict(24)
    bark = tinybark_b200.load("gpu", weights=(weights.convert(sd, synthetic.config(24)), synthetic.config(24)))
    clips = clips_of((2.0, 10.0, 5.5), seed=60)
    batch = bark.tokens_batch(clips)
    for c, b in zip(clips, batch):
        assert bark.tokens(c) == b
        assert len(b) > 0


def test_batch_encoder_gives_the_same_bits_on_every_call():
    """A batch of 9 clips (0.5-12 s, about 700 encoder rows) is encoded as one part, never
    as a first part of a few clips whose residual GEMMs would split K and add the ranges
    atomically: two calls give the same encoder rows bit for bit, and the same tokens."""
    import tinybark_b200
    from tinybark_b200 import synthetic, weights

    rng = np.random.default_rng(12)
    clips = [synthetic.clip(float(s), 400 + i) for i, s in enumerate(rng.uniform(0.5, 12.0, 9))]
    bark = tinybark_b200.load("gpu", weights=(weights.convert(state_dict(2), synthetic.config(2)), synthetic.config(2)))
    runs = []
    for _ in range(2):
        keep, enc, plan = bark.engine._encode_batch(clips)
        runs.append((enc.clone(), bark.tokens_batch(clips)))
    assert plan.batch.t3_total > 256
    assert torch.equal(runs[0][0], runs[1][0]) and runs[0][1] == runs[1][1]


def test_tokens_batch_parts_match_whole_batch_path():
    """bf16, 40 clips of 1-30 s: tokens_batch uploads and encodes the batch in parts (the
    copy of each part overlapping the previous part's encoder) and turns finished lanes
    into lists while the persistent decoder still runs; every list equals that of the
    plain path (one upload, one encoder call over the whole batch, decode, then lists)."""
    import tinybark_b200
    from tinybark_b200 import lengths, synthetic, weights
    from tinybark_b200.engine import lane_order

    sd = state_dict(2)
    bark = tinybark_b200.load("gpu", weights=(weights.convert(sd, synthetic.config(2)), synthetic.config(2)))
    eng = bark.engine
    rng = np.random.default_rng(11)
    clips = clips_of(tuple(float(x) for x in rng.uniform(1.0, 30.0, 40)), seed=90)
    got = bark.tokens_batch(clips)
    frames = [lengths.frames(len(c)) for c in clips]
    keep = lane_order(list(range(len(clips))), frames)
    plan = eng.plan([frames[i] for i in keep])
    s, o = eng.upload([np.asarray(clips[i], np.float32) for i in keep])
    tokens, counts = eng.decode(eng.encode(eng.features(s, o, plan), plan), plan)
    eng.check()
    tk, cn = tokens.cpu().numpy(), counts.cpu().numpy()
    want = [[] for _ in clips]
    for j, i in enumerate(keep):
        want[i] = tk[j, : cn[j]].tolist()
    assert sum(len(w) for w in want) > 0
    assert got == want


def test_tokens_long_is_the_pieces_transcribed_together():
    """A 70 s recording through Bark.tokens_long: its pieces (cut at quiet points, at most
    30 s each) decoded as one batch give the same tokens as each piece through Bark.tokens
    alone, joined; a 10 s recording is one piece and equals Bark.tokens."""
    import tinybark_b200
    from tinybark_b200 import longform, synthetic, weights

    sd = state_dict(2)
    bark = tinybark_b200.load("gpu", weights=(weights.convert(sd, synthetic.config(2)), synthetic.config(2)))
    long = synthetic.to_float(synthetic.clip(70.0, 5, segment=2.0))
    cuts = longform.cut_points(long)
    assert len(cuts) == 4
    pieces = [bark.tokens(long[a:b]) for a, b in zip(cuts[:-1], cuts[1:])]
    got = bark.tokens_long(long)
    assert got == longform.join(pieces) and len(got) > 0
    short = long[: 10 * 16000]
    assert bark.tokens_long(short) == bark.tokens(short)


def test_pcm16_ingest_matches_float_path():
    """int16 PCM goes to the GPU as 16-bit and is converted there (pcm / 32768): the same
    features, bit for bit, and the same tokens as the float32 path of the same audio."""
    import tinybark_b200
    from tinybark_b200 import lengths, synthetic, weights

    sd = state_dict(2)
    bark = tinybark_b200.load("gpu", weights=(weights.convert(sd, synthetic.config(2)), synthetic.config(2)))
    eng = bark.engine
    pcm = [synthetic.clip(s, 70 + i) for i, s in enumerate((3.0, 7.5, 1.2))]
    flt = [synthetic.to_float(p) for p in pcm]
    plan = eng.plan([lengths.frames(len(p)) for p in pcm])
    feats = []
    for clips in (pcm, flt):
        s, o = eng.upload(clips)
        assert s.dtype == (torch.int16 if clips is pcm else torch.float32)
        feats.append(eng.features(s, o, plan).cpu())
    assert torch.equal(feats[0], feats[1])
    assert bark.tokens_batch(pcm) == bark.tokens_batch(flt)


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_engine_from_cache_file_equals_engine_from_arrays(tmp_path, dtype):
    """2 layers written as tinybark's fp16 cache file: the engine that uploads the file's
    data block as is and repacks it on the GPU holds, byte for byte, the packed weights of
    the engine built from the same tensors as float32 arrays, and both equal the packed
    layout's numpy restatement; transcription through tinybark_b200.load on the file gives
    the same tokens."""
    import tinybark_b200
    from conftest import repack_numpy
    from tinybark_b200 import pack, synthetic, weights
    from tinybark_b200.engine import Engine

    cfg = synthetic.config(2)
    path = tmp_path / "bark.safetensors"
    weights.save(weights.convert(state_dict(2), cfg), path)
    a = Engine(path, cfg, dtype=dtype)
    arrays = weights.load(path)
    b = Engine(arrays, cfg, dtype=dtype)
    assert a.layout.regions == b.layout.regions
    assert torch.equal(a._blob, b._blob)
    offset, _, index = pack.cache_index(path)
    body = np.fromfile(path, np.uint8)[offset:]
    pieces, dev_bytes, _ = pack.aligned_runs(index)
    image = np.zeros(dev_bytes, np.uint8)  # the data block as placed in device memory
    for start, end, dev in pieces:
        image[dev : dev + end - start] = body[start:end]
    assert np.array_equal(a._blob.cpu().numpy(), repack_numpy(a.layout.jobs, image, a.layout.size))
    clips = clips_of((3.0, 7.0), seed=80)
    got = tinybark_b200.load("gpu", dtype=dtype, weights=(path, cfg)).tokens_batch(clips)
    assert got == tinybark_b200.load("gpu", dtype=dtype, weights=(arrays, cfg)).tokens_batch(clips)


def test_transcribe_batch_is_the_tokenizers_text(tmp_path):
    """transcribe_batch joins every clip's piece bytes on the GPU: its texts equal the
    tokenizer's host decode of the same clips' tokens (a seeded tokenizer of 8193 ids with
    byte-fallback pieces, since the real vocabulary is not available offline); a clip too
    short for any frame gives ""."""
    import tinybark_b200
    from conftest import synthetic_tokenizer
    from tinybark_b200 import synthetic, weights
    from tinybark_b200.text import Tokenizer

    cfg = synthetic.config(2)
    path = synthetic_tokenizer(tmp_path / "tokenizer.json")
    bark = tinybark_b200.load("gpu", weights=(weights.convert(state_dict(2), cfg), cfg), tokenizer=path)
    clips = clips_of((1.0, 4.0, 9.5, 0.005, 2.2), seed=30)
    tokens = bark.tokens_batch(clips)
    assert sum(len(t) for t in tokens) > 0 and tokens[3] == []
    tok = Tokenizer(path)
    texts = bark.transcribe_batch(clips)
    assert texts == [tok.decode(t) for t in tokens] and texts[3] == ""
    assert bark.transcribe(clips[2]) == texts[2]


def test_gpu_text_join_is_the_reference_detokeniser(tmp_path):
    """The GPU join (tb_text_offsets / tb_text_bytes, then text.finish) on 300 seeded id
    lists gives tinybark.text.Tokenizer.decode's texts (tests/golden/text.json, made by
    the reference itself under the seeded 8193-id tokenizer)."""
    from conftest import golden_json, synthetic_tokenizer
    from golden.make_golden import text_cases
    from tinybark_b200.text import Tokenizer, finish

    want = golden_json("text.json")["texts"]
    cases = text_cases()
    eng = make_engine(2, "bf16")
    table = eng.text_table(*Tokenizer(synthetic_tokenizer(tmp_path / "tokenizer.json")).table())
    ld = max(len(c) for c in cases)
    rows = np.zeros((len(cases), ld), np.int32)
    for i, c in enumerate(cases):
        rows[i, : len(c)] = c
    counts = np.array([len(c) for c in cases], np.int32)
    raw = eng.texts(torch.from_numpy(rows).cuda(), torch.from_numpy(counts).cuda(), table)
    assert [finish(r) for r in raw] == want


def test_tokens_long_matches_oracle_piece_by_piece():
    """fp32, a 40 s recording through Bark.tokens_long: the oracle pipeline (front-end,
    encoder, greedy loop) run on each piece at the same cut points, joined, gives the
    same tokens."""
    import tinybark_b200
    from oracle import decoder, frontend
    from oracle import encoder as oenc
    from tinybark_b200 import longform, synthetic, weights

    sd = state_dict(2)
    bark = tinybark_b200.load("gpu", dtype="fp32", weights=(weights.convert(sd, synthetic.config(2)), synthetic.config(2)))
    long = synthetic.to_float(synthetic.clip(40.0, 6, segment=2.0))
    cuts = longform.cut_points(long)
    assert len(cuts) >= 3
    dec = decoder.Decoder(sd)
    pieces = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        feats = frontend.features(long[a:b])
        pieces.append(dec.greedy(oenc.encode(sd, feats), len(feats)) if len(feats) >= 2 else [])
    got = bark.tokens_long(long)
    assert got == longform.join(pieces) and len(got) > 0
