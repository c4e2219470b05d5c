"""The packed weight layout on the CPU: the tb_repack jobs of pack.model_layout, run by
their numpy restatement, give every region the kernels read exactly as written out
here tensor by tensor (the layouts of the kernels' weight operands); the fp16 cache
file gives the same bytes as its tensors read as float32 arrays; tb_repack refuses bad
jobs before any device work."""

import ctypes as C

import numpy as np
import pytest
import torch

from conftest import repack_numpy, state_dict

H, CH, P, K = 1024, 256, 640, 9


def expected(w: dict, layers: int, bf16: bool) -> dict:
    """Every region as the kernels read it, from the converted tensors."""
    p = "encoder.subsampling."
    e = {"sub0_w": w[p + "layers.0.weight"].reshape(CH, 9), "sub0_b": w[p + "layers.0.bias"]}
    for i, (dw, pw) in enumerate(((2, 3), (5, 6))):
        e[f"sub_dw_w{i}"] = w[p + f"layers.{dw}.weight"].reshape(CH, 9)
        e[f"sub_dw_b{i}"] = w[p + f"layers.{dw}.bias"]
        e[f"sub_pw_w{i}"] = w[p + f"layers.{pw}.weight"].reshape(CH, CH)
        e[f"sub_pw_b{i}"] = w[p + f"layers.{pw}.bias"]
    e["sub_linear_w"] = w[p + "linear.weight"].reshape(H, CH, 16).transpose(0, 2, 1).reshape(H, -1)
    e["sub_linear_b"] = w[p + "linear.bias"]
    norms = ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out")
    for i in range(layers):
        q = f"encoder.layers.{i}."
        for j, n in enumerate(norms):
            e[f"{i}.norm_w{j}"], e[f"{i}.norm_b{j}"] = w[q + n + ".weight"], w[q + n + ".bias"]
        for f in (1, 2):
            e[f"{i}.ff{f}_w1"] = w[q + f"feed_forward{f}.linear1.weight"]
            e[f"{i}.ff{f}_w2"] = w[q + f"feed_forward{f}.linear2.weight"]
        a = q + "self_attn."
        e[f"{i}.qkv"], e[f"{i}.o_proj"] = w[a + "qkv"], w[a + "o_proj.weight"]
        e[f"{i}.bias_u"], e[f"{i}.bias_v"] = w[a + "bias_u"].reshape(-1), w[a + "bias_v"].reshape(-1)
        e[f"{i}.rel_w"] = w[a + "relative_k_proj.weight"]
        c = q + "conv."
        pw1 = w[c + "pointwise_conv1.weight"].reshape(2 * H, H)
        e[f"{i}.pw1"] = np.stack([pw1[:H], pw1[H:]], 1).reshape(2 * H, H)
        e[f"{i}.pw2"] = w[c + "pointwise_conv2.weight"].reshape(H, H)
        e[f"{i}.dw_w"], e[f"{i}.dw_b"] = w[c + "depthwise.weight"].reshape(H, K), w[c + "depthwise.bias"]
    e["enc_proj_w"], e["enc_proj_b"] = w["encoder_projector.weight"], w["encoder_projector.bias"]
    e["embedding"] = w["decoder.embedding.weight"]
    for l in range(2):
        wl = w[f"decoder.lstm.weight_l{l}"].reshape(4, P, 2 * P).transpose(1, 0, 2).reshape(4 * P, -1)
        e[f"lstm_w{l}"] = wl
        e[f"lstm_b{l}"] = w[f"decoder.lstm.bias_l{l}"].reshape(4, P).T.reshape(-1)
        if l == 0 and bf16:
            e["lstm0_hh"], e["lstm0_ih"] = wl[:, P:], wl[:, :P]
    e["dec_proj_w"] = w["decoder.decoder_projector.weight"]
    e["dec_proj_b"] = w["decoder.decoder_projector.bias"]
    joint = np.zeros((8448, P), np.float32)
    bias = np.full(8448, -np.inf, np.float32)
    joint[:8256], bias[:8256] = w["joint.token_head.weight"], w["joint.token_head.bias"]
    joint[8256:8261], bias[8256:8261] = w["joint.duration_head.weight"], w["joint.duration_head.bias"]
    e["joint_w"], e["joint_b"] = joint, bias
    return e


def region_bytes(lay, out: np.ndarray, key: str) -> np.ndarray:
    from math import prod

    r = lay.regions[key]
    n = prod(r.shape) * (2 if r.type == 1 else 4)
    return out[r.off : r.off + n]


def as_bytes(a: np.ndarray, bf16: bool) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32).reshape(-1)
    if bf16:
        return torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint8)
    return a.view(np.uint8)


@pytest.fixture(scope="module")
def converted2():
    from tinybark_b200 import synthetic, weights

    return weights.convert(state_dict(2), synthetic.config(2))


MATRICES = ("sub_pw_w", "sub_linear_w", "ff1_w", "ff2_w", "qkv", "o_proj", "rel_w", "pw1", "pw2", "enc_proj_w",
            "embedding", "lstm_w", "lstm0_", "dec_proj_w", "joint_w")


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_layout_regions_are_the_kernels_layouts(converted2, dtype):
    from tinybark_b200 import _lib as L
    from tinybark_b200 import pack

    bf16 = dtype == "bf16"
    source, index = pack.upload_arrays(converted2, "cpu")
    lay = pack.model_layout(index, 2, L.BF16 if bf16 else L.F32)
    out = repack_numpy(lay.jobs, source.numpy(), lay.size)
    want = expected(converted2, 2, bf16)
    assert set(want) == set(lay.regions)
    offs = sorted((r.off, k) for k, r in lay.regions.items())
    for (o, k), (o2, _) in zip(offs, offs[1:]):
        assert o % 256 == 0 and o + len(region_bytes(lay, out, k)) <= o2  # aligned, disjoint
    for k, a in want.items():
        mat = any(s in k for s in MATRICES)
        assert lay.regions[k].type == (L.BF16 if bf16 and mat else L.F32), k
        assert lay.regions[k].shape[0] * int(np.prod(lay.regions[k].shape[1:])) == a.size, k
        assert np.array_equal(region_bytes(lay, out, k), as_bytes(a, bf16 and mat)), k


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_fp16_cache_file_gives_the_same_bytes(converted2, tmp_path, dtype):
    """The cache file (tinybark's format: fp16 safetensors) indexed in place gives the same
    packed bytes as its tensors read back as float32 arrays."""
    from tinybark_b200 import _lib as L
    from tinybark_b200 import pack, weights

    path = tmp_path / "bark.safetensors"
    weights.save(converted2, path)
    offset, nbytes, index = pack.cache_index(path)
    body = np.fromfile(path, np.uint8)[offset:]
    assert len(body) == nbytes
    assert all(s.type == L.SRC_F16 for s in index.values())
    t = L.BF16 if dtype == "bf16" else L.F32
    lay = pack.model_layout(index, 2, t)
    got = repack_numpy(lay.jobs, body, lay.size)
    src2, index2 = pack.upload_arrays(weights.load(path), "cpu")
    lay2 = pack.model_layout(index2, 2, t)
    assert lay2.regions == lay.regions
    assert np.array_equal(got, repack_numpy(lay2.jobs, src2.numpy(), lay2.size))


def test_aligned_runs_put_every_tensor_on_a_16_byte_boundary(converted2, tmp_path):
    """The cache file's tensors placed in device memory run by run: every tensor starts
    16-byte aligned with its bytes unchanged, runs do not overlap, and the packed bytes
    from the placed block equal those from the file's block as it is."""
    from tinybark_b200 import _lib as L
    from tinybark_b200 import pack, weights

    path = tmp_path / "bark.safetensors"
    weights.save(converted2, path)
    offset, nbytes, index = pack.cache_index(path)
    body = np.fromfile(path, np.uint8)[offset:]
    assert any(s.off % 16 for s in index.values())  # the duration bias moves what follows it
    pieces, dev_bytes, moved = pack.aligned_runs(index)
    image = np.zeros(dev_bytes, np.uint8)
    for (a, b, d), (a2, _, d2) in zip(pieces, pieces[1:] + [(None, None, dev_bytes)]):
        assert d + (b - a) <= d2
        image[d : d + b - a] = body[a:b]
    for name, s in index.items():
        m, n = moved[name], int(np.prod(s.shape)) * 2
        assert m.off % 16 == 0 and m.shape == s.shape and m.type == s.type
        assert np.array_equal(image[m.off : m.off + n], body[s.off : s.off + n]), name
    lay, lay2 = pack.model_layout(index, 2, L.BF16), pack.model_layout(moved, 2, L.BF16)
    assert np.array_equal(repack_numpy(lay.jobs, body, lay.size), repack_numpy(lay2.jobs, image, lay2.size))


@pytest.mark.parametrize("seed", range(5))
def test_slice_copies_place_every_byte_once(seed):
    """upload_file's copies, slice by slice: for random runs (gaps between them, runs
    straddling slice boundaries) and slice sizes, every byte of every run arrives once at
    its device offset and nothing else is written."""
    from tinybark_b200 import pack

    rng = np.random.default_rng(seed)
    pieces, at, dev = [], 0, 0
    for _ in range(int(rng.integers(1, 8))):
        at += int(rng.integers(0, 40))
        n = int(rng.integers(1, 300))
        dev += int(rng.integers(0, 16))
        pieces.append((at, at + n, at + dev))
        at += n
    nbytes = at + int(rng.integers(0, 30))
    body = rng.integers(0, 256, nbytes, dtype=np.uint8)
    dev_bytes = pieces[-1][2] + pieces[-1][1] - pieces[-1][0]
    image, hits = np.zeros(dev_bytes, np.uint8), np.zeros(dev_bytes, np.int64)
    slice_bytes = int(rng.integers(1, 97))
    for start in range(0, nbytes, slice_bytes):
        length = min(slice_bytes, nbytes - start)
        for off, to, n in pack.slice_copies(start, length, pieces):
            assert 0 <= off and off + n <= length
            image[to : to + n] = body[start + off : start + off + n]
            hits[to : to + n] += 1
    want, covered = np.zeros(dev_bytes, np.uint8), np.zeros(dev_bytes, np.int64)
    for a, b, d in pieces:
        want[d : d + b - a] = body[a:b]
        covered[d : d + b - a] = 1
    assert np.array_equal(hits, covered) and np.array_equal(image, want)


def test_cache_index_rejects_what_it_cannot_read(tmp_path):
    import json

    from tinybark_b200 import pack

    def write(header, body=b""):
        blob = json.dumps(header).encode()
        blob += b" " * (-len(blob) % 8)
        path = tmp_path / "w.safetensors"
        path.write_bytes(len(blob).to_bytes(8, "little") + blob + body)
        return path

    ok = write({"a": {"dtype": "F16", "shape": [2, 3], "data_offsets": [0, 12]}}, bytes(12))
    assert pack.cache_index(ok)[2]["a"].shape == (2, 3)
    with pytest.raises(ValueError):
        pack.cache_index(write({"a": {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4]}}, bytes(4)))
    with pytest.raises(ValueError):
        pack.cache_index(write({"a": {"dtype": "F16", "shape": [4], "data_offsets": [0, 8]}}, bytes(6)))
    with pytest.raises(ValueError):
        pack.cache_index(write({"a": {"dtype": "F32", "shape": [1], "data_offsets": [2, 6]}}, bytes(6)))
    with pytest.raises(ValueError, match="overlap"):
        pack.cache_index(write({"a": {"dtype": "F16", "shape": [4], "data_offsets": [0, 8]},
                                "b": {"dtype": "F16", "shape": [2], "data_offsets": [6, 10]}}, bytes(10)))


def test_layout_refuses_reads_outside_a_tensor():
    from tinybark_b200 import _lib as L
    from tinybark_b200 import pack

    lay = pack.Layout({"t": pack.Source(0, (4, 8), L.SRC_F32)}, L.BF16)
    lay.view("ok", "t", (8, 4), (1, 8))  # the transpose
    with pytest.raises(ValueError):
        lay.view("over", "t", (8, 5), (1, 8))
    with pytest.raises(ValueError):
        lay.tensor("reshape", "t", (5, 8))
    with pytest.raises(KeyError):
        lay.tensor("missing", "u")


@pytest.mark.skipif(torch.cuda.is_available(), reason="argument checks on a host without a GPU")
def test_repack_checks_every_job_before_running():
    """Each job here breaks one rule; tb_repack returns TB_ERR_ARG before touching a
    buffer (the pointers are never dereferenced)."""
    from tinybark_b200 import _lib as L

    src, dst, jobs_dev = 1 << 20, 2 << 20, 3 << 20  # aligned placeholders

    def job(**kw):
        j = L.RepackJob()
        j.src_off, j.dst_off, j.src_type, j.dst_type = 0, 0, L.SRC_F16, L.BF16
        j.dims[:] = (1, 1, 4, 8)
        j.stride[:] = (0, 0, 8, 1)
        for k, v in kw.items():
            if k in ("dims", "stride"):
                getattr(j, k)[:] = v
            else:
                setattr(j, k, v)
        return j

    def status(j, src_bytes=64, dst_bytes=64, src_ptr=src):
        table = (L.RepackJob * 1)(j)
        return L.lib.tb_repack(table, 1, jobs_dev, src_ptr, src_bytes, dst, dst_bytes, None)

    bad = [
        job(src_off=2),  # reads 2 + 64 bytes of 64
        job(stride=(0, 0, 9, 1)),  # last element 3 * 9 + 7 = 34 >= 32
        job(stride=(0, 0, -8, 1)),
        job(src_off=1),  # not a multiple of 2
        job(dst_off=2, dst_type=L.F32),  # not a multiple of 4
        job(dst_off=8),  # writes 8 + 64 bytes of 64
        job(src_type=7),
        job(dst_type=5),
        job(dims=(-1, 1, 4, 8)),
        job(dims=(65536, 65536, 1, 1), stride=(0, 0, 0, 0), fill=1),  # 2^32 elements
    ]
    for j in bad:
        assert status(j) == 1
    assert status(job(), src_ptr=None) == 1  # a reading job needs a source
    assert status(job(), src_bytes=63) == 1
    assert L.lib.tb_repack((L.RepackJob * 1)(job()), 1, jobs_dev + 4, src, 64, dst, 64, None) == 1
    assert L.lib.tb_repack(None, 0, None, None, 0, None, 0, None) == 0  # nothing to do
