"""Each sm_100a kernel through the C ABI against a float64 torch restatement of the same
operation. fp32 kernels within 1e-5 (max-rel), bf16 kernels within 1e-2 of the
reference computed from the same bf16-rounded inputs."""

import ctypes

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import max_rel

pytestmark = pytest.mark.gpu

TOL = {0: 1e-5, 1: 1e-2}


@pytest.fixture(scope="module")
def L():
    from tinybark_b200 import _lib

    return _lib


def stream():
    return torch.cuda.current_stream().cuda_stream


def tdt(dtype):
    return torch.bfloat16 if dtype == 1 else torch.float32


def gemm(L, dtype, a, w, ep, err):
    L.check(L.lib.tb_gemm(dtype, a.data_ptr(), a.stride(0), w.data_ptr(), a.shape[0], w.shape[0], a.shape[1],
                          ctypes.byref(ep), err.data_ptr(), stream()), "tb_gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def operands(dtype, m, n, k, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(m, k, device="cuda", generator=g).to(tdt(dtype))
    w = (torch.randn(n, k, device="cuda", generator=g) / k**0.5).to(tdt(dtype))
    return a, w, a.double() @ w.double().T


@pytest.fixture
def err():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (77, 384, 128), (300, 512, 1024), (129, 640, 640), (1000, 1024, 4096)])
def test_gemm_store_bias(L, dtype, m, n, k, err):
    a, w, ref = operands(dtype, m, n, k)
    bias = torch.randn(n, device="cuda")
    out = torch.full((m, n), float("nan"), device="cuda")
    ep = L.Epilogue(kind=L.EPI_STORE, out_dtype=0, out=out.data_ptr(), ldo=n, bias=bias.data_ptr())
    gemm(L, dtype, a, w, ep, err)
    assert max_rel(out.cpu(), (ref + bias.double()).cpu()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [0, 1])
def test_gemm_silu_residual_relu(L, dtype, err):
    m, n, k = 333, 512, 256
    a, w, ref = operands(dtype, m, n, k, seed=1)
    out = torch.empty(m, n, device="cuda", dtype=tdt(dtype))
    gemm(L, dtype, a, w, L.Epilogue(kind=L.EPI_SILU, out_dtype=dtype, out=out.data_ptr(), ldo=n), err)
    assert max_rel(out.float().cpu(), F.silu(ref).cpu()) < TOL[dtype]

    res = torch.randn(m, n, device="cuda")
    expect = res.double() + 0.5 * ref
    gemm(L, dtype, a, w, L.Epilogue(kind=L.EPI_RESIDUAL, out=res.data_ptr(), ldo=n, alpha=0.5), err)
    assert max_rel(res.cpu(), expect.cpu()) < TOL[dtype] / 10

    bias = torch.randn(n, device="cuda")
    gemm(L, dtype, a, w, L.Epilogue(kind=L.EPI_BIAS_RELU, out_dtype=dtype, out=out.data_ptr(), ldo=n,
                                    bias=bias.data_ptr()), err)
    assert max_rel(out.float().cpu(), torch.relu(ref + bias.double()).cpu()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("m,n,k", [(125, 1024, 4096), (7, 1024, 1024), (250, 1024, 1024), (130, 1024, 1024)])
def test_gemm_residual_split_k_small_m(L, err, dtype, m, n, k):
    """Residual GEMMs of a few rows (one clip) split K over more SMs, the partial products
    added to the fp32 residual atomically (bf16 tensor-core and fp32 CUDA-core kernels):
    within the residual tolerance of the float64 reference."""
    a, w, ref = operands(dtype, m, n, k, seed=5)
    res = torch.randn(m, n, device="cuda")
    expect = res.double() + 0.5 * ref
    gemm(L, dtype, a, w, L.Epilogue(kind=L.EPI_RESIDUAL, out=res.data_ptr(), ldo=n, alpha=0.5), err)
    assert max_rel(res.cpu(), expect.cpu()) < TOL[dtype] / 10


@pytest.mark.parametrize("m", [2100, 2500])
@pytest.mark.parametrize("kind", ["store", "silu", "residual", "bias_relu", "glu", "qkv"])
def test_gemm_pairs_match_single_cta(L, err, kind, m):
    """bf16 GEMMs of at least 2048 rows run on CTA pairs (256 x 256 tiles, 256-row MMAs
    over two SMs); with the pairs switched off the same call takes one CTA per 128-row
    tile. Both give the same bits, and both match the float64 reference. m = 2100 leaves
    the second CTA of the last row pair entirely past the last row, m = 2500 partly."""
    n, k = {"store": (512, 256), "silu": (1024, 512), "residual": (256, 1024), "bias_relu": (256, 128),
            "glu": (2048, 256), "qkv": (3072, 128)}[kind]
    a, w, ref = operands(1, m, n, k, seed=21)
    bias = torch.randn(n, device="cuda")
    u, v = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    res0 = torch.randn(m, n, device="cuda")
    results = []
    for pairs in (1, 0):
        outs = [torch.full((m, 1024 if kind == "qkv" else (n // 2 if kind == "glu" else n)), float("nan"),
                           device="cuda", dtype=torch.float32 if kind in ("store", "residual") else torch.bfloat16)
                for _ in range(4 if kind == "qkv" else 1)]
        if kind == "residual":
            outs[0].copy_(res0)
        ep = {"store": lambda: L.Epilogue(kind=L.EPI_STORE, out_dtype=0, out=outs[0].data_ptr(), ldo=n,
                                          bias=bias.data_ptr()),
              "silu": lambda: L.Epilogue(kind=L.EPI_SILU, out_dtype=1, out=outs[0].data_ptr(), ldo=n),
              "residual": lambda: L.Epilogue(kind=L.EPI_RESIDUAL, out=outs[0].data_ptr(), ldo=n, alpha=0.5),
              "bias_relu": lambda: L.Epilogue(kind=L.EPI_BIAS_RELU, out_dtype=1, out=outs[0].data_ptr(), ldo=n,
                                              bias=bias.data_ptr()),
              "glu": lambda: L.Epilogue(kind=L.EPI_GLU, out_dtype=1, out=outs[0].data_ptr(), ldo=n // 2),
              "qkv": lambda: L.Epilogue(kind=L.EPI_QKV, out_dtype=1, out=outs[0].data_ptr(), out2=outs[1].data_ptr(),
                                        out3=outs[2].data_ptr(), out4=outs[3].data_ptr(), ldo=1024,
                                        bias_u=u.data_ptr(), bias_v=v.data_ptr())}[kind]()
        was = L.lib.tb_set_gemm_pairs(pairs)
        try:
            gemm(L, 1, a, w, ep, err)
        finally:
            L.lib.tb_set_gemm_pairs(was)
        results.append([o.float().cpu() for o in outs])
    for x, y in zip(*results):
        assert torch.equal(x, y)
    got = results[0]
    if kind == "store":
        want = [ref + bias.double()]
    elif kind == "silu":
        want = [F.silu(ref)]
    elif kind == "residual":
        want = [res0.double() + 0.5 * ref]
    elif kind == "bias_relu":
        want = [torch.relu(ref + bias.double())]
    elif kind == "glu":
        want = [ref[:, 0::2] * torch.sigmoid(ref[:, 1::2])]
    else:
        q = ref[:, :1024]
        want = [q + u.double(), q + v.double(), ref[:, 1024:2048], ref[:, 2048:]]
    for g, wnt in zip(got, want):
        assert max_rel(g, wnt.cpu()) < TOL[1]


@pytest.mark.parametrize("kind", ["silu", "qkv", "store"])
def test_gemm_f32_small_tiles_same_bits(L, err, kind):
    """fp32: a GEMM of a clip or two (125 rows) runs on 64 x 64 tiles, a larger one (300
    rows) on 128 x 128 tiles; every output sums over K in the same order, so the rows they
    share come out bit for bit the same, and both match the float64 product."""
    n = {"silu": 4096, "qkv": 3072, "store": 1024}[kind]
    k = 1024
    g = torch.Generator(device="cuda").manual_seed(31)
    a = torch.randn(300, k, device="cuda", generator=g)
    w = torch.randn(n, k, device="cuda", generator=g) / k**0.5
    bias = torch.randn(n, device="cuda", generator=g)
    u, v = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    results = []
    for m in (125, 300):
        outs = [torch.full((m, 1024 if kind == "qkv" else n), float("nan"), device="cuda") for _ in range(4)]
        ep = {"silu": L.Epilogue(kind=L.EPI_SILU, out_dtype=0, out=outs[0].data_ptr(), ldo=n),
              "store": L.Epilogue(kind=L.EPI_STORE, out_dtype=0, out=outs[0].data_ptr(), ldo=n, bias=bias.data_ptr()),
              "qkv": L.Epilogue(kind=L.EPI_QKV, out_dtype=0, out=outs[0].data_ptr(), out2=outs[1].data_ptr(),
                                out3=outs[2].data_ptr(), out4=outs[3].data_ptr(), ldo=1024, bias_u=u.data_ptr(),
                                bias_v=v.data_ptr())}[kind]
        gemm(L, 0, a[:m], w, ep, err)
        results.append([o[:125].cpu() for o in outs[: (4 if kind == "qkv" else 1)]])
    ref = a[:125].double() @ w.double().T
    want = {"silu": [F.silu(ref)], "store": [ref + bias.double()],
            "qkv": [ref[:, :1024] + u.double(), ref[:, :1024] + v.double(), ref[:, 1024:2048], ref[:, 2048:]]}[kind]
    for x, y, wnt in zip(results[0], results[1], want):
        assert torch.equal(x, y)
        assert max_rel(x, wnt.cpu()) < TOL[0]


@pytest.mark.parametrize("dtype", [0, 1])
def test_gemm_glu(L, dtype, err):
    m, n, k = 200, 2048, 256
    a, w, ref = operands(dtype, m, n, k, seed=2)
    out = torch.empty(m, n // 2, device="cuda", dtype=tdt(dtype))
    gemm(L, dtype, a, w, L.Epilogue(kind=L.EPI_GLU, out_dtype=dtype, out=out.data_ptr(), ldo=n // 2), err)
    expect = ref[:, 0::2] * torch.sigmoid(ref[:, 1::2])
    assert max_rel(out.float().cpu(), expect.cpu()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [0, 1])
def test_gemm_qkv(L, dtype, err):
    m, k = 150, 128
    a, w, ref = operands(dtype, m, 3072, k, seed=3)
    u, v = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    outs = [torch.empty(m, 1024, device="cuda", dtype=tdt(dtype)) for _ in range(4)]
    ep = L.Epilogue(kind=L.EPI_QKV, out_dtype=dtype, out=outs[0].data_ptr(), out2=outs[1].data_ptr(),
                    out3=outs[2].data_ptr(), out4=outs[3].data_ptr(), ldo=1024, bias_u=u.data_ptr(),
                    bias_v=v.data_ptr())
    gemm(L, dtype, a, w, ep, err)
    q, kk, vv = ref[:, :1024], ref[:, 1024:2048], ref[:, 2048:]
    for got, want in zip(outs, (q + u.double(), q + v.double(), kk, vv)):
        assert max_rel(got.float().cpu(), want.cpu()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [0, 1])
def test_gemm_lstm_cell(L, dtype, err):
    lanes = 70
    a, w, ref = operands(dtype, lanes, 2560, 1280, seed=4)
    bias = torch.randn(2560, device="cuda")
    c = torch.randn(lanes, 640, device="cuda")
    h = torch.zeros(lanes, 640, device="cuda")
    hout = torch.zeros(lanes, 1280, device="cuda", dtype=tdt(dtype))
    mask = (torch.arange(lanes, device="cuda") % 3 != 0).int()
    c0 = c.clone()
    ep = L.Epilogue(kind=L.EPI_LSTM, out_dtype=dtype, out=hout.data_ptr(), ldo=1280, out2=None, ldo2=0,
                    bias=bias.data_ptr(), c=c.data_ptr(), h=h.data_ptr(), mask=mask.data_ptr())
    gemm(L, dtype, a, w, ep, err)
    g = (ref + bias.double()).view(lanes, 640, 4)
    i, f, gg, o = torch.sigmoid(g[..., 0]), torch.sigmoid(g[..., 1]), torch.tanh(g[..., 2]), torch.sigmoid(g[..., 3])
    c_new = f * c0.double() + i * gg
    h_new = o * torch.tanh(c_new)
    keep = mask.bool()
    assert max_rel(c[keep].cpu(), c_new[keep].cpu()) < TOL[dtype]
    assert max_rel(h[keep].cpu(), h_new[keep].cpu()) < TOL[dtype]
    assert torch.equal(c[~keep], c0[~keep]) and bool((h[~keep] == 0).all())
    assert max_rel(hout[keep, :640].float().cpu(), h_new[keep].cpu()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [0, 1])
def test_gemm_argmax(L, dtype, err):
    lanes, split, n = 90, 8256, 8448
    a, w, ref = operands(dtype, lanes, n, 640, seed=5)
    bias = torch.randn(n, device="cuda")
    bias[8193:8256] = float("-inf")
    bias[split + 5 :] = float("-inf")
    keys = torch.zeros(lanes, dtype=torch.int64, device="cuda")
    keys2 = torch.zeros(lanes, dtype=torch.int64, device="cuda")
    ep = L.Epilogue(kind=L.EPI_ARGMAX, bias=bias.data_ptr(), keys=keys.data_ptr(), keys2=keys2.data_ptr(),
                    split=split, split_end=split + 5)
    gemm(L, dtype, a, w, ep, err)
    logits = ref + bias.double()
    tok = (0xFFFFFFFF - (keys & 0xFFFFFFFF)).cpu().numpy()
    dur = (0xFFFFFFFF - (keys2 & 0xFFFFFFFF)).cpu().numpy()
    lt, ld = logits[:, :split].cpu().numpy(), logits[:, split : split + 5].cpu().numpy()
    scale = np.abs(lt[np.isfinite(lt)]).max()
    for r in range(lanes):
        assert tok[r] < 8193 and lt[r, tok[r]] >= lt[r].max() - 1e-5 * scale * (1 if dtype == 0 else 100)
        assert ld[r, dur[r]] >= ld[r].max() - 1e-5 * scale * (1 if dtype == 0 else 100)
    if dtype == 0:
        assert (tok == lt.argmax(1)).all() and (dur == ld.argmax(1)).all()


@pytest.mark.parametrize("m", [1, 3, 8])
def test_gemv_f32_few_rows(L, err, m):
    """fp32 GEMMs of at most 8 rows (the fp32 decoder at batch 1-8) run the matrix-vector
    kernel (a warp per weight row, the row in registers): STORE with bias, the LSTM cell
    with a lane mask, and the joint's argmax, each against float64."""
    a, w, ref = operands(0, m, 640, 640, seed=40 + m)
    bias = torch.randn(640, device="cuda")
    out = torch.full((m, 640), float("nan"), device="cuda")
    gemm(L, 0, a, w, L.Epilogue(kind=L.EPI_STORE, out_dtype=0, out=out.data_ptr(), ldo=640, bias=bias.data_ptr()), err)
    assert max_rel(out.cpu(), (ref + bias.double()).cpu()) < TOL[0]

    a, w, ref = operands(0, m, 2560, 1280, seed=50 + m)
    bias = torch.randn(2560, device="cuda")
    c = torch.randn(m, 640, device="cuda")
    h = torch.zeros(m, 640, device="cuda")
    mask = (torch.arange(m, device="cuda") % 2 == 0).int()
    c0 = c.clone()
    gemm(L, 0, a, w, L.Epilogue(kind=L.EPI_LSTM, out_dtype=0, bias=bias.data_ptr(), c=c.data_ptr(), h=h.data_ptr(),
                                mask=mask.data_ptr()), err)
    g = (ref + bias.double()).view(m, 640, 4)
    c_new = torch.sigmoid(g[..., 1]) * c0.double() + torch.sigmoid(g[..., 0]) * torch.tanh(g[..., 2])
    h_new = torch.sigmoid(g[..., 3]) * torch.tanh(c_new)
    keep = mask.bool()
    assert max_rel(c[keep].cpu(), c_new[keep].cpu()) < TOL[0]
    assert max_rel(h[keep].cpu(), h_new[keep].cpu()) < TOL[0]
    assert torch.equal(c[~keep], c0[~keep])

    split, n = 8256, 8448
    a, w, ref = operands(0, m, n, 640, seed=60 + m)
    bias = torch.randn(n, device="cuda")
    bias[8193:split] = float("-inf")
    bias[split + 5 :] = float("-inf")
    keys = torch.zeros(m, dtype=torch.int64, device="cuda")
    keys2 = torch.zeros(m, dtype=torch.int64, device="cuda")
    gemm(L, 0, a, w, L.Epilogue(kind=L.EPI_ARGMAX, bias=bias.data_ptr(), keys=keys.data_ptr(), keys2=keys2.data_ptr(),
                                split=split, split_end=split + 5), err)
    logits = (ref + bias.double()).cpu().numpy()
    tok = (0xFFFFFFFF - (keys & 0xFFFFFFFF)).cpu().numpy()
    dur = (0xFFFFFFFF - (keys2 & 0xFFFFFFFF)).cpu().numpy()
    assert (tok == logits[:, :split].argmax(1)).all() and (dur == logits[:, split : split + 5].argmax(1)).all()


@pytest.mark.parametrize("lanes", [90, 300])
def test_gemm_argmax_first_index_exact(L, err, lanes):
    """bf16 with small-integer operands and biases: every accumulator and logit is an
    exact integer whatever the summation order, ties are common, and the epilogue must
    return the first column of the maximum, as the reference's argmax does
    (tinybark/tinygrad/model.py:43-53). 90 lanes run 64-column tiles, 300 lanes
    256-column tiles (four chunks per row, each row with its own winning chunk)."""
    split, n, k = 8193, 8448, 640
    g = torch.Generator(device="cuda").manual_seed(lanes)
    a = torch.randint(-1, 2, (lanes, k), device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randint(-1, 2, (n, k), device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randint(-2, 3, (n,), device="cuda", generator=g).float()
    bias[split + 5 :] = float("-inf")
    keys = torch.zeros(lanes, dtype=torch.int64, device="cuda")
    keys2 = torch.zeros(lanes, dtype=torch.int64, device="cuda")
    ep = L.Epilogue(kind=L.EPI_ARGMAX, bias=bias.data_ptr(), keys=keys.data_ptr(), keys2=keys2.data_ptr(),
                    split=split, split_end=split + 5)
    gemm(L, 1, a, w, ep, err)
    logits = (a.double() @ w.double().T + bias.double()).cpu().numpy()
    tok = (0xFFFFFFFF - (keys & 0xFFFFFFFF)).cpu().numpy()
    dur = (0xFFFFFFFF - (keys2 & 0xFFFFFFFF)).cpu().numpy()
    ties = sum(int((row == row.max()).sum() > 1) for row in logits[:, :split])
    assert ties > 0  # the case exercises first-index ties
    assert (tok == logits[:, :split].argmax(1)).all()
    assert (dur == logits[:, split : split + 5].argmax(1)).all()


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("fused", [False, True])
def test_layernorm(L, dtype, fused):
    rows = 300
    x = torch.randn(rows, 1024, device="cuda") * 3 + 1
    w, b = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    w2, b2 = torch.randn(1024, device="cuda"), torch.randn(1024, device="cuda")
    y = torch.empty(rows, 1024, device="cuda", dtype=tdt(dtype))
    xd = x.double()
    ref = F.layer_norm(xd, (1024,), w.double(), b.double(), 1e-5)
    xo = torch.empty_like(x) if fused else None
    L.check(L.lib.tb_layernorm(x.data_ptr(), w.data_ptr(), b.data_ptr(), xo.data_ptr() if fused else None,
                               w2.data_ptr() if fused else None, b2.data_ptr() if fused else None, y.data_ptr(),
                               dtype, rows, stream()), "tb_layernorm")
    torch.cuda.synchronize()
    if fused:
        assert max_rel(xo.cpu(), ref.cpu()) < 1e-5
        ref = F.layer_norm(ref, (1024,), w2.double(), b2.double(), 1e-5)
    assert max_rel(y.float().cpu(), ref.cpu()) < TOL[dtype]


def batch_for(L, t3_list, attn_rows):
    """A tb_batch with only the encoder-frame fields set (attention, depthwise conv)."""
    t3 = np.array(t3_list)
    off = np.concatenate([[0], np.cumsum(t3)]).astype(np.int32)
    clip = np.repeat(np.arange(len(t3), dtype=np.int32), t3)
    order = np.argsort(-t3, kind="stable")
    tiles = np.array([(c, r) for c in order for r in range(0, t3[c], attn_rows)], np.int32).reshape(-1)
    keep = [torch.from_numpy(a).cuda() for a in (off, clip, tiles)]
    b = L.Batch()
    b.clips, b.t3_total, b.max_t3 = len(t3), int(off[-1]), int(t3.max())
    b.t3_off, b.t3_clip, b.attn_tiles, b.n_attn_tiles = keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), len(tiles) // 2
    return b, keep, off


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("t3,max_len", [([1, 2, 7, 33, 130, 64], 256), ([300, 65, 128, 129], 384), ([250], 250),
                                        ([375] * 8 + [7, 200], 384)])
def test_relpos_attention(L, dtype, t3, max_len, err):
    from tinybark_b200 import kernels

    _, attn_rows = L.tile_rows(dtype)
    b, keep, off = batch_for(L, t3, attn_rows)
    R = off[-1]
    g = torch.Generator(device="cuda").manual_seed(7)
    q, k, v = (torch.randn(R, 1024, device="cuda", generator=g) for _ in range(3))
    bu, bv = torch.randn(1024, device="cuda", generator=g), torch.randn(1024, device="cuda", generator=g)
    qu, qv, k, v = (x.to(tdt(dtype)) for x in (q + bu, q + bv, k, v))
    rel = torch.randn(2 * max_len - 1, 1024, device="cuda", generator=g).to(tdt(dtype))
    rel_c = kernels.rel_bias(rel, bu, bv) if dtype == 1 else None
    out = torch.empty(R, 1024, device="cuda", dtype=tdt(dtype))
    L.check(L.lib.tb_relpos_attention(dtype, qu.data_ptr(), qv.data_ptr(), k.data_ptr(), v.data_ptr(), rel.data_ptr(),
                                      None if rel_c is None else rel_c.data_ptr(), max_len, ctypes.byref(b),
                                      out.data_ptr(), err.data_ptr(), stream()), "tb_relpos_attention")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # bf16 computes (q+u).r + (v-u).r with both operands rounded to bf16: the reference
    # uses the same rounded operands.
    qpos = qv.double() if dtype == 0 else qu.double() + (bv - bu).to(tdt(dtype)).double()
    for c, T in enumerate(t3):
        s = slice(off[c], off[c + 1])
        hq = lambda x: x[s].double().view(T, 8, 128).transpose(0, 1)
        i = torch.arange(T, device="cuda")[:, None]
        j = torch.arange(T, device="cuda")[None, :]
        r = rel.double()[max_len - 1 - i + j].view(T, T, 8, 128).permute(2, 0, 1, 3)  # (H, i, j, d)
        scores = hq(qu) @ hq(k).transpose(1, 2) + (hq(qpos)[:, :, None, :] * r).sum(-1)
        p = torch.softmax(scores / 128**0.5, -1)
        ref = (p @ hq(v)).transpose(0, 1).reshape(T, 1024)
        assert max_rel(out[s].float().cpu(), ref.cpu()) < TOL[dtype], (c, T)


@pytest.mark.parametrize("dtype", [0, 1])
def test_relpos_attention_long_form(L, dtype, err):
    """One 10-minute clip (T = 7500 encoder frames, the long-form workload) with
    full-context attention; the reference works in 500-row blocks (fp32, rel-shift as a
    gather of the banded scores) so that no T x T x 128 tensor is formed."""
    from tinybark_b200 import kernels

    T = 7500
    _, attn_rows = L.tile_rows(dtype)
    b, keep, off = batch_for(L, [T], attn_rows)
    g = torch.Generator(device="cuda").manual_seed(11)
    q, k, v = (torch.randn(T, 1024, device="cuda", generator=g) for _ in range(3))
    bu, bv = torch.randn(1024, device="cuda", generator=g), torch.randn(1024, device="cuda", generator=g)
    qu, qv, k, v = (x.to(tdt(dtype)) for x in (q + bu, q + bv, k, v))
    rel = torch.randn(2 * T - 1, 1024, device="cuda", generator=g).to(tdt(dtype))
    rel_c = kernels.rel_bias(rel, bu, bv) if dtype == 1 else None
    out = torch.empty(T, 1024, device="cuda", dtype=tdt(dtype))
    L.check(L.lib.tb_relpos_attention(dtype, qu.data_ptr(), qv.data_ptr(), k.data_ptr(), v.data_ptr(), rel.data_ptr(),
                                      None if rel_c is None else rel_c.data_ptr(), T, ctypes.byref(b), out.data_ptr(),
                                      err.data_ptr(), stream()), "tb_relpos_attention")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    qpos = qv.float() if dtype == 0 else qu.float() + (bv - bu).to(tdt(dtype)).float()
    heads = lambda x: x.float().view(-1, 8, 128).transpose(0, 1)  # (H, rows, d)
    K, V, Rh = heads(k), heads(v), heads(rel)
    worst = 0.0
    for i0 in range(0, T, 500):
        i = torch.arange(i0, min(i0 + 500, T), device="cuda")
        band = heads(qpos[i]) @ Rh.transpose(1, 2)  # (H, rows, 2T-1): position T-1-n of row n
        idx = (T - 1 - i[:, None] + torch.arange(T, device="cuda")[None, :]).expand(8, -1, -1)
        scores = heads(qu[i]) @ K.transpose(1, 2) + band.gather(2, idx)
        ref = (torch.softmax(scores / 128**0.5, -1) @ V).transpose(0, 1).reshape(len(i), 1024)
        worst = max(worst, max_rel(out[i].float().cpu(), ref.cpu()))
    assert worst < TOL[dtype]


@pytest.mark.parametrize("dtype", [0, 1])
@pytest.mark.parametrize("t3", [[1, 5, 9, 40, 3], [1, 5, 9, 40, 3, 300, 129, 5000, 33, 700]])
def test_depthwise_conv_silu(L, dtype, t3, err):
    """Ragged clips (frames outside a clip read as zero); the second batch has interior
    tiles and more 32-frame tiles than SMs, so the bf16 kernel's double buffer cycles."""
    b, keep, off = batch_for(L, t3, 32)
    R = off[-1]
    x = torch.randn(R, 1024, device="cuda").to(tdt(dtype))
    w = torch.randn(1024, 9, device="cuda")
    bias = torch.randn(1024, device="cuda")
    y = torch.full((R, 1024), float("nan"), device="cuda", dtype=tdt(dtype))
    L.check(L.lib.tb_conv_depthwise(dtype, x.data_ptr(), w.data_ptr(), bias.data_ptr(), ctypes.byref(b), y.data_ptr(),
                                    err.data_ptr(), stream()), "tb_conv_depthwise")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for c in range(len(t3)):
        s = slice(off[c], off[c + 1])
        ref = F.conv1d(x[s].double().T[None], w.double()[:, None, :], bias.double(), padding=4, groups=1024)[0].T
        assert max_rel(y[s].float().cpu(), F.silu(ref).cpu()) < TOL[dtype], c


def test_depthwise_small_batch_matches_streaming_kernel(L, err):
    """bf16: a few rows run the small-batch kernel, many rows the streaming kernel; the
    clips they share come out bit for bit the same."""
    small, big = [1, 5, 9, 40, 3, 125], [1, 5, 9, 40, 3, 125, 5000]
    outs = []
    x = torch.randn(sum(big), 1024, device="cuda").to(torch.bfloat16)
    w = torch.randn(1024, 9, device="cuda")
    bias = torch.randn(1024, device="cuda")
    for t3 in (small, big):
        b, keep, off = batch_for(L, t3, 32)
        y = torch.full((off[-1], 1024), float("nan"), device="cuda", dtype=torch.bfloat16)
        L.check(L.lib.tb_conv_depthwise(1, x.data_ptr(), w.data_ptr(), bias.data_ptr(), ctypes.byref(b), y.data_ptr(),
                                        err.data_ptr(), stream()), "tb_conv_depthwise")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        outs.append(y[: sum(small)])
    assert torch.equal(outs[0], outs[1])


@pytest.fixture(scope="module")
def engine2():
    from conftest import state_dict
    from tinybark_b200 import synthetic, weights
    from tinybark_b200.engine import Engine

    return Engine(weights.convert(state_dict(2), synthetic.config(2)), synthetic.config(2), dtype="fp32")


def test_frontend_matches_oracle(engine2):
    from conftest import golden_npz
    from oracle import frontend
    from tinybark_b200 import synthetic

    g = golden_npz("frontend.npz")
    clips = [g[f"{n}_samples"] for n in ("two_frames", "odd", "one_second")]
    clips.append(synthetic.to_float(synthetic.clip(7.3, 5)))
    plan = engine2.plan([len(c) // 160 for c in clips])
    samples, off = engine2.upload(clips)
    feats = engine2.features(samples, off, plan).cpu().numpy()
    fo = plan.batch
    start = 0
    for c in clips:
        ref = frontend.features(c)
        got = feats[start : start + len(ref)]
        start += len(ref)
        np.testing.assert_allclose(got, ref, rtol=0, atol=2e-4)


def test_subsample_matches_oracle(engine2):
    from oracle import encoder as oenc
    from oracle import frontend
    from conftest import state_dict
    from tinybark_b200 import _lib as L, synthetic

    clips = [synthetic.to_float(synthetic.clip(s, 40 + i)) for i, s in enumerate((0.05, 1.37, 4.0))]
    feats = [frontend.features(c) for c in clips]
    plan = engine2.plan([len(f) for f in feats])
    x = torch.empty(plan.batch.t3_total, 1024, device="cuda")
    fdev = torch.from_numpy(np.concatenate(feats)).cuda()
    nbytes = L.lib.tb_subsample_workspace_bytes(0, plan.batch.t2_total, plan.batch.t3_total)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    L.check(L.lib.tb_subsample(ctypes.byref(engine2.model), ctypes.byref(plan.batch), fdev.data_ptr(), x.data_ptr(),
                               ws.data_ptr(), nbytes, engine2.err.data_ptr(), stream()), "tb_subsample")
    engine2.check()
    off = plan.t3_off.cpu().numpy()
    for i, f in enumerate(feats):
        ref = oenc.subsample(state_dict(2), torch.from_numpy(f)).numpy()
        assert max_rel(x[off[i] : off[i + 1]].cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("kind,bit", [(0, 1), (1, 4)])
def test_bounded_wait_gives_up_and_reports(L, kind, bit, err):
    """A wait that nothing completes (an mbarrier, or the decoder's grid barrier) gives
    up after the library's limit, sets its TB_DEV_* bit and returns; the context then
    still runs kernels correctly."""
    import time

    scratch = torch.empty(256, dtype=torch.uint8, device="cuda")
    err.zero_()
    t0 = time.time()
    L.check(L.lib.tb_selftest_wait(kind, scratch.data_ptr(), err.data_ptr(), stream()), "tb_selftest_wait")
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert int(err.item()) == bit
    assert 1.0 < waited < 30.0
    err.zero_()
    a, w, ref = operands(1, 64, 256, 64, seed=9)
    out = torch.empty(64, 256, device="cuda", dtype=torch.float32)
    gemm(L, 1, a, w, L.Epilogue(kind=L.EPI_STORE, out_dtype=L.F32, out=out.data_ptr(), ldo=256), err)
    assert int(err.item()) == 0
    assert max_rel(out.cpu(), ref.cpu()) < TOL[1]


def random_repack_jobs(rng, n16: int, n32: int, off32: int):
    """Jobs over a source of n16 f16 values at byte 0 and n32 f32 values at byte off32:
    random 4-D strided reads (repeats and transposes included), a job of many chunks, an
    empty job, and fills; destinations packed at element-size alignment."""
    jobs, dst = [], 0
    for t in range(48):
        dst_type = int(rng.integers(0, 2))
        esz = 2 if dst_type == 1 else 4
        dst = -(-dst // esz) * esz
        if t == 7:
            dims = (1, 1, 300, 257)  # 77100 elements: 19 chunks
        elif t == 20:
            dims = (3, 0, 5, 2)  # no elements
        else:
            dims = tuple(int(d) for d in rng.integers(1, 13, 4))
        if t % 9 == 4:
            value = float(rng.choice([0.0, -np.inf, np.inf, 1.5, -3.25e38]))
            jobs.append((0, dst, (0, 0, 0, 0), dims, 0, dst_type, 1, value))
        else:
            f16 = bool(rng.integers(0, 2))
            n = n16 if f16 else n32
            strides = tuple(int(s) for s in rng.integers(0, 40, 4)) if t != 7 else (0, 0, 257, 1)
            reach = sum((d - 1) * s for d, s in zip(dims, strides) if d > 0)
            base = int(rng.integers(0, n - reach))
            src_off = (0 if f16 else off32) + base * (2 if f16 else 4)
            jobs.append((src_off, dst, strides, dims, 0 if f16 else 1, dst_type, 0, 0.0))
        dst += int(np.prod(dims)) * esz
    return jobs, dst


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_repack_matches_numpy_on_random_jobs(L, seed):
    """tb_repack against its numpy restatement, bit for bit: f16 and f32 sources (f16
    infinities and subnormals; f32 values at bf16 rounding ties and near the f32 maximum,
    which round to infinity) into f32 and bf16 destinations."""
    from conftest import repack_numpy
    from tinybark_b200 import pack

    rng = np.random.default_rng(seed)
    n16, n32 = 300_000, 200_000
    a16 = rng.standard_normal(n16).astype(np.float16)
    a16[:4] = [np.inf, -np.inf, 6e-8, -1e-5]
    a32 = (rng.standard_normal(n32) * 1e3).astype(np.float32)
    bits = a32.view(np.uint32)
    bits[:64] = (bits[:64] & 0xFFFF0000) | 0x8000  # ties: even and odd bf16 mantissas
    a32[64:66] = [3.4028235e38, -3.4e38]
    off32 = -(-a16.nbytes // 256) * 256
    src = np.zeros(off32 + a32.nbytes, np.uint8)
    src[: a16.nbytes] = a16.view(np.uint8)
    src[off32:] = a32.view(np.uint8)
    jobs, size = random_repack_jobs(rng, n16, n32, off32)
    lay = pack.Layout({}, L.BF16)
    lay.jobs, lay.size = jobs, size
    out = torch.full((size + 64,), 0xA5, dtype=torch.uint8, device="cuda")
    lay.run(torch.from_numpy(src).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = repack_numpy(jobs, src, size)
    written = np.zeros(size, bool)
    for j in jobs:
        esz = 2 if j[5] == 1 else 4
        written[j[1] : j[1] + int(np.prod(j[3])) * esz] = True
    assert np.array_equal(got[:size][written], want[written])
    assert (got[:size][~written] == 0xA5).all() and (got[size:] == 0xA5).all()  # nothing else touched


def test_text_join_matches_numpy(L):
    """tb_text_offsets + tb_text_bytes against the numpy join of each lane's piece bytes:
    empty pieces, empty / full / over-long / negative counts (clamped to [0, ld]), and ids
    outside the table, which add nothing and set the text error bit."""
    rng = np.random.default_rng(3)
    vocab, lanes, ld = 500, 300, 60
    lens = rng.integers(0, 7, vocab)
    lens[::17] = 0
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    data = rng.integers(0, 256, int(off[-1]), dtype=np.uint8)
    tokens = rng.integers(0, vocab, (lanes, ld)).astype(np.int32)
    counts = rng.integers(0, ld + 1, lanes).astype(np.int32)
    counts[:4] = [0, ld, ld + 5, -2]
    tokens[7, 0], tokens[8, 0] = vocab + 4, -1
    counts[7:9] = 5
    want = []
    for l in range(lanes):
        n = min(max(int(counts[l]), 0), ld)
        want.append(b"".join(data[off[i] : off[i + 1]].tobytes() for i in tokens[l, :n] if 0 <= i < vocab))
    dev = lambda a: torch.from_numpy(a).cuda()
    tk, cn, po, pb = dev(tokens), dev(counts), dev(off), dev(data)
    text_off = torch.full((lanes + 1,), -1, dtype=torch.int64, device="cuda")
    e = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.lib.tb_text_offsets(tk.data_ptr(), ld, cn.data_ptr(), lanes, po.data_ptr(), vocab, text_off.data_ptr(),
                                 e.data_ptr(), stream()) == 0
    o = text_off.cpu().numpy()
    assert list(np.diff(o)) == [len(w) for w in want] and o[0] == 0
    text = torch.full((int(o[-1]) + 16,), 0xA5, dtype=torch.uint8, device="cuda")
    assert L.lib.tb_text_bytes(tk.data_ptr(), ld, cn.data_ptr(), lanes, po.data_ptr(), pb.data_ptr(), pb.numel(), vocab,
                               text_off.data_ptr(), text.data_ptr(), int(o[-1]), stream()) == 0
    raw = text.cpu().numpy().tobytes()
    assert [raw[o[l] : o[l + 1]] for l in range(lanes)] == want
    assert raw[int(o[-1]) :] == b"\xa5" * 16  # nothing past the end
    assert int(e.item()) == 16


def test_fast_math_within_bounds(L):
    """The epilogues' fast arithmetic against float64 (tb_selftest_math): the Newton
    reciprocal over y in [1, 1e30] within 1e-5 relative, the one-MUFU sigmoid and SiLU (and
    their two-wide forms) over x in [-90, 90] within 2e-5 absolute (sigmoid) and relative
    2e-5 + 1e-30 (SiLU), the tanh-based sigmoid within 5e-4, the tanh-based two-wide SiLU
    within 2^-11.9 |x| (half the tanh's relative bound on |x / 2|) and the hardware tanh
    within 2^-10 relative plus 1e-6 absolute, each checked against the bound CUDA documents
    for its approximate instructions."""
    g = torch.Generator().manual_seed(5)
    n = 1 << 20
    cases = {
        0: torch.exp(torch.rand(n, generator=g, dtype=torch.float64) * 69.0).float(),  # 1 .. 1e30
        **{k: (torch.rand(n, generator=g, dtype=torch.float64) * 180 - 90).float() for k in (1, 2, 3, 4, 5, 7)},
        6: (torch.rand(n, generator=g, dtype=torch.float64) * 20 - 10).float(),
    }
    cases[3][-1] = cases[4][-1] = cases[7][-1] = 0.0
    for kind, x in cases.items():
        xd = x.cuda()
        y = torch.full_like(xd, float("nan"))
        L.check(L.lib.tb_selftest_math(kind, xd.data_ptr(), y.data_ptr(), n - (kind in (4, 7)), stream()),
                "tb_selftest_math")
        torch.cuda.synchronize()
        got = y.cpu().double()
        xx = x.double()
        sig = torch.sigmoid(xx)
        if kind in (4, 7):
            got, xx, sig = got[:-1], xx[:-1], sig[:-1]
            assert torch.isnan(y[-1].cpu())  # past n: untouched
        if kind == 0:
            assert ((got * xx - 1).abs().max() < 1e-5), kind
        elif kind in (1, 3):
            assert (got - sig).abs().max() < 2e-5, kind
        elif kind in (2, 4):
            assert ((got - xx * sig).abs() <= 2e-5 * (xx * sig).abs() + 1e-30).all(), kind
        elif kind == 5:
            assert (got - sig).abs().max() < 5e-4, kind
        elif kind == 7:  # h + h tanh(h), h = x / 2: the tanh's 2^-10.987 relative error on |h|
            ref = xx * sig
            assert ((got - ref).abs() <= 2.0**-11.9 * xx.abs() + 2.0**-23 * ref.abs() + 1e-30).all(), kind
        else:
            t = torch.tanh(xx)
            assert ((got - t).abs() <= 2.0 ** -10 * t.abs() + 1e-6).all(), kind
