"""The block-scaled FP8 (MXFP8) FFN kernels against the oracle (oracle/mx.py): the
quantizer bit for bit (codes and scales), and the block-scaled GEMM against the float64
product of the dequantized operands, with the fp32 accumulation's rounding as the bound:
|C - C_ref| <= 2^-20 * sum_k |a_k w_k| per output (K <= 4096 fp32 additions)."""

import numpy as np
import pytest
import torch

from oracle import mx

pytestmark = pytest.mark.gpu


def sample(rows, k, seed, dtype):
    """Rows of N(0, 1) values at block-varying scales (1e-6 .. 1e4), with all-zero blocks,
    one block of tiny values and one of values that saturate E4M3."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, k)) * np.exp(rng.uniform(np.log(1e-6), np.log(1e4), (rows, k // 32))).repeat(32, 1)
    x[0, :32] = 0
    x[1 % rows, 32:64] = rng.standard_normal(32) * 1e-38
    x[2 % rows, 64:96] = np.linspace(-3e4, 3e4, 32)
    t = torch.from_numpy(x.astype(np.float32))
    if dtype == "bf16":
        t = t.to(torch.bfloat16)
    return t.cuda(), t.float().numpy().astype(np.float64)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("rows,k", [(200, 512), (128, 1024), (37, 4096)])
def test_quantize_matches_oracle(dtype, rows, k):
    from tinybark_b200 import kernels as K

    x, ref = sample(rows, k, rows + k, dtype)
    q = K.MX(x)
    torch.cuda.synchronize()
    codes, exps = mx.mxfp8_quantize(ref)
    got_codes = q.codes.cpu().numpy()
    assert np.array_equal(got_codes[:rows], codes)
    assert (got_codes[rows:] == 0).all()  # padding rows
    assert np.array_equal(q.scale_exponents().cpu().numpy(), exps)


def _operands(m, n, k, seed):
    rng = np.random.default_rng(seed)
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    w = torch.from_numpy((rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32)).cuda()
    qa = mx.mxfp8_dequantize(*mx.mxfp8_quantize(a.cpu().numpy().astype(np.float64)))
    qw = mx.mxfp8_dequantize(*mx.mxfp8_quantize(w.cpu().numpy().astype(np.float64)))
    return a, w, qa @ qw.T, np.abs(qa) @ np.abs(qw).T


@pytest.mark.parametrize("m,n,k", [(300, 256, 1024), (128, 1024, 4096), (1000, 4096, 1024)])
def test_mx_gemm_matches_oracle(m, n, k):
    from tinybark_b200 import _lib as L
    from tinybark_b200 import kernels as K

    a, w, ref, mag = _operands(m, n, k, m + n)
    out = torch.full((m, n), float("nan"), device="cuda")
    ep = L.Epilogue(kind=L.EPI_STORE, out_dtype=L.F32, out=out.data_ptr(), ldo=n)
    K.gemm_mx(K.MX(a), K.MX(w), ep)
    K.check()
    got = out.cpu().numpy().astype(np.float64)
    assert (np.abs(got - ref) <= 2.0**-20 * mag + 1e-30).all()


def test_mx_gemm_silu_and_residual_epilogues():
    from tinybark_b200 import _lib as L
    from tinybark_b200 import kernels as K

    m, n, k = 260, 512, 1024
    a, w, ref, _ = _operands(m, n, k, 9)
    qa, qw = K.MX(a), K.MX(w)
    h = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    K.gemm_mx(qa, qw, L.Epilogue(kind=L.EPI_SILU, out_dtype=L.BF16, out=h.data_ptr(), ldo=n))
    res0 = torch.randn(m, n, device="cuda")
    res = res0.clone()
    K.gemm_mx(qa, qw, L.Epilogue(kind=L.EPI_RESIDUAL, out=res.data_ptr(), ldo=n, alpha=0.5))
    K.check()
    silu = ref / (1 + np.exp(-ref))
    assert np.abs(h.float().cpu().numpy() - silu).max() <= 1e-2 * np.abs(silu).max()
    want = res0.cpu().numpy() + 0.5 * ref
    assert np.abs(res.cpu().numpy() - want).max() <= 1e-5 * np.abs(want).max()


def test_encoder_with_block_scaled_ffn():
    """24 layers, bf16, the FFN GEMMs block-scaled (Engine ffn="mxfp8"), on 8 of the 30 s
    clips of the batched workload: encoder output against the float32 oracle within
    max-rel 0.1 (E4M3 keeps 3 mantissa bits: each FFN input and weight carries up to 2^-4
    relative rounding, against 2^-8 in bf16), and the decoded tokens against the bf16
    encoder's on all 8 clips, the agreement printed."""
    from conftest import max_rel, state_dict
    from oracle import encoder, frontend
    from tinybark_b200 import synthetic, weights
    from tinybark_b200.engine import Engine

    clips = [synthetic.to_float(synthetic.clip(30.0, seed)) for seed in range(1, 9)]
    sd = state_dict(24)
    conv, cfg = weights.convert(sd, synthetic.config(24)), synthetic.config(24)
    toks, encs = {}, {}
    for ffn in ("bf16", "mxfp8"):
        eng = Engine(conv, cfg, dtype="bf16", ffn=ffn)
        plan = eng.plan([len(c) // 160 for c in clips])
        s, o = eng.upload(clips)
        enc = eng.encode(eng.features(s, o, plan), plan)
        tokens, counts = eng.decode(enc, plan)
        eng.check()
        e, off = enc.cpu().numpy(), plan.t3_off.cpu().numpy()
        encs[ffn] = [e[off[i] : off[i + 1]] for i in range(len(clips))]
        t, c = tokens.cpu().numpy(), counts.cpu().numpy()
        toks[ffn] = [t[i, : c[i]].tolist() for i in range(len(clips))]
        del eng
    errs = []
    for i in (0, 5):
        ref = encoder.encode(sd, frontend.features(clips[i]))
        errs.append((max_rel(encs["bf16"][i], ref), max_rel(encs["mxfp8"][i], ref)))
    same = sum(a == b for a, b in zip(toks["bf16"], toks["mxfp8"]))
    print(f"mxfp8 FFN: encoder max-rel vs fp32 oracle {[round(e[1], 4) for e in errs]} "
          f"(bf16 {[round(e[0], 4) for e in errs]}); tokens identical to bf16 on {same}/{len(clips)} clips")
    assert max(e[1] for e in errs) < 0.1
