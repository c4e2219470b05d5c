"""Oracle (test infrastructure only): the FastConformer encoder of Parakeet-TDT-0.6B-v3
and its encoder projector, in torch float32 on the CPU, on one clip at its exact length
(no padding, so no masks: padded rows never reach valid ones, as
tinybark/mojo/bark/model.mojo:1-6 notes).

Follows transformers' ParakeetEncoder (modeling_parakeet.py: subsampling 357-424,
positions 51-98, block 442-470, attention 259-355, conv module 116-186, feed forward
101-113) with Bark's config: no attention or conv biases, no input scale
(tinybark/tinygrad/model.py:99-158), then encoder_projector (model.py:158).
Weights are the checkpoint-named state dict (tinybark_b200.synthetic.state_dict).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

HIDDEN, HEADS, HEAD_DIM = 1024, 8, 128


def _t(sd, name):
    v = sd[name]
    return v if isinstance(v, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(v))


def positions(length: int, hidden: int = HIDDEN) -> torch.Tensor:
    """(2*length-1, hidden): row n is relative position length-1-n, as interleaved
    [sin, cos] pairs; inverse frequencies and angles in float32 (modeling_parakeet.py:56-98)."""
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, hidden, 2, dtype=torch.int64).float() / hidden))
    pos = torch.arange(length - 1, -length, -1).float()
    freqs = pos[:, None] * inv_freq[None, :]
    return torch.stack([freqs.sin(), freqs.cos()], -1).reshape(2 * length - 1, hidden)


def subsample(sd, feats: torch.Tensor) -> torch.Tensor:
    """(F, 128) features to (T, 1024) (modeling_parakeet.py:357-424; tinygrad/model.py:87-97)."""
    p = "encoder.subsampling."
    x = feats[None, None]
    x = F.relu(F.conv2d(x, _t(sd, p + "layers.0.weight"), _t(sd, p + "layers.0.bias"), stride=2, padding=1))
    for dw, pw in ((2, 3), (5, 6)):
        x = F.conv2d(x, _t(sd, p + f"layers.{dw}.weight"), _t(sd, p + f"layers.{dw}.bias"), stride=2, padding=1, groups=x.shape[1])
        x = F.relu(F.conv2d(x, _t(sd, p + f"layers.{pw}.weight"), _t(sd, p + f"layers.{pw}.bias")))
    b, c, t, f = x.shape
    x = x.transpose(1, 2).reshape(b, t, c * f)
    return F.linear(x, _t(sd, p + "linear.weight"), _t(sd, p + "linear.bias"))[0]


def layernorm(x, sd, name):
    return F.layer_norm(x, (HIDDEN,), _t(sd, name + ".weight"), _t(sd, name + ".bias"), 1e-5)


def feed_forward(x, sd, p):
    return F.linear(F.silu(F.linear(x, _t(sd, p + "linear1.weight"))), _t(sd, p + "linear2.weight"))


def attention(x, sd, p, pos):
    """Relative-position MHSA: score(i, j) = ((q_i+u)·k_j + (q_i+v)·r_{T-1-i+j}) / sqrt(128),
    softmax over j, then the values and o_proj (modeling_parakeet.py:259-355; the
    rel-shift as an index, tinybark/mojo/bark/model.mojo:176-178)."""
    t = x.shape[0]
    q = F.linear(x, _t(sd, p + "q_proj.weight")).view(t, HEADS, HEAD_DIM).transpose(0, 1)
    k = F.linear(x, _t(sd, p + "k_proj.weight")).view(t, HEADS, HEAD_DIM).transpose(0, 1)
    v = F.linear(x, _t(sd, p + "v_proj.weight")).view(t, HEADS, HEAD_DIM).transpose(0, 1)
    r = F.linear(pos, _t(sd, p + "relative_k_proj.weight")).view(2 * t - 1, HEADS, HEAD_DIM).transpose(0, 1)
    qu = q + _t(sd, p + "bias_u")[:, None, :]
    qv = q + _t(sd, p + "bias_v")[:, None, :]
    ac = qu @ k.transpose(1, 2)
    bd = qv @ r.transpose(1, 2)  # (H, T, 2T-1)
    i = torch.arange(t)[:, None]
    j = torch.arange(t)[None, :]
    bd = torch.gather(bd, 2, (t - 1 - i + j).expand(HEADS, t, t))
    scores = (ac + bd) * HEAD_DIM**-0.5
    out = torch.softmax(scores, -1) @ v
    return F.linear(out.transpose(0, 1).reshape(t, HIDDEN), _t(sd, p + "o_proj.weight"))


def conv_module(x, sd, p):
    """pointwise_conv1, GLU, depthwise k=9 pad 4, BatchNorm (eval), SiLU, pointwise_conv2
    (modeling_parakeet.py:116-186)."""
    y = F.linear(x, _t(sd, p + "pointwise_conv1.weight")[:, :, 0])
    y = y[:, :HIDDEN] * torch.sigmoid(y[:, HIDDEN:])
    y = F.conv1d(y.T[None], _t(sd, p + "depthwise_conv.weight"), padding=4, groups=HIDDEN)[0]
    mean, var = _t(sd, p + "norm.running_mean"), _t(sd, p + "norm.running_var")
    gamma, beta = _t(sd, p + "norm.weight"), _t(sd, p + "norm.bias")
    y = (y - mean[:, None]) / torch.sqrt(var[:, None] + 1e-5) * gamma[:, None] + beta[:, None]
    y = F.silu(y).T
    return F.linear(y, _t(sd, p + "pointwise_conv2.weight")[:, :, 0])


def block(x, sd, i, pos):
    """One conformer block (modeling_parakeet.py:442-470)."""
    p = f"encoder.layers.{i}."
    x = x + 0.5 * feed_forward(layernorm(x, sd, p + "norm_feed_forward1"), sd, p + "feed_forward1.")
    x = x + attention(layernorm(x, sd, p + "norm_self_att"), sd, p + "self_attn.", pos)
    x = x + conv_module(layernorm(x, sd, p + "norm_conv"), sd, p + "conv.")
    x = x + 0.5 * feed_forward(layernorm(x, sd, p + "norm_feed_forward2"), sd, p + "feed_forward2.")
    return layernorm(x, sd, p + "norm_out")


def layer_count(sd) -> int:
    n = 0
    while f"encoder.layers.{n}.norm_out.weight" in sd:
        n += 1
    return n


@torch.inference_mode()
def encode(sd, feats: np.ndarray, layers: int | None = None, hidden: bool = False):
    """(F, 128) features to encoder frames projected for the joint, (T, 640) float32.
    With hidden=True, also the (T, 1024) encoder output before the projector."""
    layers = layer_count(sd) if layers is None else layers
    x = subsample(sd, torch.from_numpy(np.ascontiguousarray(feats, np.float32)))
    pos = positions(x.shape[0])
    for i in range(layers):
        x = block(x, sd, i, pos)
    enc = F.linear(x, _t(sd, "encoder_projector.weight"), _t(sd, "encoder_projector.bias"))
    return (enc.numpy(), x.numpy()) if hidden else enc.numpy()


def hf_encoder(sd, layers: int, max_positions: int = 8192):
    """transformers' ParakeetEncoder with Bark's config and `sd` loaded, float32, eval:
    the third-party module the reference's PyTorch backend runs
    (tinybark/pytorch/model.py:12; modeling_parakeet.py:576-640)."""
    from transformers import ParakeetEncoder, ParakeetEncoderConfig

    cfg = ParakeetEncoderConfig(
        num_mel_bins=128, attention_bias=False, convolution_bias=False, scale_input=False,
        num_hidden_layers=layers, max_position_embeddings=max_positions,
        dropout=0.0, dropout_positions=0.0, layerdrop=0.0, activation_dropout=0.0, attention_dropout=0.0,
    )
    model = ParakeetEncoder(cfg).eval()
    prefix = "encoder."
    own = {k[len(prefix):]: _t(sd, k) for k in sd if k.startswith(prefix) and not k.startswith("encoder_projector")}
    own = {k: v for k, v in own.items() if not k.startswith("layers.") or int(k.split(".")[1]) < layers}
    missing, unexpected = model.load_state_dict(own, strict=False)
    assert not unexpected and all("num_batches_tracked" in m for m in missing), (missing[:5], unexpected[:5])
    return model
