"""The converted weight layout the cuda backend consumes, and its on-disk form.

The layout is the one tinybark's converter defines (tinybark/weights.py:62-89): q/k/v
fused into one [3072, 1024] matrix, each conv module's BatchNorm folded into its
depthwise conv, each LSTM layer's input and hidden weights fused into one [2560, 1280]
matrix with one summed bias, and the joint head split into a token head padded to a
multiple of 64 rows (zero weights, -inf bias) and a 5-row duration head. The names and
the arithmetic have to be the same as the reference's for the cuda backend to read the
same cache file, so `convert` follows it step by step.

The on-disk form is tinybark's fp16 safetensors cache (tinybark/weights.py:92-120):
an 8-byte little-endian header length, a JSON header padded with spaces to a multiple
of 8 bytes, then every tensor as fp16 in header order.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

BN_EPS = 1e-5
VOCAB_ALIGN = 64


def convert(sd: dict[str, np.ndarray], config: dict) -> dict[str, np.ndarray]:
    """Checkpoint-named float32 state dict to the converted layout (tinybark/weights.py:62-89).
    `sd` is not modified."""
    sd = dict(sd)
    layers, vocab = config["encoder_config"]["num_hidden_layers"], config["vocab_size"]
    out: dict[str, np.ndarray] = {}
    for i in range(layers):
        a = f"encoder.layers.{i}.self_attn."
        out[a + "qkv"] = np.concatenate([sd.pop(a + f"{n}_proj.weight") for n in "qkv"])
        for n in ("o_proj.weight", "relative_k_proj.weight", "bias_u", "bias_v"):
            out[a + n] = sd.pop(a + n)
        c = f"encoder.layers.{i}.conv."
        scale = sd.pop(c + "norm.weight") / np.sqrt(sd.pop(c + "norm.running_var") + BN_EPS)
        out[c + "depthwise.weight"] = sd.pop(c + "depthwise_conv.weight") * scale[:, None, None]
        out[c + "depthwise.bias"] = sd.pop(c + "norm.bias") - sd.pop(c + "norm.running_mean") * scale
        sd.pop(c + "norm.num_batches_tracked", None)
    for l in range(config["num_decoder_layers"]):
        p = "decoder.lstm."
        out[p + f"weight_l{l}"] = np.concatenate([sd.pop(p + f"weight_ih_l{l}"), sd.pop(p + f"weight_hh_l{l}")], 1)
        out[p + f"bias_l{l}"] = sd.pop(p + f"bias_ih_l{l}") + sd.pop(p + f"bias_hh_l{l}")
    weight, bias = sd.pop("joint.head.weight"), sd.pop("joint.head.bias")
    pad = -vocab % VOCAB_ALIGN
    out["joint.token_head.weight"] = np.pad(weight[:vocab], ((0, pad), (0, 0)))
    out["joint.token_head.bias"] = np.pad(bias[:vocab], (0, pad), constant_values=-np.inf)
    out["joint.duration_head.weight"], out["joint.duration_head.bias"] = weight[vocab:], bias[vocab:]
    out.update(sd)
    return {k: np.ascontiguousarray(v) for k, v in out.items()}


def save(tensors: dict[str, np.ndarray], path: str | Path) -> None:
    """Writes the fp16 safetensors cache format (tinybark/weights.py:92-103)."""
    header, offset = {}, 0
    for name, value in tensors.items():
        header[name] = {"dtype": "F16", "shape": list(value.shape), "data_offsets": [offset, offset + value.size * 2]}
        offset += value.size * 2
    blob = json.dumps(header).encode()
    blob += b" " * (-len(blob) % 8)
    with open(path, "wb") as file:
        file.write(len(blob).to_bytes(8, "little") + blob)
        for value in tensors.values():
            file.write(value.astype(np.float16).tobytes())


def load(path: str | Path) -> dict[str, np.ndarray]:
    """Reads a converted cache file in one read (the pattern of
    tinybark/tinygrad/weights.py:10-26), returning float32 arrays."""
    data = Path(path).read_bytes()
    n = int.from_bytes(data[:8], "little")
    header = json.loads(data[8 : 8 + n])
    body = memoryview(data)[8 + n :]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        if info["dtype"] not in ("F16", "F32"):
            raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
        start, end = info["data_offsets"]
        dtype = np.float16 if info["dtype"] == "F16" else np.float32
        out[name] = np.frombuffer(body[start:end], dtype=dtype).reshape(info["shape"]).astype(np.float32)
    return out
