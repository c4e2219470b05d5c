"""The converted weight layout the cuda backend consumes, and its on-disk form.

The converted layout is tinybark's (tinybark/weights.py:62-89); its rules, as this
module states them:

- self-attention: q, k and v projections stacked by rows into `self_attn.qkv`
  [3072, 1024]; o_proj, relative_k_proj, bias_u and bias_v unchanged;
- conv module: its BatchNorm (eps 1e-5) folded into the depthwise conv, per channel
  s = gamma / sqrt(running_var + eps): `conv.depthwise.weight` = w * s,
  `conv.depthwise.bias` = beta - running_mean * s (num_batches_tracked dropped);
- LSTM layer l: `weight_l{l}` = [W_ih | W_hh] side by side [2560, 1280],
  `bias_l{l}` = b_ih + b_hh;
- joint: the head's first `vocab` rows become the token head, padded to a multiple of
  64 rows with zero weights and -inf biases; the rows after them are the duration head;
- every other tensor unchanged.

The values have to equal tinybark's bit for bit (the same float32 operations), and
tensors are emitted in tinybark's order (the rewritten tensors layer by layer, then
the LSTM, then the joint, then the untouched tensors in their source order), so that
`save` writes the same cache file tinybark writes.

The on-disk form is tinybark's fp16 safetensors cache (tinybark/weights.py:92-120):
an 8-byte little-endian header length, a JSON header padded with spaces to a multiple
of 8 bytes, then every tensor as fp16 in header order.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Callable, Iterator, NamedTuple

import numpy as np

BN_EPS = 1e-5
VOCAB_ALIGN = 64


class Rule(NamedTuple):
    """Tensors `outputs` computed by `fn` from the source tensors `inputs`; `drop` names
    source tensors consumed without being used."""

    outputs: tuple[str, ...]
    inputs: tuple[str, ...]
    fn: Callable[..., tuple[np.ndarray, ...]]
    drop: tuple[str, ...] = ()


def _stack_rows(*mats: np.ndarray) -> tuple[np.ndarray]:
    return (np.concatenate(mats, axis=0),)


def _side_by_side(a: np.ndarray, b: np.ndarray) -> tuple[np.ndarray]:
    return (np.concatenate((a, b), axis=1),)


def _same(x: np.ndarray) -> tuple[np.ndarray]:
    return (x,)


def _sum(a: np.ndarray, b: np.ndarray) -> tuple[np.ndarray]:
    return (a + b,)


def _fold_batchnorm(w: np.ndarray, gamma, var, beta, mean) -> tuple[np.ndarray, np.ndarray]:
    s = gamma / np.sqrt(var + BN_EPS)
    return w * s[:, None, None], beta - mean * s


def _split_joint(vocab: int):
    def split(w: np.ndarray, b: np.ndarray):
        rows = -(-vocab // VOCAB_ALIGN) * VOCAB_ALIGN
        tok_w = np.zeros((rows, w.shape[1]), w.dtype)
        tok_w[:vocab] = w[:vocab]
        tok_b = np.full(rows, -np.inf, b.dtype)
        tok_b[:vocab] = b[:vocab]
        return tok_w, tok_b, w[vocab:], b[vocab:]

    return split


def rules(config: dict) -> Iterator[Rule]:
    """The conversion as rules, in the order their outputs appear in the layout."""
    for i in range(config["encoder_config"]["num_hidden_layers"]):
        att, conv = f"encoder.layers.{i}.self_attn.", f"encoder.layers.{i}.conv."
        yield Rule((att + "qkv",), tuple(att + f"{n}_proj.weight" for n in "qkv"), _stack_rows)
        for name in ("o_proj.weight", "relative_k_proj.weight", "bias_u", "bias_v"):
            yield Rule((att + name,), (att + name,), _same)
        yield Rule((conv + "depthwise.weight", conv + "depthwise.bias"),
                   tuple(conv + n for n in ("depthwise_conv.weight", "norm.weight", "norm.running_var", "norm.bias",
                                            "norm.running_mean")),
                   _fold_batchnorm, drop=(conv + "norm.num_batches_tracked",))
    lstm = "decoder.lstm."
    for l in range(config["num_decoder_layers"]):
        yield Rule((lstm + f"weight_l{l}",), (lstm + f"weight_ih_l{l}", lstm + f"weight_hh_l{l}"), _side_by_side)
        yield Rule((lstm + f"bias_l{l}",), (lstm + f"bias_ih_l{l}", lstm + f"bias_hh_l{l}"), _sum)
    yield Rule(("joint.token_head.weight", "joint.token_head.bias", "joint.duration_head.weight",
                "joint.duration_head.bias"), ("joint.head.weight", "joint.head.bias"), _split_joint(config["vocab_size"]))


def convert(sd: dict[str, np.ndarray], config: dict) -> dict[str, np.ndarray]:
    """Checkpoint-named float32 state dict to the converted layout. `sd` is not
    modified; a tensor a rule needs and `sd` lacks raises KeyError."""
    out: dict[str, np.ndarray] = {}
    used: set[str] = set()
    for rule in rules(config):
        values = rule.fn(*(sd[name] for name in rule.inputs))
        out.update(zip(rule.outputs, values))
        used.update(rule.inputs)
        used.update(rule.drop)
    for name, value in sd.items():
        if name not in used:
            out[name] = value
    return {name: np.ascontiguousarray(value) for name, value in out.items()}


def header(tensors: dict[str, np.ndarray]) -> bytes:
    """The safetensors header of `tensors` stored as fp16 in their order, padded with
    spaces to a multiple of 8 bytes."""
    entries, start = {}, 0
    for name, value in tensors.items():
        end = start + 2 * value.size
        entries[name] = {"dtype": "F16", "shape": list(value.shape), "data_offsets": [start, end]}
        start = end
    text = json.dumps(entries).encode()
    return text.ljust(-(-len(text) // 8) * 8, b" ")


def save(tensors: dict[str, np.ndarray], path: str | Path) -> None:
    """Writes `tensors` as tinybark's fp16 cache file, one tensor at a time."""
    head = header(tensors)
    with open(path, "wb") as f:
        f.write(np.uint64(len(head)).astype("<u8").tobytes())
        f.write(head)
        for value in tensors.values():
            np.asarray(value, "<f2").tofile(f)


def load(path: str | Path) -> dict[str, np.ndarray]:
    """Reads a converted cache file in one read (the pattern of
    tinybark/tinygrad/weights.py:10-26), returning float32 arrays."""
    data = Path(path).read_bytes()
    n = int.from_bytes(data[:8], "little")
    head = json.loads(data[8 : 8 + n])
    body = memoryview(data)[8 + n :]
    out = {}
    for name, info in head.items():
        if name == "__metadata__":
            continue
        if info["dtype"] not in ("F16", "F32"):
            raise ValueError(f"{name}: unsupported dtype {info['dtype']}")
        start, end = info["data_offsets"]
        dtype = np.float16 if info["dtype"] == "F16" else np.float32
        out[name] = np.frombuffer(body[start:end], dtype=dtype).reshape(info["shape"]).astype(np.float32)
    return out
