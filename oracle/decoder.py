"""Oracle (test infrastructure only): the TDT prediction network, the joint and the
greedy loop, torch float32 on the CPU, on checkpoint-named weights.

- step: embedding, 2-layer LSTM (PyTorch gate order i, f, g, o), decoder_projector
  (tinybark/tinygrad/model.py:162-176; tinybark/ort/export.py:28-37).
- joint: ReLU(encoder frame + decoder output), the head's first 8193 rows are tokens
  and the last 5 durations, first index wins ties (tinybark/tinygrad/model.py:177-179;
  tinybark/ort/export.py:40-50; tinybark/mojo/bark/model.mojo:275-284).
- greedy: the loop of tinybark/tinygrad/model.py:196-233 = tinybark/ort/__init__.py:55-86.
"""

from __future__ import annotations

import numpy as np
import torch

from tinybark_b200 import lengths

BLANK, EOS, VOCAB = 8192, 3, 8193
DURATIONS = (0, 1, 2, 3, 4)


class Decoder:
    def __init__(self, sd, layers: int = 2):
        t = lambda n: torch.from_numpy(np.ascontiguousarray(sd[n], np.float32))
        self.layers = layers
        self.embedding = t("decoder.embedding.weight")
        self.w_ih = [t(f"decoder.lstm.weight_ih_l{l}") for l in range(layers)]
        self.w_hh = [t(f"decoder.lstm.weight_hh_l{l}") for l in range(layers)]
        self.b_ih = [t(f"decoder.lstm.bias_ih_l{l}") for l in range(layers)]
        self.b_hh = [t(f"decoder.lstm.bias_hh_l{l}") for l in range(layers)]
        self.proj_w, self.proj_b = t("decoder.decoder_projector.weight"), t("decoder.decoder_projector.bias")
        self.head_w, self.head_b = t("joint.head.weight"), t("joint.head.bias")
        self.hidden = self.proj_w.shape[0]

    def zero_state(self):
        z = torch.zeros(self.layers, self.hidden)
        return z.clone(), z.clone()

    @torch.inference_mode()
    def step(self, token: int, h: torch.Tensor, c: torch.Tensor):
        """One prediction-network step; returns (decoder output (640,), h, c)."""
        x = self.embedding[token]
        h, c = h.clone(), c.clone()
        for l in range(self.layers):
            gates = self.w_ih[l] @ x + self.b_ih[l] + self.w_hh[l] @ h[l] + self.b_hh[l]
            i, f, g, o = gates.chunk(4)
            c[l] = torch.sigmoid(f) * c[l] + torch.sigmoid(i) * torch.tanh(g)
            h[l] = torch.sigmoid(o) * torch.tanh(c[l])
            x = h[l]
        return self.proj_w @ x + self.proj_b, h, c

    @torch.inference_mode()
    def joint(self, encoded: torch.Tensor, decoded: torch.Tensor):
        """(token, duration index, top-2 token logit margin) for one encoder frame."""
        z = torch.relu(encoded + decoded)
        logits = self.head_w @ z + self.head_b
        tok = logits[:VOCAB]
        top = torch.topk(tok, 2).values
        return int(torch.argmax(tok)), int(torch.argmax(logits[VOCAB:])), float(top[0] - top[1])

    def greedy(self, encoded: np.ndarray, frames: int, margins: list | None = None) -> list[int]:
        """Greedy TDT decoding of one clip's projected encoder frames (T, 640), for a clip
        of `frames` feature frames (tinybark/tinygrad/model.py:218-234)."""
        enc = torch.from_numpy(np.ascontiguousarray(encoded, np.float32))
        valid = enc.shape[0]
        h, c = self.zero_state()
        decoded, h, c = self.step(BLANK, h, c)
        out, frame = [], 0
        for _ in range(lengths.decode_cap(frames)):
            if frame >= valid:
                break
            token, d, margin = self.joint(enc[frame], decoded)
            if margins is not None:
                margins.append(margin)
            duration = DURATIONS[d]
            if token == BLANK:
                frame += max(duration, 1)
                continue
            out.append(token)
            if token == EOS:
                break
            decoded, h, c = self.step(token, h, c)
            frame += duration
        return out


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


class BatchDecoder:
    """The greedy loop of `Decoder.greedy` for many clips at once (each lane runs the same
    loop on its own clip; lanes are independent), with each iteration's token and duration
    margins recorded: the gap between the largest and second largest of the 8193 token
    logits, and of the 5 duration logits.

    bf16=True restates the arithmetic of the bf16 decoder kernels instead of float32:
    weights rounded to bf16 (the embedding, both LSTM layers, the projector and the joint
    head; biases stay float32) and the GEMM inputs rounded to bf16 where the kernels store
    them (h0 and h1 after each cell, the joint input relu(enc + dec)); products, gates,
    cell states and logits in float32. It is the kernel's algorithm with its rounding
    points, not a bit-exact model of it (summation order and the activation functions'
    approximations differ), so its tokens equal the kernel's up to the first iteration
    whose margin is within those differences."""

    def __init__(self, sd, bf16: bool = False, layers: int = 2):
        r = _bf16 if bf16 else (lambda x: x)
        t = lambda n: torch.from_numpy(np.ascontiguousarray(sd[n], np.float32))
        self.bf16, self.layers = bf16, layers
        self.embedding = r(t("decoder.embedding.weight"))
        self.w_ih = [r(t(f"decoder.lstm.weight_ih_l{l}")) for l in range(layers)]
        self.w_hh = [r(t(f"decoder.lstm.weight_hh_l{l}")) for l in range(layers)]
        self.bias = [t(f"decoder.lstm.bias_ih_l{l}") + t(f"decoder.lstm.bias_hh_l{l}") for l in range(layers)]
        self.proj_w, self.proj_b = r(t("decoder.decoder_projector.weight")), t("decoder.decoder_projector.bias")
        self.head_w, self.head_b = r(t("joint.head.weight")), t("joint.head.bias")
        self.hidden = self.proj_w.shape[0]
        self._round = r

    def _step(self, tokens: torch.Tensor, h: torch.Tensor, c: torch.Tensor):
        """Prediction-network step for lanes with the given tokens: (dec, h, c), h and c
        [layers, lanes, hidden]; h as the kernels store it (bf16-rounded in bf16 mode)."""
        x = self.embedding[tokens]
        h, c = h.clone(), c.clone()
        for l in range(self.layers):
            gates = x @ self.w_ih[l].T + h[l] @ self.w_hh[l].T + self.bias[l]
            i, f, g, o = gates.chunk(4, dim=1)
            c[l] = torch.sigmoid(f) * c[l] + torch.sigmoid(i) * torch.tanh(g)
            h[l] = self._round(torch.sigmoid(o) * torch.tanh(c[l]))
            x = h[l]
        return x @ self.proj_w.T + self.proj_b, h, c

    @torch.inference_mode()
    def greedy(self, encoded: list[np.ndarray], frames: list[int]):
        """Greedy TDT decoding of every clip (projected encoder frames (T_i, 640), feature
        frames F_i). Returns (tokens per clip, per clip a list of (tokens emitted before
        the iteration, token margin, duration margin) for each iteration run)."""
        n = len(encoded)
        valid = torch.tensor([len(e) for e in encoded])
        cap = torch.tensor([lengths.decode_cap(f) for f in frames])
        width = int(valid.max()) if n else 0
        enc = torch.zeros(n, max(width, 1), self.hidden)
        for i, e in enumerate(encoded):
            enc[i, : len(e)] = torch.from_numpy(np.ascontiguousarray(e, np.float32))
        h = torch.zeros(self.layers, n, self.hidden)
        c = torch.zeros(self.layers, n, self.hidden)
        dec, h, c = self._step(torch.full((n,), BLANK, dtype=torch.long), h, c)
        frame = torch.zeros(n, dtype=torch.long)
        running = (valid > 0) & (cap > 0)
        out: list[list[int]] = [[] for _ in range(n)]
        trace: list[list[tuple[int, float, float]]] = [[] for _ in range(n)]
        durations = torch.tensor(DURATIONS)
        it = 0
        while bool(running.any()):
            running &= (it < cap) & (frame < valid)
            lanes = torch.nonzero(running).flatten()
            if len(lanes) == 0:
                break
            z = self._round(torch.relu(enc[lanes, frame[lanes]] + dec[lanes]))
            logits = z @ self.head_w.T + self.head_b
            tok_top = torch.topk(logits[:, :VOCAB], 2)
            dur_top = torch.topk(logits[:, VOCAB:], 2)
            tok = tok_top.indices[:, 0]
            dur = durations[dur_top.indices[:, 0]]
            tm = (tok_top.values[:, 0] - tok_top.values[:, 1]).tolist()
            dm = (dur_top.values[:, 0] - dur_top.values[:, 1]).tolist()
            emit = []
            for j, lane in enumerate(lanes.tolist()):
                trace[lane].append((len(out[lane]), tm[j], dm[j]))
                t = int(tok[j])
                if t == BLANK:
                    frame[lane] += max(int(dur[j]), 1)
                    continue
                out[lane].append(t)
                if t == EOS:
                    running[lane] = False
                    continue
                emit.append((lane, t, int(dur[j])))
            if emit:
                idx = torch.tensor([e[0] for e in emit])
                d2, h2, c2 = self._step(torch.tensor([e[1] for e in emit]), h[:, idx], c[:, idx])
                dec[idx], h[:, idx], c[:, idx] = d2, h2, c2
                frame[idx] += torch.tensor([e[2] for e in emit])
            it += 1
        return out, trace


def agreement(got: list[int], want: list[int], trace: list[tuple[int, float, float]], bound: float):
    """Compares a kernel's tokens for one clip with the oracle's: (tokens that must agree,
    tokens that agree, margin at the first iteration below `bound` or None). The tokens
    that must agree are those the oracle emitted before its first iteration whose token or
    duration margin is below `bound` (all of them if there is none)."""
    must, low = len(want), None
    for emitted, tm, dm in trace:
        if min(tm, dm) < bound:
            must, low = emitted, min(tm, dm)
            break
    same = 0
    for a, b in zip(got, want):
        if a != b:
            break
        same += 1
    if low is None and len(got) != len(want):
        same = min(same, must - 1)
    return must, same, low
