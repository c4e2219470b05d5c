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
