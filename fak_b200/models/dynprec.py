"""Dynamic precision on the reference path: try the quantized forward, keep it only when confident.

A ``DynamicPrecisionSession`` holds one model twice: in fp32 and with every 2-D weight rounded
through Q8_0.  Each prefill or decode step first runs the Q8_0 model; its last-position logits are
accepted when the top-1 logit leads the runner-up by at least ``min_margin`` (raw logit units) and
the top-1 softmax probability is at least ``min_prob`` (0 disables either test).  A rejected step
is discarded -- the KV cache is restored to its state before the step -- and the same tokens are
recomputed in fp32.  ``stats`` counts the tokens and decisions per tier.

With both thresholds at 0 every Q8_0 step is accepted (a fixed Q8_0 session, with stats).

Reference: internal/model/dynamic_precision.go (PrecisionTier, DynamicPrecisionPolicy margin /
probability gates, Q8-attempt then roll back and recompute in f32, PrecisionStats).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from ..gguf.quants import dequantize_q8_0, quantize_q8_0
from .reference import ReferenceModel


def q8_0_round(t: torch.Tensor) -> torch.Tensor:
    """A weight matrix as the Q8_0 blocks would hold it (rows of a multiple of 32)."""
    a = t.detach().to("cpu", torch.float32).numpy()
    out = dequantize_q8_0(quantize_q8_0(a.reshape(-1))).reshape(a.shape).astype(np.float32)
    return torch.from_numpy(out)


@dataclasses.dataclass
class PrecisionStats:
    q8_tokens: int = 0
    f32_tokens: int = 0
    accepted: int = 0
    rejected: int = 0
    last_margin: float = 0.0
    last_prob: float = 0.0


class DynamicPrecisionSession:
    def __init__(self, model: ReferenceModel, min_margin: float = 0.0, min_prob: float = 0.0):
        self.f32 = model
        tq = {k: (q8_0_round(v) if v.dim() == 2 and v.shape[-1] % 32 == 0 else v) for k, v in model.t.items()}
        self.q8 = ReferenceModel(model.cfg, tq, model.device)
        self.min_margin, self.min_prob = float(min_margin), float(min_prob)
        self.kv: list = []
        self.pos = 0
        self.stats = PrecisionStats()

    def accepts(self, margin: float, prob: float) -> bool:
        return (self.min_margin <= 0 or margin >= self.min_margin) and (self.min_prob <= 0 or prob >= self.min_prob)

    @torch.no_grad()
    def run(self, ids) -> torch.Tensor:
        """Prefill or decode ``ids`` at the session's position; returns the last position's logits."""
        ids = torch.as_tensor(ids, dtype=torch.long).reshape(-1)
        saved = [tuple(t.clone() for t in layer) for layer in self.kv]
        logits = self.q8.forward(ids, self.pos, self.kv)[-1]
        top = torch.topk(logits, 2).values
        margin = float(top[0] - top[1])
        prob = float(torch.softmax(logits, -1).max())
        self.stats.last_margin, self.stats.last_prob = margin, prob
        if self.accepts(margin, prob):
            self.stats.accepted += 1
            self.stats.q8_tokens += ids.numel()
        else:
            self.stats.rejected += 1
            self.kv[:] = saved                       # roll back the Q8_0 step's keys and values
            logits = self.f32.forward(ids, self.pos, self.kv)[-1]
            self.stats.f32_tokens += ids.numel()
        self.pos += ids.numel()
        return logits

    def generate_greedy(self, prompt: list[int], n_new: int) -> list[int]:
        out = []
        logits = self.run(prompt)
        for _ in range(n_new):
            t = int(torch.argmax(logits))
            out.append(t)
            logits = self.run([t])
        return out
