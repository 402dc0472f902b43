"""Token sampling: greedy, temperature, top-k, top-p, logit bias, frequency/presence penalties.

Semantics follow the reference's in-kernel sampler (internal/agent/inkernel_sampling.go:21-185):
penalties are applied to raw logits from the tokens generated so far, then temperature,
then top-k and top-p truncation; temperature 0 is greedy (first index of the max).
"""
from __future__ import annotations

import dataclasses

import torch

from .constraints import LogitMask, apply_constraint, guided_decode_enabled


@dataclasses.dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    logit_bias: dict[int, float] | None = None
    seed: int | None = None
    mask: LogitMask | None = None  # structural constraint; active only with guided decoding on

    @property
    def greedy(self) -> bool:
        """Plain argmax (the device-side greedy path): no bias, penalties or active mask."""
        return (self.temperature <= 0.0 and not self.logit_bias and self.frequency_penalty == 0.0
                and self.presence_penalty == 0.0 and not (self.mask is not None and guided_decode_enabled()))


def _apply_penalties(row: torch.Tensor, sp: SamplingParams, generated: list[int]) -> torch.Tensor:
    # mask (hard) then clamped logit bias (soft), then repetition penalties
    row = apply_constraint(row, sp.mask, sp.logit_bias, generated)
    if (sp.frequency_penalty or sp.presence_penalty) and generated:
        ids = torch.tensor(generated, device=row.device, dtype=torch.long)
        counts = torch.bincount(ids, minlength=row.numel()).to(row.dtype)
        row = row - sp.frequency_penalty * counts - sp.presence_penalty * (counts > 0).to(row.dtype)
    return row


def sample_row(row: torch.Tensor, sp: SamplingParams, generated: list[int]) -> int:
    row = _apply_penalties(row.float(), sp, generated)
    if sp.temperature <= 0.0:
        return int(torch.argmax(row))
    logits = row / sp.temperature
    if sp.top_k and sp.top_k < logits.numel():
        kth = torch.topk(logits, sp.top_k).values[-1]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    probs = torch.softmax(logits, dim=-1)
    if sp.top_p < 1.0:
        sp_, si = torch.sort(probs, descending=True)
        cum = torch.cumsum(sp_, dim=-1)
        cut = cum - sp_ > sp.top_p
        sp_ = sp_.masked_fill(cut, 0.0)
        probs = torch.zeros_like(probs).scatter_(0, si, sp_)
        probs = probs / probs.sum()
    gen = None
    if sp.seed is not None:
        gen = torch.Generator(device=row.device)
        gen.manual_seed(sp.seed + len(generated))
    return int(torch.multinomial(probs, 1, generator=gen))


def sample(logits: torch.Tensor, params: list[SamplingParams], reqs) -> list[int]:
    if all(p.greedy for p in params):
        return torch.argmax(logits, dim=-1).tolist()
    return [sample_row(logits[i], params[i], list(reqs[i].full_output)) for i in range(len(params))]
