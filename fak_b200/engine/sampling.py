"""Token sampling: greedy, temperature, top-k, top-p, logit bias, frequency/presence penalties.

Semantics follow the reference's in-kernel sampler (internal/agent/inkernel_sampling.go:21-185):
penalties are applied to raw logits from the tokens generated so far, then temperature,
then top-k and top-p truncation; temperature 0 is greedy (first index of the max).

The serving path samples on the device (``csrc/kernels/sampler.cu``, one CTA per row inside the
decode graph): ``pack_params`` lays out each row's parameters and ``device_sample`` runs the kernel
on a block of logit rows (prefill's first tokens, the synchronous loop).  The draw of a request is
keyed by its seed and the number of tokens it has generated (Philox), so it does not depend on the
batch it runs in.  ``sample`` / ``sample_row`` are the host path kept for guided decoding (token
masks computed on the host).
"""
from __future__ import annotations

import dataclasses

import numpy as np
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


# ------------------------------------------------------------------------------ device sampler
MAX_BIAS = 4096      # logit-bias entries of one decode batch (all lanes together)


def request_seed(engine_seed: int, rid: int) -> int:
    """A 64-bit seed for a request without one (splitmix64 of the engine seed and the request id)."""
    z = (int(engine_seed) * 0x9E3779B97F4A7C15 + int(rid) + 0x632BE59BD9B4E019) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return z ^ (z >> 31)


def pack_params(sps: list[SamplingParams], steps: list[int], seeds: list[int], max_bias: int | None = MAX_BIAS
                ) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Rows of the device sampler's 10-word parameter block (temperature, top_k, top_p, frequency and
    presence penalty, bias offset / count, seed lo / hi, step) and the flat logit-bias lists
    (at most ``max_bias`` entries: the decode graph's static bias buffer; None = unbounded)."""
    n = len(sps)
    f = np.zeros((n, 10), np.float32)
    w = f.view(np.int32)
    tok: list[int] = []
    val: list[float] = []
    for b, (sp, st, sd) in enumerate(zip(sps, steps, seeds)):
        f[b, 0] = sp.temperature
        w[b, 1] = int(sp.top_k)
        f[b, 2] = sp.top_p
        f[b, 3] = sp.frequency_penalty
        f[b, 4] = sp.presence_penalty
        bias = sorted((sp.logit_bias or {}).items())
        w[b, 5] = len(tok)
        w[b, 6] = len(bias)
        tok += [int(t) for t, _ in bias]
        val += [float(v) for _, v in bias]
        w[b, 7] = np.uint32(sd & 0xFFFFFFFF).view(np.int32)
        w[b, 8] = np.uint32((sd >> 32) & 0xFFFFFFFF).view(np.int32)
        w[b, 9] = int(st)
    if max_bias is not None and len(tok) > max_bias:
        raise ValueError(f"logit_bias entries of one batch exceed {max_bias}")
    return w.copy(), np.asarray(tok, np.int32), np.asarray(val, np.float32)


def count_rows(generated: list[list[int]], V: int, device) -> torch.Tensor:
    """int32 [B, V]: how often each token appears in each row's generated tokens."""
    c = torch.zeros(len(generated), V, dtype=torch.int32, device=device)
    rows = [b for b, g in enumerate(generated) for _ in g]
    cols = [t for g in generated for t in g]
    if rows:
        c.index_put_((torch.tensor(rows, device=device), torch.tensor(cols, device=device)),
                     torch.ones(len(rows), dtype=torch.int32, device=device), accumulate=True)
    return c


def needs_counts(sps: list[SamplingParams]) -> bool:
    return any(sp.frequency_penalty != 0.0 or sp.presence_penalty != 0.0 for sp in sps)


def device_sample(logits: torch.Tensor, V: int, sps: list[SamplingParams], steps: list[int], seeds: list[int],
                  generated: list[list[int]], softcap: float = 0.0) -> list[int]:
    """Draw one token per row of ``logits`` [n, >=V] f32 on the device (the rows are modified)."""
    from ..ops import kernels as K
    dev = logits.device
    P, tok, val = pack_params(sps, steps, seeds, max_bias=None)   # own buffers: any size
    p = torch.from_numpy(P).to(dev)
    bt = torch.from_numpy(tok if len(tok) else np.full(1, -1, np.int32)).to(dev)
    bv = torch.from_numpy(val if len(val) else np.zeros(1, np.float32)).to(dev)
    counts = count_rows(generated, V, dev) if needs_counts(sps) else None
    out = torch.empty(len(sps), dtype=torch.int32, device=dev)
    K.sample_rows(logits, V, p, bt, bv, counts, out, len(sps), softcap)
    return out.tolist()
