"""Pipeline parallelism: the model's layers in contiguous bands, one band per rank.

* ``partition_layers`` -- balanced contiguous bands (the first ``n_layers % n_stages`` stages take
  one extra layer), the plan every rank derives identically;
* ``StageTransport`` -- hidden states between neighbouring stages over torch.distributed
  point-to-point (NCCL on GPUs, gloo on CPUs): a fixed-size header (rows, width, start position)
  followed by the fp32 payload;
* ``PipelineGreedy`` -- greedy generation through the pipeline: stage 0 embeds, every stage runs
  its band and forwards the residual stream, the last stage applies the final norm, LM head and
  argmax and broadcasts the token to all stages.  Each stage keeps the KV of its own layers.

The stage model is any object with ``embed(ids)``, ``forward_band(x, start_pos, l0, l1, kv)``,
``final(x) -> logits`` -- the fp32 reference model satisfies it, so a pipeline is checked
bit-for-bit against single-process decoding.

Reference: PartitionPlan / StageSpec (internal/model/pipeline.go:41-157), MarshalHidden (:159-222),
StageTransport with Local/TCP transports (:224-233, pipeline_transport.go:31-105) and the
incremental PipelineStageDecoder (pipeline.go:382-546).
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist


def partition_layers(n_layers: int, n_stages: int) -> list[tuple[int, int]]:
    if not 1 <= n_stages <= n_layers:
        raise ValueError(f"cannot split {n_layers} layers into {n_stages} stages")
    base, extra = divmod(n_layers, n_stages)
    bands, l0 = [], 0
    for s in range(n_stages):
        n = base + (1 if s < extra else 0)
        bands.append((l0, l0 + n))
        l0 += n
    return bands


@dataclasses.dataclass
class StageTransport:
    group: object = None

    def send(self, x: torch.Tensor, start_pos: int, dst: int) -> None:
        hdr = torch.tensor([x.shape[0], x.shape[1], start_pos], dtype=torch.int64, device=x.device)
        dist.send(hdr, dst, group=self.group)
        dist.send(x.float().contiguous(), dst, group=self.group)

    def recv(self, src: int, device) -> tuple[torch.Tensor, int]:
        hdr = torch.empty(3, dtype=torch.int64, device=device)
        dist.recv(hdr, src, group=self.group)
        T, d, pos = (int(v) for v in hdr.tolist())
        x = torch.empty(T, d, dtype=torch.float32, device=device)
        dist.recv(x, src, group=self.group)
        return x, pos


class ReferenceStageModel:
    """Adapts the fp32 reference model to a pipeline stage."""

    def __init__(self, ref):
        self.ref = ref
        self.cfg = ref.cfg

    def embed(self, ids):
        return self.ref.embed(torch.as_tensor(ids, dtype=torch.long, device=self.ref.device))

    def forward_band(self, x, start_pos, l0, l1, kv):
        return self.ref.forward_band(x, start_pos, l0, l1, kv)

    def final(self, x):
        from ..models.reference import rmsnorm
        return self.ref.lm_head(rmsnorm(x, self.ref.t["output_norm.weight"], self.cfg.rms_eps))


class PipelineGreedy:
    def __init__(self, model, rank: int, n_stages: int, group=None, ranks: list[int] | None = None):
        self.m = model
        self.rank, self.n = rank, n_stages
        self.ranks = ranks or list(range(n_stages))   # global rank of each stage
        self.band = partition_layers(model.cfg.n_layers, n_stages)[rank]
        self.tx = StageTransport(group)
        self.group = group
        self.kv: list = []

    def _step(self, ids: list[int], start_pos: int, device) -> int | None:
        """One pipeline pass over ``ids``; returns the greedy next token on every stage."""
        if self.rank == 0:
            x = self.m.embed(ids)
        else:
            x, start_pos = self.tx.recv(self.ranks[self.rank - 1], device)
        x = self.m.forward_band(x, start_pos, self.band[0], self.band[1], self.kv)
        tok = torch.zeros(1, dtype=torch.int64, device=device)
        if self.rank < self.n - 1:
            self.tx.send(x, start_pos, self.ranks[self.rank + 1])
        else:
            tok[0] = int(torch.argmax(self.m.final(x)[-1]))
        dist.broadcast(tok, self.ranks[-1], group=self.group)
        return int(tok[0])

    @torch.no_grad()
    def generate(self, prompt: list[int], n_new: int, device="cpu") -> list[int]:
        self.kv = []
        nxt = self._step(prompt, 0, device)
        out, pos = [], len(prompt)
        for _ in range(n_new):
            out.append(nxt)
            nxt = self._step([nxt], pos, device)
            pos += 1
        return out
