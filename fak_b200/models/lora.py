"""LoRA adapters: low-rank weight deltas, merged into the weights at load or applied per step.

A PEFT adapter patches a linear weight W [out, in] with factors A [r, in] and B [out, r]:
dW = (alpha / r) B A (alpha / sqrt(r) with rsLoRA), so y = W x + dW x.  Adapters on the same weight
compose additively, and a ``LoRASet`` switches named bundles on and off.

* merge (``merged_source``): the device weights are dequantized, patched and re-encoded in their own
  block type once at load, so decoding runs the unmodified kernels -- zero per-token overhead for
  one pinned adapter set;
* dynamic (``LoRASet.delta``, used by the fp32 reference model): the factors stay separate and the
  delta ``scale * (x A^T) B^T`` is added after each patched projection, so bundles switch without
  reloading, at r (in + out) / (in out) extra multiply-adds per weight.

Adapter files: ``adapter_config.json`` (r, lora_alpha, target_modules, peft_type, use_rslora) and
``adapter_model.safetensors`` with ``base_model.model.<module>.lora_A.weight`` / ``lora_B.weight``.

Reference: LoRAAdapter / LoRASet / MergeLoRA / LoadLoRAAdapter (internal/model/lora.go:67-476).
"""
from __future__ import annotations

import dataclasses
import json
import math
import os

import numpy as np
import torch

from ..gguf import GGMLType


@dataclasses.dataclass
class LoRAAdapter:
    target: str               # weight name in the GGUF namespace (blk.{i}.attn_q.weight, ...)
    A: torch.Tensor           # [r, in]
    B: torch.Tensor           # [out, r]
    alpha: float
    bundle: str = "default"
    rslora: bool = False

    def __post_init__(self) -> None:
        if self.A.dim() != 2 or self.B.dim() != 2 or self.A.shape[0] != self.B.shape[1]:
            raise ValueError(f"lora {self.bundle}:{self.target}: factor shapes A{tuple(self.A.shape)} "
                             f"B{tuple(self.B.shape)} do not chain")
        self.A = self.A.float()
        self.B = self.B.float()

    @property
    def rank(self) -> int:
        return int(self.A.shape[0])

    @property
    def scaling(self) -> float:
        return self.alpha / (math.sqrt(self.rank) if self.rslora else self.rank)

    def delta(self, x: torch.Tensor) -> torch.Tensor:
        return ((x.float() @ self.A.to(x.device).T) @ self.B.to(x.device).T) * self.scaling

    def delta_weight(self) -> torch.Tensor:
        return (self.B @ self.A) * self.scaling

    def overhead_fraction(self) -> float:
        out_, in_ = self.B.shape[0], self.A.shape[1]
        return self.rank * (in_ + out_) / (in_ * out_)


class LoRASet:
    def __init__(self) -> None:
        self.adapters: list[LoRAAdapter] = []
        self.active: dict[str, bool] = {}

    def add(self, a: LoRAAdapter) -> None:
        for b in self.adapters:
            if b.bundle == a.bundle and b.target == a.target:
                raise ValueError(f"lora {a.bundle}: duplicate adapter for {a.target}")
        self.adapters.append(a)
        self.active.setdefault(a.bundle, True)

    def activate(self, bundle: str) -> None:
        self.active[bundle] = True

    def deactivate(self, bundle: str) -> None:
        self.active[bundle] = False

    def bundles(self) -> list[str]:
        return sorted(self.active)

    def targets(self) -> list[str]:
        return sorted({a.target for a in self.adapters if self.active.get(a.bundle)})

    def active_for(self, target: str) -> list[LoRAAdapter]:
        return [a for a in self.adapters if a.target == target and self.active.get(a.bundle)]

    def delta(self, target: str, x: torch.Tensor) -> torch.Tensor | None:
        out = None
        for a in self.active_for(target):
            d = a.delta(x)
            out = d if out is None else out + d
        return out

    def merge_into(self, target: str, w: torch.Tensor) -> torch.Tensor:
        """w [out, in] + the sum of the active deltas of ``target`` (a new tensor)."""
        w = w.float().clone()
        for a in self.active_for(target):
            if tuple(a.delta_weight().shape) != tuple(w.shape):
                raise ValueError(f"lora {a.bundle}:{target}: delta {tuple(a.delta_weight().shape)} "
                                 f"does not match the weight {tuple(w.shape)}")
            w += a.delta_weight().to(w.device)
        return w


def load_peft_adapter(path: str, lora_set: LoRASet | None = None, bundle: str | None = None) -> LoRASet:
    """Read a PEFT LoRA adapter directory into ``lora_set`` (a new set when None)."""
    from .hf import _to_f32, gguf_name, read_safetensors
    s = lora_set if lora_set is not None else LoRASet()
    with open(os.path.join(path, "adapter_config.json")) as f:
        cfg = json.load(f)
    r = int(cfg.get("r", 0))
    if r <= 0:
        raise ValueError(f"lora {path}: adapter_config.json has r={r}")
    if str(cfg.get("peft_type", "LORA")).upper() != "LORA":
        raise ValueError(f"lora {path}: peft_type {cfg.get('peft_type')!r} is not LORA")
    alpha = float(cfg.get("lora_alpha") or r)
    rslora = bool(cfg.get("use_rslora", False))
    name = bundle or os.path.basename(os.path.normpath(path))
    pairs: dict[str, dict[str, torch.Tensor]] = {}
    for n, (dt, shape, arr) in read_safetensors(os.path.join(path, "adapter_model.safetensors")).items():
        base = n[len("base_model.model."):] if n.startswith("base_model.model.") else n
        for kind in ("lora_A", "lora_B"):
            suf = f".{kind}.weight"
            if base.endswith(suf):
                t = torch.from_numpy(_to_f32(dt, np.asarray(arr)).reshape(shape).copy())
                pairs.setdefault(base[: -len(suf)] + ".weight", {})[kind] = t
    if not pairs:
        raise ValueError(f"lora {path}: no lora_A / lora_B tensors")
    for hf_name, ab in sorted(pairs.items()):
        if set(ab) != {"lora_A", "lora_B"}:
            raise ValueError(f"lora {path}: {hf_name} is missing a factor")
        target = gguf_name(hf_name)
        if target is None:
            raise ValueError(f"lora {path}: no model weight for {hf_name}")
        s.add(LoRAAdapter(target, ab["lora_A"], ab["lora_B"], alpha, name, rslora))
    return s


def merged_source(source, lora_set: LoRASet):
    """Wrap a (config, getter, close) weight source so patched matrices come back merged and
    re-encoded in their own block type (Q8_0 when the type has no encoder)."""
    from ..gguf.quants import _QUANT, dequantize, quantize
    cfg, get, close = source
    targets = set(lora_set.targets())

    def get2(name: str):
        shape, t, raw = get(name)
        if name not in targets:
            return shape, t, raw
        w = torch.from_numpy(dequantize(raw.cpu().numpy().reshape(-1), t, tuple(shape)).astype(np.float32))
        w = lora_set.merge_into(name, w).numpy()
        t2 = t if (GGMLType(t) in _QUANT or t in (GGMLType.F32, GGMLType.F16, GGMLType.BF16)) else GGMLType.Q8_0
        if t2 == GGMLType.G4:
            t2 = GGMLType.Q8_0   # a merged delta breaks the checkpoint's groups: keep 8-bit precision
        enc = quantize(w, t2)
        return shape, int(t2), torch.from_numpy(enc.reshape(shape[0], -1))

    return cfg, get2, close
