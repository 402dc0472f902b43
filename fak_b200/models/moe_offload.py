"""MoE experts offloaded to host memory: their FFNs run on the CPU, everything else on the GPU.

The expert matrices are most of a MoE model's bytes but only the top-k of them fire per token, so
a model too large for the GPU can keep them in host RAM (in their GGML blocks, as loaded with
``load_weights(..., offload_experts=True)``) while the router, attention and every dense
projection stay on the device -- llama.cpp's ``--n-cpu-moe`` split.  Per MoE layer the device
routes the tokens (``moe_route``), normalises the residual rows, and the host copy of those rows
goes through ``fak_b200._cpu.CpuExperts`` (C++: int8 x int8 per 32-block for Q8_0 experts,
dequantize-and-dot otherwise, rows spread over a thread pool); the weighted sum comes back and is
added to the residual on the device.

The step synchronises with the host at every MoE layer, so decode runs without CUDA graphs; the
engine switches them off when experts are offloaded.  One GPU per replica (no tensor / expert
parallelism over the offloaded experts).

Reference: internal/model/moe_offload.go:25-125 (splitKernel: expert weights to the host kernel,
the rest to the device; ``isExpertWeight``), cmd/fak/serve.go ``--cpu-offload-experts``.
"""
from __future__ import annotations

import torch

from ..ops import kernels as K


def _host_rows(w) -> torch.Tensor:
    """The packed GGML rows of a host QuantWeight (its buffer without the row-pitch padding)."""
    from ..ops import quant as dq
    packed = dq.row_bytes(w.qtype, w.cols)
    return w.buf[: w.rows * w.pitch].view(w.rows, w.pitch)[:, :packed].contiguous()


class ExpertOffload:
    """Host-resident experts of every MoE layer of ``weights`` and the per-layer CPU expert FFN."""

    def __init__(self, weights, act_quant: bool = True):
        from .cpu import cpu_ext
        from .moe import _gate_epi
        cfg = weights.cfg
        self.cfg = cfg
        self.cx = cpu_ext().CpuExperts(cfg.n_layers, cfg.d_model, cfg.expert_ffn_dim, _gate_epi(cfg), act_quant)
        for i, L in enumerate(weights.layers):
            gu, dn = L.experts_gate_up, L.experts_down
            if gu is None:
                continue
            if gu.buf.is_cuda or dn.buf.is_cuda:
                raise ValueError("expert offload needs the experts loaded into host memory "
                                 "(load_weights(..., offload_experts=True))")
            bg = L.experts_gate_up_bias.float().contiguous() if L.experts_gate_up_bias is not None else None
            bd = L.experts_down_bias.float().contiguous() if L.experts_down_bias is not None else None
            self.cx.set_layer(i, L.expert_ids[0], len(L.expert_ids), _host_rows(gu), gu.qtype, _host_rows(dn),
                              dn.qtype, bg, bd)
        self.host_bytes = int(self.cx.bytes())

    def run(self, i: int, L, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor) -> None:
        """x[T, d] (device fp32, the residual) += the routed experts' outputs for its normalised rows."""
        cfg = self.cfg
        xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * L.ffn_norm
        xh, ih, wh = xn.cpu(), ids.cpu().contiguous(), wts.cpu().contiguous()
        out = torch.zeros_like(xh)
        self.cx.ffn(i, xh, ih, wh, out)
        x.add_(out.to(x.device, non_blocking=False))
        K.count()

    def decode(self, rn, i: int, B: int) -> None:
        """One decode layer's MoE block (the routing kernel on the device, the experts here)."""
        from .moe import _route, _state
        L, st = rn.w.layers[i], _state(rn)
        x = rn.x[:B]
        _route(rn, L, x, st.ids[:B], st.wts[:B])
        K.count()
        self.run(i, L, x, st.ids[:B], st.wts[:B])

    def prefill(self, rn, i: int, x: torch.Tensor) -> None:
        from .moe import _route
        L, k = rn.w.layers[i], self.cfg.n_experts_used
        ids = torch.empty(x.shape[0], k, dtype=torch.int32, device=x.device)
        wts = torch.empty(x.shape[0], k, dtype=torch.float32, device=x.device)
        _route(rn, L, x, ids, wts)
        K.count()
        self.run(i, L, x, ids, wts)
