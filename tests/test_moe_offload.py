"""Host-resident MoE experts (``fak_b200._cpu.CpuExperts``, the CPU side of the expert offload)
against an fp32 PyTorch reference of the same routed expert FFN."""
import numpy as np
import pytest
import torch

from fak_b200.gguf import quants as Q
from fak_b200.gguf.constants import GGMLType

cpu = pytest.importorskip("fak_b200._cpu")


def _experts(qt, E, d, f, seed):
    from fak_b200.models.weights import interleave_gate_up
    rng = np.random.default_rng(seed)
    gate = (rng.standard_normal((E, f, d)) * 0.05).astype(np.float32)
    up = (rng.standard_normal((E, f, d)) * 0.05).astype(np.float32)
    down = (rng.standard_normal((E, d, f)) * 0.05).astype(np.float32)

    def q(a):   # quantized rows and their dequantized values
        raw = Q.quantize(a.reshape(-1, a.shape[-1]), qt).reshape(a.shape[0] * a.shape[1], -1)
        deq = Q.dequantize(raw.reshape(-1), qt).reshape(a.shape)
        return torch.from_numpy(raw), torch.from_numpy(deq)
    g_raw, g = q(gate)
    u_raw, u = q(up)
    d_raw, dn = q(down)
    gu_raw = torch.cat([interleave_gate_up(g_raw[e * f:(e + 1) * f], u_raw[e * f:(e + 1) * f]) for e in range(E)])
    return gu_raw.contiguous(), d_raw.contiguous(), g, u, dn


def _reference(x, ids, wts, g, u, dn, e0, n, gate):
    out = torch.zeros_like(x, dtype=torch.float64)
    for b in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[b, j])
            if not e0 <= e < e0 + n:
                continue
            gv, uv = g[e].double() @ x[b].double(), u[e].double() @ x[b].double()
            h = torch.nn.functional.silu(gv) * uv if gate == 2 else \
                torch.nn.functional.gelu(gv, approximate="tanh") * uv
            out[b] += float(wts[b, j]) * (dn[e].double() @ h)
    return out.float()


@pytest.mark.parametrize("qt", [GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K])
@pytest.mark.parametrize("gate", [2, 3])
def test_cpu_experts_match_reference(qt, gate):
    E, d, f, B, k = 4, 256, 512, 5, 2
    gu_raw, d_raw, g, u, dn = _experts(qt, E, d, f, seed=int(qt) + gate)
    x = torch.randn(B, d, generator=torch.Generator().manual_seed(1))
    ids = torch.tensor([[0, 3], [1, 2], [3, 3], [2, 0], [1, 1]], dtype=torch.int32)
    wts = torch.rand(B, k, generator=torch.Generator().manual_seed(2))
    cx = cpu.CpuExperts(1, d, f, gate, False)   # fp32 activations: dequantize-and-dot
    cx.set_layer(0, 0, E, gu_raw, int(qt), d_raw, int(qt))
    out = torch.zeros(B, d)
    cx.ffn(0, x, ids, wts, out)
    ref = _reference(x, ids, wts, g, u, dn, 0, E, gate)
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-5), (out - ref).abs().max()
    again = torch.zeros(B, d)
    cx.ffn(0, x, ids, wts, again)
    assert torch.equal(out, again)


def test_cpu_experts_band_and_int8_path():
    """A rank's band [e0, e0 + n) adds only its own experts' slots; Q8_0 experts with int8
    activations stay within int8 rounding of the fp32 result."""
    E, d, f, B = 4, 256, 256, 3
    gu_raw, d_raw, g, u, dn = _experts(GGMLType.Q8_0, E, d, f, seed=7)
    x = torch.randn(B, d, generator=torch.Generator().manual_seed(3))
    ids = torch.tensor([[0, 2], [3, 1], [2, 3]], dtype=torch.int32)
    wts = torch.tensor([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5]])
    rows_gu, rows_dn = 2 * f, d
    cx = cpu.CpuExperts(2, d, f, 2, False)
    cx.set_layer(1, 2, 2, gu_raw[2 * rows_gu:].contiguous(), 8, d_raw[2 * rows_dn:].contiguous(), 8)
    out = torch.zeros(B, d)
    cx.ffn(1, x, ids, wts, out)
    ref = _reference(x, ids, wts, g, u, dn, 2, 2, 2)
    assert torch.allclose(out, ref, rtol=1e-4, atol=1e-5)
    assert torch.all(out[0] != 0) and torch.all(out[1] != 0)
    cq = cpu.CpuExperts(1, d, f, 2, True)
    cq.set_layer(0, 0, E, gu_raw, 8, d_raw, 8)
    outq = torch.zeros(B, d)
    cq.ffn(0, x, ids, wts, outq)
    full = _reference(x, ids, wts, g, u, dn, 0, E, 2)
    assert float((outq - full).norm() / full.norm()) < 2e-2


def test_cpu_experts_rejects_bad_shapes():
    cx = cpu.CpuExperts(1, 256, 256, 2, True)
    with pytest.raises(RuntimeError):
        cx.set_layer(0, 0, 2, torch.zeros(10, dtype=torch.uint8), 8, torch.zeros(10, dtype=torch.uint8), 8)
    with pytest.raises(RuntimeError):
        cpu.CpuExperts(1, 256, 256, 7, True)
