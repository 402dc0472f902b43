"""C++ CPU runtime vs the PyTorch fp32 reference (CPU)."""
import numpy as np
import pytest
import torch

from fak_b200.config import preset
from fak_b200.gguf.synth import write_synthetic_gguf
from fak_b200.models.reference import ReferenceModel

cpu = pytest.importorskip("fak_b200._cpu")


@pytest.mark.parametrize("name,mix", [("tiny-llama", "q8_0"), ("tiny-qwen2", "q4_k_m")])
def test_cpuref_matches_reference(tmp_path, name, mix):
    from fak_b200.models.cpu import load_cpu_model
    p = str(tmp_path / f"{name}.gguf")
    write_synthetic_gguf(p, preset(name), mix, seed=4, std=0.05)
    ref = ReferenceModel.from_gguf(p)
    exact, _ = load_cpu_model(p, act_quant=False)
    ids = np.random.default_rng(0).integers(0, preset(name).vocab_size, 20).tolist()
    want = ref.forward(torch.tensor(ids))
    exact.reset()
    for i, t in enumerate(ids):
        lg = torch.tensor(exact.step(t))
    assert torch.allclose(lg, want[-1], atol=1e-3, rtol=1e-3), (lg - want[-1]).abs().max()
    assert exact.generate(ids, 10) == ref.generate_greedy(ids, 10)
    fast, _ = load_cpu_model(p, act_quant=True)
    fast.reset()
    for t in ids:
        lf = torch.tensor(fast.step(t))
    cos = torch.nn.functional.cosine_similarity(lf, want[-1], dim=0).item()
    assert cos > 0.995, cos
