"""GGUF container, block formats and synthetic checkpoints (CPU)."""
import numpy as np
import pytest

from fak_b200.config import config_from_gguf_metadata, preset
from fak_b200.gguf import GGMLType, GGUFError, GGUFWriter, open_gguf
from fak_b200.gguf import quants as Q
from fak_b200.gguf.synth import choose_type, use_more_bits, write_synthetic_gguf


@pytest.mark.parametrize("qt,tol", [(GGMLType.Q8_0, 0.01), (GGMLType.Q4_K, 0.12), (GGMLType.Q6_K, 0.05)])
def test_quant_roundtrip(qt, tol):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((16, 512)) * 0.02).astype(np.float32)
    raw = Q.quantize(x, qt)
    y = Q.dequantize(raw, qt).reshape(x.shape)
    assert np.abs(y - x).max() <= tol * np.abs(x).max()
    assert raw.size == x.size // Q.BLOCK_INFO[qt][0] * Q.BLOCK_INFO[qt][1]


def test_q4k_layout_known_block():
    # one super-block with a ramp: element e has value e; min-offset scheme must decode back closely
    x = (np.arange(256, dtype=np.float32) - 128) / 256.0
    raw = Q.quantize_q4_k(x)
    assert raw.size == 144
    y = Q.dequantize_q4_k(raw)
    # each 32-wide sub-block spans [min(x, 0), max(x)] in 15 steps
    assert np.abs(y - x).max() <= 0.5 / 15 + 1e-3
    assert np.corrcoef(x, y)[0, 1] > 0.999
    # scale/min packing is invertible for all 6-bit values
    sc = np.arange(8)[None, :] * 9 % 64
    mn = (np.arange(8)[None, :] * 7 + 3) % 64
    s2, m2 = Q.unpack_scale_min_k4(Q.pack_scale_min_k4(sc, mn))
    assert (s2 == sc).all() and (m2 == mn).all()


def test_q6k_signed_scales_and_offsets():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(512).astype(np.float32)
    raw = Q.quantize_q6_k(x).reshape(2, 210)
    sc = raw[:, 192:208].view(np.int8)
    assert (sc < 0).any()  # scales carry the sign of each sub-block's extreme value
    assert np.abs(Q.dequantize_q6_k(raw.reshape(-1)) - x).max() < 0.1


def test_legacy_dequant_shapes():
    rng = np.random.default_rng(2)
    for qt, nbytes in [(GGMLType.Q4_0, 18), (GGMLType.Q4_1, 20), (GGMLType.Q5_0, 22), (GGMLType.Q5_1, 24),
                       (GGMLType.Q2_K, 84), (GGMLType.Q5_K, 176)]:
        blk = Q.BLOCK_INFO[qt][0]
        raw = rng.integers(0, 255, size=4 * nbytes, dtype=np.uint8)
        # keep f16 scales finite
        out = Q.dequantize(raw, qt)
        assert out.shape == (4 * blk,)


def test_writer_reader_roundtrip(tmp_path):
    p = tmp_path / "t.gguf"
    w = GGUFWriter(str(p), arch="llama")
    w.add("llama.block_count", 3)
    w.add("general.name", "x")
    w.add("tokenizer.ggml.tokens", ["a", "b", "c"])
    w.add("some.floats", [1.0, 2.5])
    a = np.arange(64, dtype=np.float32).reshape(2, 32)
    w.add_tensor("a", (2, 32), GGMLType.F32, a)
    q = Q.quantize((np.arange(64, dtype=np.float32) / 64).reshape(2, 32), GGMLType.Q8_0)
    w.add_tensor("b", (2, 32), GGMLType.Q8_0, lambda: q)
    w.write()
    g = open_gguf(str(p))
    assert g.metadata["llama.block_count"] == 3
    assert g.metadata["tokenizer.ggml.tokens"] == ["a", "b", "c"]
    assert g.metadata["some.floats"] == [1.0, 2.5]
    assert g.tensors["a"].shape == (2, 32)
    np.testing.assert_array_equal(g.dequantize("a"), a)
    assert g.raw("b").tobytes() == q.tobytes()
    assert g.tensors["b"].offset % 32 == 0


def test_reader_rejects_garbage(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOTGGUF" + b"\0" * 64)
    with pytest.raises(GGUFError):
        open_gguf(str(p))
    p.write_bytes(b"GGUF")
    with pytest.raises(GGUFError):
        open_gguf(str(p))


def test_q4_k_m_mix_rules():
    cfg = preset("qwen2.5-7b")
    assert choose_type(cfg, "output.weight", (152064, 3584), "output", "q4_k_m") == GGMLType.Q6_K
    assert choose_type(cfg, "blk.0.attn_q.weight", (3584, 3584), "attn_q", "q4_k_m") == GGMLType.Q4_K
    assert choose_type(cfg, "blk.0.attn_v.weight", (512, 3584), "attn_v", "q4_k_m") == GGMLType.Q6_K
    n = cfg.n_layers
    picked = [i for i in range(n) if use_more_bits(i, n)]
    assert 0 in picked and n - 1 in picked and len(picked) < n
    assert choose_type(cfg, "blk.0.attn_norm.weight", (3584,), "norm", "q4_k_m") == GGMLType.F32


@pytest.mark.parametrize("name,mix", [("tiny-llama", "q8_0"), ("tiny-qwen2", "q4_k_m"), ("tiny-qwen3moe", "q8_0")])
def test_synthetic_checkpoint_config_roundtrip(tmp_path, name, mix):
    cfg = preset(name)
    p = str(tmp_path / f"{name}.gguf")
    write_synthetic_gguf(p, cfg, mix, seed=1)
    g = open_gguf(p)
    got = config_from_gguf_metadata(g.metadata, {k: v.shape for k, v in g.tensors.items()})
    assert got == cfg
    assert len(g.metadata["tokenizer.ggml.tokens"]) == cfg.vocab_size


def test_split_files(tmp_path):
    for i in (1, 2):
        w = GGUFWriter(str(tmp_path / f"m-0000{i}-of-00002.gguf"), arch="llama")
        w.add_tensor(f"t{i}", (32,), GGMLType.F32, np.full(32, i, np.float32))
        w.write()
    g = open_gguf(str(tmp_path / "m-00001-of-00002.gguf"))
    assert set(g.tensors) == {"t1", "t2"}
    assert g.dequantize("t2")[0] == 2
