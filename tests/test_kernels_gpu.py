"""Numerics of the sm_100a kernels against plain fp32 PyTorch references (GPU only)."""
import math

import numpy as np
import pytest
import torch

from fak_b200.gguf import quants as Q
from fak_b200.gguf.constants import GGMLType

pytestmark = pytest.mark.gpu

QTYPES = [(GGMLType.Q8_0, 32), (GGMLType.Q4_K, 256), (GGMLType.Q6_K, 256)]
# G4 (AWQ / GPTQ group-int4) runs only tile-packed (tgemv) and through the dequantizer
QTYPES_TILE = QTYPES + [(GGMLType.G4, 256)]


def _ext():
    from fak_b200.ops._ext import ext
    return ext()


def _swiglu_ref(y, gelu: bool = False):
    """SwiGLU (or GEGLU with GELU-tanh) over 8-row interleaved (gate x8, up x8) blocks of the output dim."""
    M, N = y.shape
    blocks = y.view(M, N // 16, 2, 8)
    g = blocks[:, :, 0]
    a = torch.nn.functional.gelu(g, approximate="tanh") if gelu else torch.nn.functional.silu(g)
    return (a * blocks[:, :, 1]).reshape(M, N // 2)


@pytest.mark.parametrize("qt,blk", QTYPES_TILE)
def test_quantize_matches_numpy_bitexact(qt, blk):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((64, 4 * 256)) * 0.02).astype(np.float32)
    ref = Q.quantize(x, qt)
    got = _ext().quantize_blocks(torch.from_numpy(x).cuda().reshape(-1), int(qt)).cpu().numpy()
    assert got.shape == ref.shape
    match = (got == ref).mean()
    # same format, same decoded values up to one quantization step
    dg, dr = Q.dequantize(got, qt), Q.dequantize(ref, qt)
    step = np.abs(x).max() / (127 if qt == GGMLType.Q8_0 else 15)
    assert np.abs(dg - dr).max() <= step, match
    assert match > 0.9, match


@pytest.mark.parametrize("qt,blk", QTYPES_TILE)
def test_dequantize_rows(qt, blk):
    from fak_b200.ops import quant as dq
    rng = np.random.default_rng(2)
    rows, cols = 48, 3 * 256
    x = (rng.standard_normal((rows, cols)) * 0.05).astype(np.float32)
    raw = Q.quantize(x, qt).reshape(rows, -1)
    from fak_b200.models.weights import QuantWeight
    w = QuantWeight.from_rows(torch.from_numpy(raw), int(qt), cols, torch.device("cuda"))
    ref = Q.dequantize(raw.reshape(-1), qt).reshape(rows, cols)
    got = w.dense(torch.float32, cache=False).cpu().numpy()
    np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)
    gotb = w.dense(torch.bfloat16, cache=False).float().cpu().numpy()
    np.testing.assert_allclose(gotb, ref, rtol=1e-2, atol=1e-3)


@pytest.mark.parametrize("qt,blk", QTYPES)
@pytest.mark.parametrize("B", [1, 3, 5, 8])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_qgemv(qt, blk, B, epi):
    from fak_b200.models.weights import QuantWeight
    from fak_b200.ops import kernels as K
    torch.manual_seed(0)
    N, Kd = 512 + 64, 1024 if qt != GGMLType.Q8_0 else 576
    rng = np.random.default_rng(3)
    Wf = (rng.standard_normal((N, Kd)) * 0.05).astype(np.float32)
    raw = Q.quantize(Wf, qt).reshape(N, -1)
    w = QuantWeight.from_rows(torch.from_numpy(raw), int(qt), Kd, torch.device("cuda"))
    Wd = torch.from_numpy(Q.dequantize(raw.reshape(-1), qt).reshape(N, Kd)).cuda()
    x = torch.randn(B, Kd, device="cuda")
    act = K.ActQ(8, Kd, "cuda")
    K.quant_act(x, act)
    bias = torch.randn(N, device="cuda") * 0.1
    ref = x @ Wd.T + bias
    if epi == K.EPI_SWIGLU:
        ref = _swiglu_ref(ref)
        y = torch.zeros(B, N // 2, device="cuda")
    else:
        y = torch.randn(B, N, device="cuda")
        if epi == K.EPI_ADD:
            ref = ref + y
    K.gemv(w, act, B, y, bias, epi)
    torch.cuda.synchronize()
    err = (y - ref).abs().max().item() / ref.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
    # SwiGLU multiplies two int8-activation dot products, which roughly doubles the relative error
    tol_cos, tol_err = (0.999, 0.06) if epi == K.EPI_SWIGLU else (0.9995, 0.03)
    assert cos > tol_cos and err < tol_err, (cos, err)


def test_quant_act_rmsnorm():
    from fak_b200.ops import kernels as K
    x = torch.randn(4, 512, device="cuda") * 3
    g = torch.rand(512, device="cuda") + 0.5
    act = K.ActQ(4, 512, "cuda")
    K.quant_act(x, act, g, 1e-6)
    xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * g
    deq = act.q.float().view(4, 16, 32) * act.ds[:, :, 0:1]
    assert torch.allclose(deq.view(4, 512), xn, atol=xn.abs().max().item() / 127 * 0.51 + 1e-6)
    # the sum is that of the dequantized values (consistent with the int8 dot products)
    assert torch.allclose(act.ds[:, :, 1], deq.sum(-1), atol=1e-4)


def _paged_cache(ctx_lens, Hkv, D, n_pages=256, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(n_pages - 1, generator=torch.Generator().manual_seed(seed)) + 1
    bts, used = [], 0
    for L in ctx_lens:
        n = math.ceil(L / 16)
        bts.append(perm[used:used + n].tolist())
        used += n
    W = max(len(b) for b in bts)
    bt = torch.zeros(len(ctx_lens), W, dtype=torch.int32)
    for i, b in enumerate(bts):
        bt[i, :len(b)] = torch.tensor(b)
    return kc, vc, bt.cuda()


def _gather(kc, bt_row, L):
    pages = kc[bt_row.long()]  # [n, Hkv, 16, D]
    return pages.permute(0, 2, 1, 3).reshape(-1, kc.shape[1], kc.shape[3])[:L].float()


@pytest.mark.parametrize("D,H,Hkv", [(128, 28, 4), (64, 9, 3), (128, 8, 8)])
@pytest.mark.parametrize("n_split,pps", [(1, 1), (7, 1), (64, 2), (200, 8)])
@pytest.mark.parametrize("window", [0, 40])
def test_decode_attention(D, H, Hkv, n_split, pps, window):
    """Split-KV decode attention against fp32; (200, 8): fixed 8-page splits, most of the grid past
    every sequence's pages (those splits write nothing and the combine skips them)."""
    from fak_b200.ops import kernels as K
    ctx = [1, 17, 100, 333, 1000]
    B = len(ctx)
    kc, vc, bt = _paged_cache(ctx, Hkv, D)
    q = torch.randn(B, H, D, device="cuda")
    out = torch.zeros(B, H * D, device="cuda")
    act = K.ActQ(B, H * D, "cuda")
    ws = torch.full((B * H * n_split * (D + 2),), float("nan"), device="cuda")   # unread slots stay NaN
    K.decode_attention(q, kc, vc, bt, torch.tensor(ctx, dtype=torch.int32, device="cuda"), n_split, out=out, act=act,
                       workspace=ws, window=window, pages_per_split=pps)
    torch.cuda.synchronize()
    G = H // Hkv
    for b, L in enumerate(ctx):
        lo = max(0, L - window) if window else 0   # sliding window: the last `window` keys
        Kb, Vb = _gather(kc, bt[b], L)[lo:], _gather(vc, bt[b], L)[lo:]
        qb = q[b].bfloat16().float()
        s = torch.einsum("hd,thd->ht", qb, Kb.repeat_interleave(G, 1)) / math.sqrt(D)
        ref = torch.einsum("ht,thd->hd", torch.softmax(s, -1), Vb.repeat_interleave(G, 1)).reshape(-1)
        assert torch.allclose(out[b], ref, atol=2e-2, rtol=2e-2), (b, (out[b] - ref).abs().max())
    deq = act.q.float().view(B, -1, 32) * act.ds[:, :, 0:1]
    assert torch.allclose(deq.view(B, -1), out, atol=out.abs().max().item() / 127 + 1e-5)


@pytest.mark.parametrize("qt", [GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q8_0])
def test_embed_rows(qt):
    """The embedding gather (rows spread over several CTAs) returns the dequantized table rows, and
    an id out of range reads row 0 and sets error code 2."""
    from fak_b200.models.weights import QuantWeight
    from fak_b200.ops import kernels as K
    rng = np.random.default_rng(2)
    V, d = 300, 3584
    Wf = (rng.standard_normal((V, d)) * 0.05).astype(np.float32)
    raw = Q.quantize(Wf, qt).reshape(V, -1)
    w = QuantWeight.from_rows(torch.from_numpy(raw), int(qt), d, torch.device("cuda"))
    Wd = torch.from_numpy(Q.dequantize(raw.reshape(-1), qt).reshape(V, d)).cuda()
    ids = torch.tensor([5, 299, 0, 123, 77], dtype=torch.int32, device="cuda")
    out = torch.zeros(5, d, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.embed(w, ids, out, None, err, scale=2.0)
    torch.cuda.synchronize()
    assert torch.allclose(out, 2.0 * Wd[ids.long()], atol=1e-5) and int(err.item()) == 0
    K.embed(w, torch.tensor([V + 3], dtype=torch.int32, device="cuda"), out, None, err)
    torch.cuda.synchronize()
    assert torch.allclose(out[0], Wd[0], atol=1e-5) and int(err.item()) == 2


@pytest.mark.parametrize("n_split,cascade", [(1, 0), (7, 0), (16, 32)])
def test_decode_attention_sinks(n_split, cascade):
    """Attention sinks (gpt-oss): one extra logit per head in the softmax denominator, through the
    single-split path, the split combine and the cascade prefix slots."""
    from fak_b200.ops import kernels as K
    D, H, Hkv = 64, 8, 2
    shared = 64 if cascade else 0
    ctx = [shared + 17, shared + 100, shared + 333]
    B = len(ctx)
    kc, vc, bt = _paged_cache(ctx, Hkv, D, seed=4)
    if cascade:   # the first shared/16 pages identical in every block table
        bt[:, :shared // 16] = bt[0, :shared // 16]
    q = torch.randn(B, H, D, device="cuda")
    sinks = torch.randn(H, device="cuda") * 2
    out = torch.zeros(B, H * D, device="cuda")
    ws = torch.zeros(B * H * (n_split + cascade) * (D + 2), device="cuda")
    extra = {"shared_pages": torch.tensor([shared // 16], dtype=torch.int32, device="cuda"),
             "prefix_splits": cascade} if cascade else {}
    K.decode_attention(q, kc, vc, bt, torch.tensor(ctx, dtype=torch.int32, device="cuda"), n_split, out=out,
                       workspace=ws, sinks=sinks, **extra)
    torch.cuda.synchronize()
    G = H // Hkv
    for b, L in enumerate(ctx):
        Kb, Vb = _gather(kc, bt[b], L), _gather(vc, bt[b], L)
        s = torch.einsum("hd,thd->ht", q[b].bfloat16().float(), Kb.repeat_interleave(G, 1)) / math.sqrt(D)
        pr = torch.softmax(torch.cat([s, sinks[:, None]], 1), 1)[:, :-1]
        ref = torch.einsum("ht,thd->hd", pr, Vb.repeat_interleave(G, 1)).reshape(-1)
        assert torch.allclose(out[b], ref, atol=2e-2, rtol=2e-2), (b, (out[b] - ref).abs().max())


def test_prefill_attention_sinks():
    from fak_b200.models.runner import PrefillMeta
    from fak_b200.ops import kernels as K
    D, H, Hkv = 64, 8, 2
    qlens, pos0s = [70, 5, 130], [0, 40, 300]
    ctx = [p + q for p, q in zip(pos0s, qlens)]
    kc, vc, bt = _paged_cache(ctx, Hkv, D, seed=6)
    T = sum(qlens)
    q = torch.randn(T, H, D, device="cuda").bfloat16()
    sinks = torch.randn(H, device="cuda") * 2
    out = torch.zeros(T, H * D, device="cuda", dtype=torch.bfloat16)
    meta = PrefillMeta.build(qlens, pos0s, "cuda")
    K.prefill_attention(q, kc, vc, bt, meta, out, 0, sinks=sinks)
    torch.cuda.synchronize()
    G = H // Hkv
    off = 0
    for s_, (ql, p0) in enumerate(zip(qlens, pos0s)):
        Kb = _gather(kc, bt[s_], p0 + ql).repeat_interleave(G, 1)
        Vb = _gather(vc, bt[s_], p0 + ql).repeat_interleave(G, 1)
        sc = torch.einsum("qhd,thd->hqt", q[off:off + ql].float(), Kb) / math.sqrt(D)
        qpos = torch.arange(p0, p0 + ql, device="cuda")[:, None]
        kpos = torch.arange(p0 + ql, device="cuda")[None, :]
        sc = sc.masked_fill((kpos > qpos)[None], float("-inf"))
        sk = sinks[:, None, None].expand(H, ql, 1)
        pr = torch.softmax(torch.cat([sc, sk], -1), -1)[..., :-1]
        ref = torch.einsum("hqt,thd->qhd", pr, Vb).reshape(ql, -1)
        got = out[off:off + ql].float()
        assert torch.allclose(got, ref, atol=3e-2, rtol=3e-2), (s_, (got - ref).abs().max())
        off += ql


@pytest.mark.parametrize("D,H,Hkv", [(128, 28, 4), (64, 9, 3)])
@pytest.mark.parametrize("window", [0, 50])
def test_prefill_attention(D, H, Hkv, window):
    from fak_b200.models.runner import PrefillMeta
    from fak_b200.ops import kernels as K
    qlens, pos0s = [70, 5, 130], [0, 40, 300]
    ctx = [p + q for p, q in zip(pos0s, qlens)]
    kc, vc, bt = _paged_cache(ctx, Hkv, D, seed=3)
    T = sum(qlens)
    q = torch.randn(T, H, D, device="cuda").bfloat16()
    out = torch.zeros(T, H * D, device="cuda", dtype=torch.bfloat16)
    meta = PrefillMeta.build(qlens, pos0s, "cuda")
    K.prefill_attention(q, kc, vc, bt, meta, out, window)
    torch.cuda.synchronize()
    G = H // Hkv
    off = 0
    for s, (ql, p0) in enumerate(zip(qlens, pos0s)):
        Kb = _gather(kc, bt[s], p0 + ql).repeat_interleave(G, 1)
        Vb = _gather(vc, bt[s], p0 + ql).repeat_interleave(G, 1)
        qs = q[off:off + ql].float()
        sc = torch.einsum("qhd,thd->hqt", qs, Kb) / math.sqrt(D)
        qpos = torch.arange(p0, p0 + ql, device="cuda")[:, None]
        kpos = torch.arange(p0 + ql, device="cuda")[None, :]
        masked = (kpos > qpos) | ((kpos <= qpos - window) if window else torch.zeros_like(kpos > qpos))
        sc = sc.masked_fill(masked[None], float("-inf"))
        ref = torch.einsum("hqt,thd->qhd", torch.softmax(sc, -1), Vb).reshape(ql, -1)
        got = out[off:off + ql].float()
        assert torch.allclose(got, ref, atol=3e-2, rtol=3e-2), (s, (got - ref).abs().max())
        off += ql


@pytest.mark.parametrize("H,Hkv", [(28, 4), (8, 8)])
@pytest.mark.parametrize("qlens,pos0s", [([256, 256, 5], [8192, 300, 40]), ([130, 1, 383], [0, 17, 1000])])
def test_prefill_attention_tcgen05(H, Hkv, qlens, pos0s):
    """The tcgen05 / TMEM prefill attention against an fp32 reference (ragged chunk, cached prefixes,
    partial 128-query tiles, keys not a multiple of the 128-key tile), over a multi-layer cache."""
    from fak_b200.models.runner import PrefillMeta
    from fak_b200.ops import kernels as K
    D, L, layer = 128, 3, 1
    ctx = [p + q for p, q in zip(pos0s, qlens)]
    n_pages = sum(math.ceil(c / 16) for c in ctx) + 8
    g = torch.Generator(device="cuda").manual_seed(7)
    kc = torch.randn(L, n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(L, n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(n_pages - 1, generator=torch.Generator().manual_seed(3)) + 1
    W = max(math.ceil(c / 16) for c in ctx)
    bt = torch.zeros(len(ctx), W, dtype=torch.int32)
    used = 0
    for i, c in enumerate(ctx):
        n = math.ceil(c / 16)
        bt[i, :n] = perm[used:used + n]
        used += n
    bt = bt.cuda()
    T = sum(qlens)
    q = (torch.randn(T, H, D, device="cuda", generator=g) * 1.5).bfloat16()
    out = torch.zeros(T, H * D, device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    meta = PrefillMeta.build(qlens, pos0s, "cuda")
    K.prefill_attention_tc(q, kc, vc, layer, bt, meta, out, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    G = H // Hkv
    off = 0
    for s, (ql, p0) in enumerate(zip(qlens, pos0s)):
        Kb = _gather(kc[layer], bt[s], p0 + ql).repeat_interleave(G, 1)
        Vb = _gather(vc[layer], bt[s], p0 + ql).repeat_interleave(G, 1)
        qs = q[off:off + ql].float()
        sc = torch.einsum("qhd,thd->hqt", qs, Kb) / math.sqrt(D)
        qpos = torch.arange(p0, p0 + ql, device="cuda")[:, None]
        kpos = torch.arange(p0 + ql, device="cuda")[None, :]
        sc = sc.masked_fill((kpos > qpos)[None], float("-inf"))
        ref = torch.einsum("hqt,thd->qhd", torch.softmax(sc, -1), Vb).reshape(ql, -1)
        got = out[off:off + ql].float()
        assert torch.allclose(got, ref, atol=3e-2, rtol=3e-2), (s, (got - ref).abs().max())
        off += ql


@pytest.mark.parametrize("D,qk_norm", [(128, False), (64, True)])
def test_rope_kv(D, qk_norm):
    from fak_b200.models.reference import apply_rope, rmsnorm, rope_cos_sin
    from fak_b200.models.runner import rope_tables
    from fak_b200.ops import kernels as K
    H, Hkv, T = 6, 2, 9
    qkv = torch.randn(T, (H + 2 * Hkv) * D, device="cuda")
    pos = torch.tensor([0, 1, 2, 5, 17, 100, 1000, 4095, 33], dtype=torch.int32, device="cuda")
    slot = torch.arange(T, dtype=torch.int32, device="cuda") + 16 * 3
    cos, sin = rope_tables(4096, D, 1e6, "cuda")
    kc = torch.zeros(8, Hkv, 16, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    qn = torch.rand(D, device="cuda") + 0.5 if qk_norm else None
    kn = torch.rand(D, device="cuda") + 0.5 if qk_norm else None
    qo = torch.zeros(T, H, D, device="cuda")
    K.rope_kv(qkv, pos, slot, cos, sin, H, Hkv, qn, kn, 1e-6, qo, None, kc, vc)
    torch.cuda.synchronize()
    q = qkv[:, :H * D].view(T, H, D)
    k = qkv[:, H * D:(H + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (H + Hkv) * D:].view(T, Hkv, D)
    if qk_norm:
        q, k = rmsnorm(q, qn, 1e-6), rmsnorm(k, kn, 1e-6)
    c, s = rope_cos_sin(pos.cpu().long(), D, 1e6)
    qr, kr = apply_rope(q.cpu(), c, s), apply_rope(k.cpu(), c, s)
    assert torch.allclose(qo.cpu(), qr, atol=1e-4)
    kk = kc[3].permute(1, 0, 2)[:T].float().cpu()
    vv = vc[3].permute(1, 0, 2)[:T].float().cpu()
    assert torch.allclose(kk, kr, atol=2e-2)
    assert torch.allclose(vv, v.cpu(), atol=2e-2)


def test_argmax_first_index():
    from fak_b200.ops import kernels as K
    x = torch.randn(3, 50000, device="cuda")
    x[1, 7] = 100.0
    x[1, 9] = 100.0
    out = torch.zeros(3, dtype=torch.int32, device="cuda")
    K.argmax(x, 50000, out)
    assert out.tolist() == torch.argmax(x, -1).tolist()
    assert out[1].item() == 7


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 256, 128), (200, 512, 576), (1280, 4608, 3584), (77, 240, 1536),
                                   (1024, 16384, 256)])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
def test_gemm_tcgen05(M, N, K, epi):
    from fak_b200.ops import kernels as Kn
    torch.manual_seed(M + N + K)
    a = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    bias = torch.randn(N, device="cuda") * 0.1
    ref = a.float() @ b.float().T + bias
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    if epi >= 2:
        ref = _swiglu_ref(ref, gelu=epi == 3)
        out = torch.zeros(M, N // 2, device="cuda")
    else:
        out = torch.randn(M, N, device="cuda")
        if epi == 1:
            ref = ref + out
    Kn.gemm(a, b, out, epi, bias, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.allclose(out, ref, atol=2e-3 * math.sqrt(K), rtol=1e-2), (out - ref).abs().max()


def _tg_case(qt, N, Kd, B, seed=3):
    from fak_b200.models.weights import QuantWeight
    from fak_b200.ops import kernels as K
    rng = np.random.default_rng(seed)
    Wf = (rng.standard_normal((N, Kd)) * 0.05).astype(np.float32)
    raw = Q.quantize(Wf, qt).reshape(N, -1)
    w = QuantWeight.from_rows(torch.from_numpy(raw), int(qt), Kd, torch.device("cuda")).pack()
    Wd = torch.from_numpy(Q.dequantize(raw.reshape(-1), qt).reshape(N, Kd)).cuda()
    x = torch.randn(B, Kd, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))
    act = K.ActQ(max(8, B), Kd, "cuda")
    K.quant_act(x, act)
    return w, Wd, x, act


@pytest.mark.parametrize("qt,blk", QTYPES_TILE)
@pytest.mark.parametrize("B", [1, 5, 8, 13, 32])
@pytest.mark.parametrize("epi", [0, 1, 2, 3])
@pytest.mark.parametrize("N", [576, 16 * 2400])
def test_tgemv_tile_packed(qt, blk, B, epi, N):
    """Tile-packed tensor-core GEMV vs an fp32 reference; N=576 runs split-K, the tall matrix one
    slice per tile."""
    from fak_b200.ops import kernels as K
    Kd = 1024 if qt != GGMLType.Q8_0 else 576
    w, Wd, x, act = _tg_case(qt, N, Kd, B)
    bias = torch.randn(N, device="cuda") * 0.1
    ref = x @ Wd.T + bias
    if epi >= K.EPI_SWIGLU:
        ref = _swiglu_ref(ref, gelu=epi == K.EPI_GEGLU)
        y = torch.zeros(B, N // 2, device="cuda")
    else:
        y = torch.randn(B, N, device="cuda")
        if epi == K.EPI_ADD:
            ref = ref + y
    K.gemv(w, act, B, y, bias, epi)
    torch.cuda.synchronize()
    err = (y - ref).abs().max().item() / ref.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
    tol_cos, tol_err = (0.999, 0.06) if epi >= K.EPI_SWIGLU else (0.9995, 0.03)
    assert cos > tol_cos and err < tol_err, (cos, err)


@pytest.mark.parametrize("qt,blk", QTYPES_TILE)
def test_tgemv_batch_invariant_and_repeatable(qt, blk):
    """Each token's output is bit-identical whether it runs alone or in a batch of 8 or 32, and the
    split-K tickets are left at zero so a second launch gives the same bits."""
    from fak_b200.ops import kernels as K
    Kd = 3584 if qt != GGMLType.Q8_0 else 576
    w, Wd, x, act = _tg_case(qt, 512, Kd, 32, seed=7)
    y32 = torch.zeros(32, 512, device="cuda")
    K.gemv(w, act, 32, y32)           # four n8 token tiles per launch
    y8 = torch.zeros(8, 512, device="cuda")
    K.gemv(w, act, 8, y8)             # one tile
    assert torch.equal(y8, y32[:8])
    again = torch.zeros_like(y8)
    K.gemv(w, act, 8, again)
    assert torch.equal(y8, again)
    for b in (0, 3, 7, 21, 31):
        solo = K.ActQ(8, Kd, "cuda")
        K.quant_act(x[b:b + 1], solo)
        y1 = torch.zeros(1, 512, device="cuda")
        K.gemv(w, solo, 1, y1)
        assert torch.equal(y1[0], y32[b]), b
    assert not K.tgemv_workspace("cuda")[1].any()


@pytest.mark.parametrize("Na,Nb", [(4096, 512), (512, 64)])
@pytest.mark.parametrize("B", [1, 5, 13, 32, 40])
@pytest.mark.parametrize("unit", [False, True])
def test_tgemv_pair(Na, Nb, B, unit):
    """One launch of a Q4_K and a Q6_K matrix over the same activations (q|k and v of a Q4_K_M
    layer) vs an fp32 reference of each; a token's outputs are bit-identical alone and in the batch,
    and the split-K tickets of both halves are left at zero."""
    from fak_b200.ops import kernels as K
    Kd = 3584
    wa, Wa, x, _ = _tg_case(GGMLType.Q4_K, Na, Kd, B, seed=21)
    wb, Wb, _, _ = _tg_case(GGMLType.Q6_K, Nb, Kd, B, seed=22)
    act = K.ActQ(max(8, B), Kd, "cuda", unit=unit)
    K.quant_act(x, act)
    ba, bb = torch.randn(Na, device="cuda") * 0.1, torch.randn(Nb, device="cuda") * 0.1
    ya, yb = torch.zeros(B, Na, device="cuda"), torch.zeros(B, Nb, device="cuda")
    assert K.gemv_pair(wb, wa, act, B, yb, ya, bb, ba)    # either order; the Q4_K matrix goes first
    torch.cuda.synchronize()
    for y, ref in ((ya, x @ Wa.T + ba), (yb, x @ Wb.T + bb)):
        err = (y - ref).abs().max().item() / ref.abs().max().item()
        cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
        assert cos > 0.9995 and err < 0.03, (cos, err)
    for b in sorted({0, B // 2, B - 1}):
        solo = K.ActQ(8, Kd, "cuda", unit=unit)
        K.quant_act(x[b:b + 1], solo)
        y1a, y1b = torch.zeros(1, Na, device="cuda"), torch.zeros(1, Nb, device="cuda")
        assert K.gemv_pair(wa, wb, solo, 1, y1a, y1b, ba, bb)
        assert torch.equal(y1a[0], ya[b]) and torch.equal(y1b[0], yb[b]), b
    assert not K.tgemv_workspace("cuda")[1].any()


@pytest.mark.parametrize("qt", [GGMLType.Q4_K, GGMLType.Q6_K])
@pytest.mark.parametrize("B", [1, 5, 13, 32])
@pytest.mark.parametrize("N,Kd", [(576, 4096), (16 * 2400, 1024)])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_tgemv_unit_scale(qt, B, N, Kd, epi):
    """Activations with one scale per 256 columns take the integer-accumulating Q4_K / Q6_K path: it
    must compute exactly what the per-32 float path computes from the same quantized activations (the
    sub-block scales are integers, so only float rounding differs), and stay close to fp32."""
    from fak_b200.ops import kernels as K
    w, Wd, x, _ = _tg_case(qt, N, Kd, B, seed=11)
    act_u = K.ActQ(max(8, B), Kd, "cuda", unit=True)
    K.quant_act(x, act_u)
    ds = act_u.ds[:B].view(B, Kd // 256, 8, 2)
    assert torch.equal(ds[..., 0], ds[..., :1, 0].expand_as(ds[..., 0])), "one scale per unit"
    act_p = K.ActQ(max(8, B), Kd, "cuda")           # the same bytes through the per-32 path
    act_p.q.copy_(act_u.q)
    act_p.ds.copy_(act_u.ds)
    bias = torch.randn(N, device="cuda") * 0.1
    outs = []
    for act in (act_u, act_p):
        y = torch.zeros(B, N // 2, device="cuda") if epi == K.EPI_SWIGLU else torch.ones(B, N, device="cuda")
        K.gemv(w, act, B, y, bias, epi)
        outs.append(y)
    torch.cuda.synchronize()
    yu, yp = outs
    scale = yp.abs().max().item()
    assert (yu - yp).abs().max().item() <= 1e-4 * scale + 1e-6, (yu - yp).abs().max().item()
    deq = (act_u.q[:B].float().view(B, -1, 32) * act_u.ds[:B, :, :1]).view(B, Kd)
    ref = deq @ Wd.T + bias
    if epi == K.EPI_SWIGLU:
        ref = _swiglu_ref(ref)
    elif epi == K.EPI_ADD:
        ref = ref + 1.0
    assert (yu - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-6
    xr = x @ Wd.T + bias
    if epi == K.EPI_SWIGLU:
        xr = _swiglu_ref(xr)
    elif epi == K.EPI_ADD:
        xr = xr + 1.0
    cos = torch.nn.functional.cosine_similarity(yu.flatten(), xr.flatten(), dim=0).item()
    assert cos > (0.998 if epi == K.EPI_SWIGLU else 0.999), cos


@pytest.mark.parametrize("D,H,Hkv", [(128, 28, 4), (64, 9, 3)])
def test_decode_attention_fused_merge_bitexact(D, H, Hkv):
    """The in-kernel split merge (tickets) gives the same bits as the separate combine kernel and
    leaves the tickets at zero."""
    from fak_b200.ops import kernels as K
    ctx = [1, 17, 100, 333, 1000, 4100]
    B = len(ctx)
    kc, vc, bt = _paged_cache(ctx, Hkv, D, n_pages=512)
    q = torch.randn(B, H, D, device="cuda")
    cl = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    ws = torch.zeros(B * H * 32 * (D + 2), device="cuda")
    outs = []
    for tickets in (None, torch.zeros(B * Hkv, dtype=torch.int32, device="cuda")):
        for _ in range(2):
            out = torch.zeros(B, H * D, device="cuda")
            act = K.ActQ(B, H * D, "cuda")
            K.decode_attention(q, kc, vc, bt, cl, 32, out=out, act=act, workspace=ws, tickets=tickets)
            torch.cuda.synchronize()
            outs.append((out, act.q.clone(), act.ds.clone()))
        if tickets is not None:
            assert not tickets.any()
    for o in outs[1:]:
        assert torch.equal(o[0], outs[0][0]) and torch.equal(o[1], outs[0][1]) and torch.equal(o[2], outs[0][2])


@pytest.mark.parametrize("qt,blk", QTYPES_TILE)
@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("N", [576, 16 * 2400])
def test_tgemv_fp32_input_fused_norm(qt, blk, norm, N):
    """fp32 activations normalised and quantized inside the GEMV match the fp32 reference and the
    separately quantized path; a token's result does not depend on the batch."""
    from fak_b200.ops import kernels as K
    Kd = 1024 if qt != GGMLType.Q8_0 else 576
    B = 5
    w, Wd, x, act = _tg_case(qt, N, Kd, B, seed=11)
    x = x * 3
    gamma = (torch.rand(Kd, device="cuda") + 0.5) if norm else None
    xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma if norm else x
    ref = xn @ Wd.T
    y = torch.zeros(B, N, device="cuda")
    K.gemv(w, K.FAct(x, gamma, 1e-6), B, y)
    torch.cuda.synchronize()
    err = (y - ref).abs().max().item() / ref.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(y.flatten(), ref.flatten(), dim=0).item()
    assert cos > 0.9995 and err < 0.03, (cos, err)
    for b in (0, 3):
        y1 = torch.zeros(1, N, device="cuda")
        K.gemv(w, K.FAct(x[b:b + 1], gamma, 1e-6), 1, y1)
        assert torch.equal(y1[0], y[b]), b


@pytest.mark.parametrize("M,N,K", [(1280, 37888, 512), (77, 240, 1536)])
def test_gemm_tcgen05_gated_bf16_out(M, N, K):
    """The gated (SwiGLU) epilogue writing bf16 directly gives the bf16 rounding of the fp32 result."""
    from fak_b200.ops import kernels as Kn
    torch.manual_seed(N)
    a = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    f32 = torch.zeros(M, N // 2, device="cuda")
    b16 = torch.zeros(M, N // 2, device="cuda", dtype=torch.bfloat16)
    Kn.gemm(a, b, f32, 2)
    Kn.gemm(a, b, b16, 2)
    torch.cuda.synchronize()
    assert torch.equal(b16, f32.bfloat16())


def test_gemm_tcgen05_bf16_out_many_tiles_per_cta():
    """Persistent GEMM: several output tiles per CTA (both TMEM accumulators reused), bf16 output."""
    from fak_b200.ops import kernels as Kn
    torch.manual_seed(5)
    M, N, K = 1536, 12288, 512
    a = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    b = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    ref = a.float() @ b.float().T
    out = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    Kn.gemm(a, b, out, 0, None, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert torch.allclose(out.float(), ref, atol=2e-2 * math.sqrt(K) / 8 + 1e-2, rtol=2e-2), (out.float() - ref).abs().max()


@pytest.mark.parametrize("n_keys,qpos,topk", [(300, 299, 64), (5000, 4321, 2048), (40, 10, 64)])
def test_dsa_index_topk_and_sparse_attention(n_keys, qpos, topk):
    """GLM-DSA path: f64 indexer scores, top-k selection (ties to the lower position) and MLA sparse
    attention (kd 192, vd 128) against the PyTorch definitions."""
    from fak_b200.models.dsa import dsa_decode, index_scores_ref, sparse_attend_ref, topk_ref
    from fak_b200.ops._ext import ext
    g = torch.Generator(device="cuda").manual_seed(n_keys)
    nh, dim, H, kd, vd = 32, 128, 16, 192, 128
    iq = torch.randn(nh, dim, device="cuda", generator=g)
    ik = torch.randn(n_keys, dim, device="cuda", generator=g)
    ik[7] = ik[3]                                           # an exact tie: position 3 wins
    w = torch.randn(nh, device="cuda", generator=g)
    q = torch.randn(H, kd, device="cuda", generator=g)
    kc = torch.randn(n_keys, H, kd, device="cuda", generator=g)
    vc = torch.randn(n_keys, H, vd, device="cuda", generator=g)
    score = ext().dsa_index_score(iq, ik, w, qpos, 0.1)
    ref = index_scores_ref(iq, ik, w, qpos, 0.1)
    assert torch.allclose(score[: qpos + 1], ref[: qpos + 1], rtol=1e-12, atol=1e-9)
    assert torch.isinf(score[qpos + 1:]).all()
    out, sel = dsa_decode(q, kc, vc, iq, ik, w, qpos, topk, 0.1, 1 / math.sqrt(kd))
    want_sel = topk_ref(ref.cpu(), qpos, topk)
    assert sel.tolist() == want_sel
    want = sparse_attend_ref(q, kc, vc, want_sel, 1 / math.sqrt(kd))
    assert torch.allclose(out, want, atol=1e-4, rtol=1e-4), (out - want).abs().max()



@pytest.mark.parametrize("D,H,Hkv,B", [(128, 28, 4, 5), (64, 9, 3, 2), (128, 8, 8, 8)])
@pytest.mark.parametrize("shared", [0, 3, 40])
def test_decode_attention_cascade(D, H, Hkv, B, shared):
    """Cascade attention (the batch's shared prefix pages attended once for all lanes) gives the
    per-sequence result: same pages, same softmax, merged with each lane's own suffix."""
    from fak_b200.ops import kernels as K
    g = torch.Generator(device="cuda").manual_seed(shared + B)
    n_pages = 512
    kc = torch.randn(n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    ctx = [shared * 16 + 1 + 37 * i for i in range(B)]
    W = max(math.ceil(c / 16) for c in ctx)
    bt = torch.zeros(B, W, dtype=torch.int32)
    nxt = 1 + shared
    for i, c in enumerate(ctx):
        bt[i, :shared] = torch.arange(1, 1 + shared)                 # the same physical prefix pages
        own = math.ceil(c / 16) - shared
        bt[i, shared:shared + own] = torch.arange(nxt, nxt + own)
        nxt += own
    bt = bt.cuda()
    q = torch.randn(B, H, D, device="cuda", generator=g)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    ws = torch.zeros(B * H * 64 * (D + 2), device="cuda")
    ref = torch.zeros(B, H * D, device="cuda")
    K.decode_attention(q, kc, vc, bt, ctx_t, 16, out=ref, workspace=ws)
    out = torch.zeros(B, H * D, device="cuda")
    sp = torch.tensor([shared], dtype=torch.int32, device="cuda")
    K.decode_attention(q, kc, vc, bt, ctx_t, 16, out=out, workspace=ws, shared_pages=sp, prefix_splits=32)
    torch.cuda.synchronize()
    assert torch.allclose(out, ref, atol=2e-3, rtol=2e-3), (out - ref).abs().max()
    if shared == 0:
        assert torch.equal(out, ref)   # nothing shared: bit-identical to the plain path
