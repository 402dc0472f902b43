"""The allocation-free decode attention entry point (C symbol ``fak_decode_attention_noalloc``).

The entry point keeps its split-KV partials in a static device array instead of a caller-supplied
workspace.  This file is named so that pytest collects it last: it must pass both in a fresh
process (its first call performs the per-device set-up) and after every other GPU test.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

_P = ctypes.c_void_p
_I = ctypes.c_int


def _lib():
    from fak_b200.ops._ext import ext
    lib = ctypes.CDLL(ext().__file__)
    fn = lib.fak_decode_attention_noalloc
    fn.restype = _I
    fn.argtypes = [_P, _P, _P, _P, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _I, _P, ctypes.c_char_p,
                   ctypes.c_size_t]
    return fn


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _call(fn, q, kc, vc, bt, ctx, n_split, out, qx, ds):
    B, H, D = q.shape
    err = ctypes.create_string_buffer(256)
    rc = fn(_ptr(q), _ptr(kc), _ptr(vc), _ptr(bt), bt.stride(0), _ptr(ctx), B, H, kc.shape[1], D, n_split, 1,
            _ptr(out), _ptr(qx), _ptr(ds), 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err,
            len(err))
    return rc, err.value.decode()


def _case(seed, ctx_lens, H, Hkv, D):
    g = torch.Generator(device="cuda").manual_seed(seed)
    n_pages = sum(math.ceil(L / 16) for L in ctx_lens) + 1
    kc = torch.randn(n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    vc = torch.randn(n_pages, Hkv, 16, D, device="cuda", generator=g).bfloat16()
    perm = torch.randperm(n_pages - 1, generator=torch.Generator().manual_seed(seed)) + 1
    W = max(math.ceil(L / 16) for L in ctx_lens)
    bt = torch.zeros(len(ctx_lens), W, dtype=torch.int32)
    used = 0
    for i, L in enumerate(ctx_lens):
        n = math.ceil(L / 16)
        bt[i, :n] = perm[used:used + n]
        used += n
    q = torch.randn(len(ctx_lens), H, D, device="cuda", generator=g)
    ctx = torch.tensor(ctx_lens, dtype=torch.int32, device="cuda")
    return q, kc, vc, bt.cuda(), ctx


def _outputs(B, H, D):
    return (torch.zeros(B, H * D, device="cuda"), torch.zeros(B, H * D, dtype=torch.int8, device="cuda"),
            torch.zeros(B, H * D // 32, 2, device="cuda"))


@pytest.mark.parametrize("D,H,Hkv,n_split", [(128, 28, 4, 16), (64, 9, 3, 7), (128, 8, 8, 1)])
def test_noalloc_matches_allocating_entry_point(D, H, Hkv, n_split):
    from fak_b200.ops import kernels as K
    fn = _lib()
    # two calls in a row on different inputs: the second must not see the first call's partials
    # (its shorter contexts leave many splits empty)
    for seed, ctx_lens in ((3, [1, 17, 100, 333, 1000]), (4, [5, 40, 16, 2])):
        q, kc, vc, bt, ctx = _case(seed, ctx_lens, H, Hkv, D)
        B = q.shape[0]
        want = torch.zeros(B, H * D, device="cuda")
        act = K.ActQ(B, H * D, "cuda")
        ws = torch.zeros(B * H * n_split * (D + 2), device="cuda")
        K.decode_attention(q, kc, vc, bt, ctx, n_split, out=want, act=act, workspace=ws)
        out, qx, ds = _outputs(B, H, D)
        rc, msg = _call(fn, q, kc, vc, bt, ctx, n_split, out, qx, ds)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert torch.allclose(out, want, atol=2e-2, rtol=2e-2), (out - want).abs().max()
        assert torch.equal(qx, act.q), "quantized output differs"
        assert torch.allclose(ds, act.ds, atol=1e-5, rtol=1e-5)


def test_noalloc_rejects_oversized_call():
    fn = _lib()
    q, kc, vc, bt, ctx = _case(5, [64] * 8, 32, 8, 128)
    out, qx, ds = _outputs(8, 32, 128)
    rc, msg = _call(fn, q, kc, vc, bt, ctx, 32, out, qx, ds)  # 8 * 32 * 32 = 8192 slots > 4096
    assert rc == 2 and "exceeds the static scratch limit" in msg, (rc, msg)
    torch.cuda.synchronize()
    assert not out.any() and not qx.any(), "a rejected call must launch nothing"
