"""The allocation-free decode attention entry point (C symbol ``fak_decode_attention_noalloc``).

It is meant for callers that cannot allocate device memory while they run (a C/C++ runtime linking
the library without PyTorch, or a server whose memory is sized once at start-up): its split-KV
partials live in a static device array instead of a caller-supplied workspace.  The declaration is
``fak_b200/csrc/kernels/fak_noalloc.h``; the ctypes signature below mirrors it.

This file is named so that pytest collects it last.  The entry point must work both in a fresh
process, where its first call performs the per-device set-up (``test_noalloc_fresh_process`` runs
that case in a child interpreter), and after every other GPU test has used the extension.
"""
import ctypes
import math
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

_P = ctypes.c_void_p
_I = ctypes.c_int
EINVAL, ETOOBIG = 1, 2   # FAK_NOALLOC_EINVAL / FAK_NOALLOC_ETOOBIG of fak_noalloc.h


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


def _call(fn, q, kc, vc, bt, ctx, n_split, out, qx, ds, ldo=0, D=None, Hkv=None):
    B, H, Dq = q.shape
    err = ctypes.create_string_buffer(256)
    rc = fn(_ptr(q), _ptr(kc), _ptr(vc), _ptr(bt), bt.stride(0), _ptr(ctx), B, H,
            kc.shape[1] if Hkv is None else Hkv, Dq if D is None else D, n_split, 1,
            _ptr(out), _ptr(qx), _ptr(ds), ldo, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), err,
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


def _outputs(B, K):
    return (torch.zeros(B, K, device="cuda"), torch.zeros(B, K, dtype=torch.int8, device="cuda"),
            torch.zeros(B, K // 32, 2, device="cuda"))


def _allocating(q, kc, vc, bt, ctx, n_split, ldo=0):
    """The existing entry point (workspace from the torch allocator) on the same inputs."""
    from fak_b200.ops import kernels as K
    B, H, D = q.shape
    Kc = ldo or H * D
    want = torch.zeros(B, Kc, device="cuda")
    act = K.ActQ(B, Kc, "cuda")
    ws = torch.zeros(B * H * n_split * (D + 2), device="cuda")
    K.decode_attention(q, kc, vc, bt, ctx, n_split, out=want, act=act, workspace=ws, ldo=ldo)
    return want, act


@pytest.mark.parametrize("D,H,Hkv,n_split", [(128, 28, 4, 16), (64, 9, 3, 7), (128, 8, 8, 1)])
def test_noalloc_matches_allocating_entry_point(D, H, Hkv, n_split):
    fn = _lib()
    # two calls in a row on different inputs: the second must not see the first call's partials
    # (its shorter contexts leave many splits empty)
    for seed, ctx_lens in ((3, [1, 17, 100, 333, 1000]), (4, [5, 40, 16, 2])):
        q, kc, vc, bt, ctx = _case(seed, ctx_lens, H, Hkv, D)
        B = q.shape[0]
        want, act = _allocating(q, kc, vc, bt, ctx, n_split)
        out, qx, ds = _outputs(B, H * D)
        rc, msg = _call(fn, q, kc, vc, bt, ctx, n_split, out, qx, ds)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert torch.allclose(out, want, atol=2e-2, rtol=2e-2), (out - want).abs().max()
        assert torch.equal(qx, act.q), "quantized output differs"
        assert torch.allclose(ds, act.ds, atol=1e-5, rtol=1e-5)


def test_noalloc_quantized_only_with_row_stride():
    """out = NULL (int8 output only) into rows wider than H * D: the extra columns stay untouched."""
    fn = _lib()
    D, H, Hkv, n_split = 128, 28, 4, 16
    ldo = H * D + 32
    for seed, ctx_lens in ((7, [300, 9, 64]), (8, [1, 2000])):
        q, kc, vc, bt, ctx = _case(seed, ctx_lens, H, Hkv, D)
        B = q.shape[0]
        _, act = _allocating(q, kc, vc, bt, ctx, n_split, ldo=ldo)
        _, qx, ds = _outputs(B, ldo)
        rc, msg = _call(fn, q, kc, vc, bt, ctx, n_split, None, qx, ds, ldo=ldo)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert torch.equal(qx[:, :H * D], act.q[:, :H * D]), "quantized output differs"
        assert torch.allclose(ds[:, :H * D // 32], act.ds[:, :H * D // 32], atol=1e-5, rtol=1e-5)
        assert not qx[:, H * D:].any() and not ds[:, H * D // 32:].any(), "columns past H * D were written"


@pytest.mark.parametrize("what", ["head_dim_96", "heads_not_multiple", "ldo_too_small", "no_output"])
def test_noalloc_rejects_bad_arguments(what):
    fn = _lib()
    q, kc, vc, bt, ctx = _case(6, [40, 70], 8, 4, 128)
    out, qx, ds = _outputs(2, 8 * 128)
    kw = {}
    if what == "head_dim_96":
        kw["D"] = 96
    elif what == "heads_not_multiple":
        kw["Hkv"] = 3
    elif what == "ldo_too_small":
        kw["ldo"] = 8 * 128 - 32
    rc, msg = _call(fn, q, kc, vc, bt, ctx, 4, None if what == "no_output" else out,
                    None if what == "no_output" else qx, ds, **kw)
    assert rc == EINVAL and msg.startswith("fak_decode_attention_noalloc"), (rc, msg)
    torch.cuda.synchronize()
    assert not out.any() and not qx.any() and not ds.any(), "a rejected call must launch nothing"


def test_noalloc_rejects_oversized_call():
    fn = _lib()
    q, kc, vc, bt, ctx = _case(5, [64] * 8, 32, 8, 128)
    out, qx, ds = _outputs(8, 32 * 128)
    rc, msg = _call(fn, q, kc, vc, bt, ctx, 32, out, qx, ds)  # 8 * 32 * 32 = 8192 slots > 4096
    assert rc == ETOOBIG and "exceeds the static scratch limit" in msg, (rc, msg)
    torch.cuda.synchronize()
    assert not out.any() and not qx.any(), "a rejected call must launch nothing"


_FRESH = r"""
import sys
sys.path.insert(0, sys.argv[1])
import torch
import tests.test_zz_no_alloc as T
fn = T._lib()
for seed, ctx_lens in ((11, [33, 500, 7]), (12, [900, 1])):
    q, kc, vc, bt, ctx = T._case(seed, ctx_lens, 28, 4, 128)
    out, qx, ds = T._outputs(q.shape[0], 28 * 128)
    rc, msg = T._call(fn, q, kc, vc, bt, ctx, 16, out, qx, ds)   # the first call does the set-up
    assert rc == 0, msg
    want, act = T._allocating(q, kc, vc, bt, ctx, 16)
    torch.cuda.synchronize()
    assert torch.allclose(out, want, atol=2e-2, rtol=2e-2), float((out - want).abs().max())
    assert torch.equal(qx, act.q)
print("fresh ok")
"""


def test_noalloc_fresh_process():
    """The per-device set-up path: the entry point's first call in a new process, before any other
    call of the extension, checked against the allocating entry point."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _FRESH, root], capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0 and "fresh ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
