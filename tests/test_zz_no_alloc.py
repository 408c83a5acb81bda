"""The allocation-free LayerNorm backward (b2_layernorm_bwd_noalloc), called through the C ABI.

It exists for callers that cannot allocate device memory in the middle of a step — a host framework
that owns every byte of VRAM through its own allocator or a fixed budget, or an FFI caller that only
holds the tensors. Its dw/db partial sums live in a fixed 2 MiB array inside the library instead of a
caller-provided workspace. This test compares it with the regular entry point (which takes a
workspace) on two calls in a row, so the second call runs on the scratch the first one left behind.
The file name makes pytest collect it last."""

import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class LnArgs(ctypes.Structure):
    # mirrors b2_layernorm_args in include/b2rt.h
    _fields_ = [(n, ctypes.c_void_p) for n in ("x", "w", "b", "y", "mean", "rstd", "g", "dx", "dw", "db", "workspace")] + [
        ("rows", ctypes.c_int64), ("D", ctypes.c_int64), ("eps", ctypes.c_float), ("dtype", ctypes.c_int32)]


def lib():
    import torch_vulkan_b200  # noqa: F401  (loads libb2rt.so into the process)

    L = ctypes.CDLL(os.path.join(ROOT, "torch_vulkan_b200", "libb2rt.so"))
    L.b2_layernorm_bwd.argtypes = [ctypes.POINTER(LnArgs), ctypes.c_void_p]
    L.b2_layernorm_bwd_noalloc.argtypes = [ctypes.POINTER(LnArgs), ctypes.c_void_p]
    L.b2_layernorm_bwd_workspace_bytes.argtypes = [ctypes.POINTER(LnArgs)]
    L.b2_layernorm_bwd_workspace_bytes.restype = ctypes.c_uint64
    return L


def ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def run_once(L, x, w, g, mean, rstd, noalloc):
    rows, D = x.shape
    dx, dw, db = torch.empty_like(x), torch.empty_like(w), torch.empty_like(w)
    a = LnArgs()
    a.x, a.w, a.g, a.mean, a.rstd = ptr(x), ptr(w), ptr(g), ptr(mean), ptr(rstd)
    a.dx, a.dw, a.db = ptr(dx), ptr(dw), ptr(db)
    a.rows, a.D, a.eps, a.dtype = rows, D, 1e-6, {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[x.dtype]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = L.b2_layernorm_bwd_noalloc(ctypes.byref(a), stream)
    else:
        ws = torch.empty(int(L.b2_layernorm_bwd_workspace_bytes(ctypes.byref(a))) // 4 + 1, device=x.device)
        a.workspace = ptr(ws)
        rc = L.b2_layernorm_bwd(ctypes.byref(a), stream)
    assert rc == 0
    torch.cuda.synchronize()
    return dx, dw, db


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,D", [(1024, 2048), (37, 3000), (300, 96)])
def test_noalloc_layernorm_backward_matches_regular_entry(dt, rows, D):
    L = lib()
    gen = torch.Generator().manual_seed(rows + D)
    x = (torch.randn(rows, D, generator=gen) * 2).to(dt).cuda()
    w = (1 + 0.1 * torch.randn(D, generator=gen)).to(dt).cuda()
    g = torch.randn(rows, D, generator=gen).to(dt).cuda()
    _, mean, rstd = torch.native_layer_norm(x, (D,), w, None, 1e-6)
    mean, rstd = mean.reshape(rows).contiguous(), rstd.reshape(rows).contiguous()
    ref = run_once(L, x, w, g, mean, rstd, noalloc=False)
    for _ in range(2):  # the second call reuses the scratch the first one wrote
        got = run_once(L, x, w, g, mean, rstd, noalloc=True)
        assert torch.equal(got[0], ref[0])  # dx does not touch the scratch
        tol = dict(rtol=1e-5, atol=1e-4) if dt == torch.float32 else dict(rtol=1.6e-2, atol=1e-2)
        for name, a, b in (("dw", got[1], ref[1]), ("db", got[2], ref[2])):
            assert torch.allclose(a.float(), b.float(), **tol), (name, (a.float() - b.float()).abs().max().item())


def test_noalloc_long_rows_use_fewer_partial_slots():
    """fp32 rows of 100000 elements take the long-row kernels; the 2 MiB scratch holds only two partial
    slots of 2 x 100000 floats (the regular entry plans far more), so each slot sums 300 of the 600 rows."""
    L = lib()
    rows, D = 600, 100_000
    gen = torch.Generator().manual_seed(rows + D)
    x = torch.randn(rows, D, generator=gen).cuda()
    w = (1 + 0.1 * torch.randn(D, generator=gen)).cuda()
    g = torch.randn(rows, D, generator=gen).cuda()
    _, mean, rstd = torch.native_layer_norm(x, (D,), w, None, 1e-6)
    mean, rstd = mean.reshape(rows).contiguous(), rstd.reshape(rows).contiguous()
    ref = run_once(L, x, w, g, mean, rstd, noalloc=False)
    for _ in range(2):
        got = run_once(L, x, w, g, mean, rstd, noalloc=True)
        assert torch.equal(got[0], ref[0])
        for name, a, b in (("dw", got[1], ref[1]), ("db", got[2], ref[2])):
            assert torch.allclose(a, b, rtol=1e-5, atol=1e-4), (name, (a - b).abs().max().item())


def test_noalloc_rejects_rows_wider_than_the_scratch():
    L = lib()
    D = 300_000  # 2 * D floats > the 512 Ki-float scratch
    x = torch.zeros(1, D, device="cuda")
    w = torch.ones(D, device="cuda")
    a = LnArgs()
    stats = torch.zeros(1, device="cuda")
    a.x, a.w, a.g, a.mean, a.rstd = ptr(x), ptr(w), ptr(x), ptr(stats), ptr(stats)
    dw = torch.empty_like(w)
    a.dw = ptr(dw)
    a.rows, a.D, a.eps, a.dtype = 1, D, 1e-5, 0
    assert L.b2_layernorm_bwd_noalloc(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) < 0
