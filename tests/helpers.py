"""Seeded input generators (same recipes as the reference tests, so the golden fixtures made from the
reference's own generators pin them) and comparison helpers."""

from __future__ import annotations

import numpy as np
import torch


def rnd_mm(shape, dtype, seed=0):
    """tests/test_mm.py:26-28"""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g).to(dtype)


def rnd_unit(shape, dtype=torch.float32, seed=0, scale=1.0):
    """tests/test_fused_attention.py:43-45: uniform in [-scale, scale)"""
    g = torch.Generator().manual_seed(seed)
    return ((torch.rand(shape, generator=g) * 2 - 1) * scale).to(dtype)


def rnd_normal(shape, dtype=torch.float32, seed=0, scale=1.0):
    """tests/test_rows.py:24-26: N(0, scale^2)"""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype)


def rnd_range(shape, dtype=torch.float32, lo=-3.0, hi=3.0, seed=0):
    """tests/test_ops_ew.py:27-29: uniform in [lo, hi)"""
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(shape, generator=g) * (hi - lo) + lo).to(dtype)


def make_int8(rows, cols, seed=0):
    """tests/test_dequant_int8.py:24-30: q uniform in [-127,127], bf16 block-64 scales in [1e-4, 0.0201)"""
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (rows, cols), generator=g, dtype=torch.int8)
    nb = (cols + 63) // 64
    scale = (torch.rand(rows, nb, generator=g) * 0.02 + 1e-4).to(torch.bfloat16)
    return q, scale


def from_np(a: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    t = torch.from_numpy(np.array(a))
    if dtype == torch.bfloat16:
        return t.view(torch.bfloat16)
    return t.to(dtype)


def gemm_check(out, ref64, dtype, k):
    """tests/test_mm.py:31-38: |out - ref| <= tol * max(|ref|, 1) * (1 + 0.01 sqrt(K))"""
    o = out.detach().cpu().double()
    assert o.shape == ref64.shape, (o.shape, ref64.shape)
    scale = max(ref64.abs().max().item() if ref64.numel() else 0.0, 1.0)
    tol = {torch.float32: 2e-5, torch.bfloat16: 1.2e-2, torch.float16: 2e-3, torch.float64: 1e-12}[dtype]
    err = (o - ref64).abs().max().item() if o.numel() else 0.0
    assert err <= tol * scale * (1 + k ** 0.5 * 0.01), f"max err {err} scale {scale}"


ROW_TOL = {torch.float32: 3e-5, torch.bfloat16: 1.2e-2, torch.float16: 2.5e-3}


def row_close(out, ref64, dtype, mult=1.0):
    """tests/test_rows.py:29-34"""
    o, r = out.detach().cpu().double(), ref64.double()
    assert o.shape == r.shape, (o.shape, r.shape)
    scale = max(r.abs().max().item(), 1.0)
    err = (o - r).abs().max().item()
    assert err <= ROW_TOL[dtype] * scale * mult, f"max err {err} (scale {scale})"


ATTN_REL = {torch.float32: 3e-5, torch.bfloat16: 2e-2, torch.float16: 4e-3}


def rel_err(a, b):
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


EW_TOL = {torch.float32: (1e-5, 1e-6), torch.bfloat16: (2e-2, 1e-3), torch.float16: (4e-3, 1e-4)}


def ew_close(out, ref, dtype, scale=1.0):
    """tests/test_ops_ew.py:32-37"""
    rtol, atol = EW_TOL[dtype]
    g, c = out.detach().cpu().double(), ref.double()
    assert g.shape == c.shape
    assert torch.allclose(g, c, rtol=rtol * scale, atol=atol * scale), f"max diff {(g - c).abs().max().item()}"
