"""CPU oracle for the hot path — TEST INFRASTRUCTURE ONLY.

Restates, on the CPU and in float64 where the operation is floating point, what the reference
(torch-vulkan) computes for each hot-path operator. Only ``tests/``, ``__graft_entry__.smoke()`` and
the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this module, and only as a
checker or as the timed CPU baseline; the product path (``torch_vulkan_b200``) never calls it.

The reference's CPU path is stock PyTorch CPU ATen — it is what torch-vulkan's CPU fallback runs
(csrc/shim.cpp:70-131) and what every one of its tests compares against — plus the pure-PyTorch int8
dequant of torch_vulkan/__init__.py:203-205. Those pinned third-party semantics (PyTorch; the
reference was validated on 2.8.0, README.md:9, this container has 2.11.0) are restated here; the
bit-level bf16/f16 rounding of the reference shaders (vkrt/shaders/types.glsl:18-50) is restated in C
in ``oracle/rounding.c`` and checked against torch's own conversion.

Parity pins: ``tests/golden/`` holds outputs of the reference's own Python code run in this
container (its dequant and its tests' seeded input generators, executed from the reference sources by
``tests/golden/make_golden.py``) and the oracle is checked against them in ``tests/test_oracle.py``.
"""

from __future__ import annotations

import math

import numpy as np
import torch

# ----------------------------------------------------------------------------------------------------
# int8 weight-only dequant (torch_vulkan/__init__.py:193-205; shader vkrt/shaders/dq8.comp.in:27-62)
# ----------------------------------------------------------------------------------------------------


def dequant_int8(q: torch.Tensor, scale: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    """out[r,c] = round(float(q[r,c]) * float(scale(r,c))): one fp32 multiply, one RNE rounding.

    scale bf16 [rows, ceil(cols/64)] -> scale(r,c) = scale[r, c//64] (the reference layout);
    scale fp32 [rows]                -> scale(r,c) = scale[r]        (per-row layout of BASELINE config 1).
    """
    q = q.cpu()
    scale = scale.cpu()
    cols = q.shape[1]
    if scale.dtype == torch.bfloat16 and scale.dim() == 2:
        s = scale.float().repeat_interleave(64, dim=1)[:, :cols]
    else:
        s = scale.float().reshape(-1, 1)
    return (q.float() * s).to(out_dtype)


def int8_linear(x, q, scale, bias=None):
    """float64 reference of x @ (dequant(q, scale) as bf16)^T + bias (weights rounded to bf16 first,
    exactly as they enter the tensor cores)."""
    w = dequant_int8(q, scale, torch.bfloat16).double()
    y = x.cpu().double() @ w.t()
    if bias is not None:
        y = y + bias.cpu().double()
    return y


def int8_linear_dx(dy, q, scale):
    w = dequant_int8(q, scale, torch.bfloat16).double()
    return dy.cpu().double() @ w


# ----------------------------------------------------------------------------------------------------
# GEMM (csrc/ops_mm.cpp:61-175; tests/test_mm.py:31-38 compares against float64)
# ----------------------------------------------------------------------------------------------------


def addmm(bias, a, b, alpha=1.0, beta=1.0):
    """beta*bias + alpha*(a @ b) in float64 from the dtype-rounded inputs; beta == 0 ignores bias."""
    r = alpha * (a.cpu().double() @ b.cpu().double())
    if bias is not None and beta != 0:
        r = r + beta * bias.cpu().double()
    return r


def mm(a, b):
    return addmm(None, a, b)


def gemm_tolerance(dtype, k):
    """Absolute tolerance factor of tests/test_mm.py:31-38: tol * max(|ref|,1) * (1 + 0.01 sqrt(K))."""
    tol = {torch.float32: 2e-5, torch.bfloat16: 1.2e-2, torch.float16: 2e-3, torch.float64: 1e-12}[dtype]
    return tol * (1 + 0.01 * math.sqrt(k))


# ----------------------------------------------------------------------------------------------------
# attention (csrc/ops_attn.cpp:166-295; vkrt/shaders/attn.comp.in:210-394)
# ----------------------------------------------------------------------------------------------------


def sdpa_fwd(q, k, v, scale=None):
    """O = softmax(scale * Q K^T) V and lse = logsumexp(scale * Q K^T) (natural log), float64."""
    qd, kd, vd = (t.cpu().double() for t in (q, k, v))
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    s = (qd @ kd.transpose(-1, -2)) * scale
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse.unsqueeze(-1))
    return p @ vd, lse


def sdpa_bwd(q, k, v, do, scale=None):
    """dQ, dK, dV of sdpa_fwd for upstream gradient dO (FlashAttention-2 equations, float64)."""
    qd, kd, vd, g = (t.cpu().double() for t in (q, k, v, do))
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    s = (qd @ kd.transpose(-1, -2)) * scale
    p = torch.softmax(s, dim=-1)
    o = p @ vd
    dv = p.transpose(-1, -2) @ g
    dp = g @ vd.transpose(-1, -2)
    delta = (o * g).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    dq = (ds @ kd) * scale
    dk = (ds.transpose(-1, -2) @ qd) * scale
    return dq, dk, dv


def attention_flops(B, H, Sq, Sk, D):
    """fwd 4*B*H*Sq*Sk*D, bwd 2.5x fwd (convention of tools/bench_attention.py:39)."""
    f = 4.0 * B * H * Sq * Sk * D
    return f, 2.5 * f


# ----------------------------------------------------------------------------------------------------
# rows (csrc/ops_rows.cpp:59-181; vkrt/shaders/softmax.comp.in, ln.comp.in)
# ----------------------------------------------------------------------------------------------------


def softmax(x, dim=-1, safe=False):
    xd = x.cpu().double()
    y = torch.softmax(xd, dim)
    if safe:
        y = torch.where(torch.isneginf(xd).all(dim, keepdim=True), torch.zeros_like(y), y)
    return y


def softmax_bwd(y, g, dim=-1):
    yd, gd = y.cpu().double(), g.cpu().double()
    return yd * (gd - (gd * yd).sum(dim, keepdim=True))


def layer_norm(x, normalized_shape, w=None, b=None, eps=1e-5):
    """(y, mean, rstd) in float64; mean/rstd have the reference's fp32-stat shape [..., 1...]."""
    xd = x.cpu().double()
    nd = len(normalized_shape)
    dims = tuple(range(xd.dim() - nd, xd.dim()))
    mean = xd.mean(dims, keepdim=True)
    var = ((xd - mean) ** 2).mean(dims, keepdim=True)
    rstd = 1.0 / torch.sqrt(var + eps)
    y = (xd - mean) * rstd
    if w is not None:
        y = y * w.cpu().double()
    if b is not None:
        y = y + b.cpu().double()
    return y, mean, rstd


def layer_norm_bwd(x, g, normalized_shape, w=None, eps=1e-5):
    """(dx, dw, db) through float64 autograd of layer_norm."""
    xd = x.cpu().double().requires_grad_(True)
    wd = w.cpu().double().requires_grad_(True) if w is not None else None
    bd = torch.zeros(normalized_shape, dtype=torch.float64, requires_grad=True) if w is not None else None
    y = torch.nn.functional.layer_norm(xd, normalized_shape, wd, bd, eps)
    y.backward(g.cpu().double())
    return xd.grad, (wd.grad if wd is not None else None), (bd.grad if bd is not None else None)


# ----------------------------------------------------------------------------------------------------
# optimizer ternaries (csrc/ops_ew.cpp:405-455; tools/gen_shaders.py:83-92)
# ----------------------------------------------------------------------------------------------------


def addcmul(x, t1, t2, value):
    return x.cpu().double() + value * t1.cpu().double() * t2.cpu().double()


def addcdiv(x, t1, t2, value):
    return x.cpu().double() + value * t1.cpu().double() / t2.cpu().double()


def lerp(x, end, weight):
    xd, ed = x.cpu().double(), end.cpu().double()
    return xd + weight * (ed - xd)


# ----------------------------------------------------------------------------------------------------
# bit-level rounding (numpy restatement of vkrt/shaders/types.glsl:45-50; C twin in rounding.c)
# ----------------------------------------------------------------------------------------------------


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns; NaN -> 0x7FC0."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r
