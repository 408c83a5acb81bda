"""softmax / layer_norm forward and backward vs the float64 oracle (cases of the reference
tests/test_rows.py:39-230) and at BASELINE config 3's shapes."""

import pytest
import torch
import torch.nn.functional as F

import oracle
from tests.helpers import rnd_normal, row_close

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


@pytest.fixture(autouse=True)
def tv():
    import torch_vulkan_b200 as tv

    tv.reset_counts()
    return tv


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape,dim", [((7, 33), -1), ((3, 5, 4), 1), ((3, 5, 4), 0), ((2, 1000), 1), ((4, 5000), -1),
                                       ((5, 1), -1), ((2, 3, 4, 5), 2), ((3, 1024), -1), ((2, 2048), -1), ((2, 9000), -1),
                                       ((1, 40000), -1)])
def test_softmax_forward(tv, dt, shape, dim):
    x = rnd_normal(shape, dt, scale=3.0)
    out = torch.softmax(x.cuda(), dim)
    assert out.dtype == dt
    row_close(out, oracle.softmax(x, dim), dt)
    assert tv.kernel_counts().get("aten::_softmax", 0) == 1 and tv.fallback_counts() == {}


def test_softmax_masked_large_and_noncontiguous():
    x = rnd_normal((4, 40), scale=50.0)
    x[:, 5:12] = float("-inf")
    row_close(torch.softmax(x.cuda(), -1), oracle.softmax(x, -1), torch.float32)
    y = rnd_normal((6, 8, 9))
    row_close(torch.softmax(y.cuda().transpose(0, 2), -1), oracle.softmax(y.transpose(0, 2), -1), torch.float32)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(5, 4, 37), (16, 1024), (3, 3000)])
def test_softmax_backward(tv, dt, shape):
    x = rnd_normal(shape, dt, scale=2.0)
    g = rnd_normal(shape, dt, seed=3)
    xd = x.cuda().requires_grad_(True)
    torch.softmax(xd, -1).backward(g.cuda())
    y = torch.softmax(x.double(), -1)
    row_close(xd.grad, oracle.softmax_bwd(y, g), dt, mult=2.0)
    assert tv.kernel_counts().get("aten::_softmax_backward_data", 0) == 1


def test_half_to_float_and_safe_softmax(tv):
    x = rnd_normal((4, 33), torch.bfloat16, scale=3.0)
    out = torch.softmax(x.cuda(), -1, dtype=torch.float32)
    assert out.dtype == torch.float32
    row_close(out, oracle.softmax(x, -1), torch.float32, mult=300.0)
    y = rnd_normal((4, 33))
    y[1, :] = float("-inf")
    y[2, :5] = float("-inf")
    o = torch._safe_softmax(y.cuda(), -1)
    assert torch.allclose(o.cpu(), oracle.softmax(y, -1, safe=True).float(), atol=1e-6)
    assert torch.equal(o.cpu()[1], torch.zeros(33))
    assert tv.kernel_counts().get("aten::_safe_softmax", 0) == 1


def test_softmax_config3_shape():
    """bf16 [16,1024,1024] logits ~N(0,4)."""
    x = rnd_normal((16, 1024, 1024), torch.bfloat16, seed=0, scale=2.0)
    g = rnd_normal((16, 1024, 1024), torch.bfloat16, seed=1)
    xd = x.cuda().requires_grad_(True)
    y = torch.softmax(xd, -1)
    y.backward(g.cuda())
    ref = oracle.softmax(x, -1)
    row_close(y, ref, torch.bfloat16)
    row_close(xd.grad, oracle.softmax_bwd(ref, g), torch.bfloat16, mult=2.0)
    # size-independent property: every row sums to 1 (within bf16 rounding of 1024 terms)
    assert (y.float().sum(-1) - 1).abs().max().item() < 2e-2


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("rows,D", [(3, 7), (5, 256), (4, 1000), (2, 2048), (1, 1), (3, 5000), (2, 20000)])
@pytest.mark.parametrize("affine", [False, True])
def test_layer_norm_forward(tv, dt, rows, D, affine):
    x = rnd_normal((rows, D), dt, scale=2.0)
    w = rnd_normal((D,), dt, 1) if affine else None
    b = rnd_normal((D,), dt, 2) if affine else None
    out = F.layer_norm(x.cuda(), (D,), None if w is None else w.cuda(), None if b is None else b.cuda(), 1e-5)
    row_close(out, oracle.layer_norm(x, (D,), w, b)[0], dt, mult=2.0)
    assert tv.kernel_counts().get("aten::native_layer_norm", 0) == 1 and tv.fallback_counts() == {}


def test_layer_norm_multi_dim_and_stats_dtype():
    x = rnd_normal((1, 1, 8, 8, 128), torch.bfloat16, scale=2.0)
    row_close(F.layer_norm(x.cuda(), (128,), eps=1e-6), oracle.layer_norm(x, (128,), eps=1e-6)[0], torch.bfloat16, mult=2.0)
    y = rnd_normal((4, 3, 5))
    row_close(F.layer_norm(y.cuda(), (3, 5)), oracle.layer_norm(y, (3, 5))[0], torch.float32)
    xb = rnd_normal((4, 64), torch.bfloat16).cuda()
    out, mean, rstd = torch.native_layer_norm(xb, (64,), None, None, 1e-5)
    assert mean.dtype == torch.float32 and rstd.dtype == torch.float32 and out.dtype == torch.bfloat16
    assert mean.shape == (4, 1)
    _, m64, r64 = oracle.layer_norm(xb.cpu(), (64,), eps=1e-5)
    assert torch.allclose(mean.cpu().double(), m64, rtol=1e-3, atol=1e-6)
    assert torch.allclose(rstd.cpu().double(), r64, rtol=1e-3)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("affine", [False, True])
@pytest.mark.parametrize("rows,D", [(6, 96), (1024, 2048), (37, 3000), (3, 20000)])
def test_layer_norm_backward(tv, dt, affine, rows, D):
    x = rnd_normal((rows, D), dt, scale=2.0)
    w = rnd_normal((D,), dt, 1) if affine else None
    b = rnd_normal((D,), dt, 2) if affine else None
    g = rnd_normal((rows, D), dt, 3)
    dx64, dw64, db64 = oracle.layer_norm_bwd(x, g, (D,), w, 1e-5)
    xd = x.cuda().requires_grad_(True)
    wd = w.cuda().requires_grad_(True) if affine else None
    bd = b.cuda().requires_grad_(True) if affine else None
    F.layer_norm(xd, (D,), wd, bd, 1e-5).backward(g.cuda())
    row_close(xd.grad, dx64, dt, mult=4.0)
    if affine:
        # dw, db: 2e-2 of max|ref| in bf16 (the gradient tolerance of the hot path), 3e-5 in fp32
        rel_close(wd.grad, dw64, 2e-2 if dt == torch.bfloat16 else 3e-5)
        rel_close(bd.grad, db64, 2e-2 if dt == torch.bfloat16 else 3e-5)
    assert tv.kernel_counts().get("aten::native_layer_norm_backward", 0) == 1


def rel_close(out, ref64, rtol):
    o, r = out.detach().cpu().double(), ref64.double()
    assert o.shape == r.shape
    err = (o - r).abs().max().item()
    assert err <= rtol * r.abs().max().item(), f"max err {err} (max|ref| {r.abs().max().item()})"


def test_layer_norm_config3():
    """BASELINE configs[2] LayerNorm: bf16 [1024, 2048] ~N(0,1), w ~N(1,0.1), b ~N(0,0.1), eps 1e-6, grad ~N(0,1).
    y within bf16 tolerance, fp32 mean/rstd within 1e-3 relative, dx/dw/db within 2e-2 of max|ref|."""
    x = rnd_normal((1024, 2048), torch.bfloat16, seed=0)
    w = (1 + rnd_normal((2048,), seed=1, scale=0.1)).to(torch.bfloat16)
    b = rnd_normal((2048,), torch.bfloat16, seed=2, scale=0.1)
    g = rnd_normal((1024, 2048), torch.bfloat16, seed=3)
    xd, wd, bd = (t.cuda().requires_grad_(True) for t in (x, w, b))
    y, mean, rstd = torch.native_layer_norm(xd, (2048,), wd, bd, 1e-6)
    y64, m64, r64 = oracle.layer_norm(x, (2048,), w, b, eps=1e-6)
    row_close(y, y64, torch.bfloat16, mult=2.0)
    assert torch.allclose(mean.detach().cpu().double(), m64, rtol=1e-3, atol=1e-6)
    assert torch.allclose(rstd.detach().cpu().double(), r64, rtol=1e-3)
    y.backward(g.cuda())
    dx64, dw64, db64 = oracle.layer_norm_bwd(x, g, (2048,), w, 1e-6)
    rel_close(xd.grad, dx64, 2e-2)
    rel_close(wd.grad, dw64, 2e-2)
    rel_close(bd.grad, db64, 2e-2)
