"""mm / bmm / addmm / baddbmm through the ATen registrations vs the float64 oracle
(cases of the reference tests/test_mm.py:46-221), plus the tcgen05 path at the DiT shapes."""

import pytest
import torch

import oracle
from tests.helpers import gemm_check, rnd_mm

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
SHAPES = [(1, 1, 1), (7, 5, 3), (64, 16, 64), (65, 17, 63), (128, 129, 300), (33, 1000, 40), (5, 2048, 7)]


@pytest.fixture(autouse=True)
def _lib():
    import torch_vulkan_b200 as tv

    tv.enable(True)
    tv.reset_counts()
    yield tv


def dev(t):
    return t.cuda()


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("m,k,n", SHAPES)
def test_mm_shapes(_lib, dt, m, k, n):
    a, b = rnd_mm((m, k), dt, 1), rnd_mm((k, n), dt, 2)
    out = torch.mm(dev(a), dev(b))
    assert out.dtype == dt and out.shape == (m, n)
    gemm_check(out, oracle.mm(a, b), dt, k)
    assert _lib.kernel_counts().get("aten::mm") == 1
    assert _lib.fallback_counts() == {}


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("ta", [False, True])
@pytest.mark.parametrize("tb", [False, True])
def test_mm_transposed_operands_without_copy(dt, ta, tb):
    m, k, n = 70, 45, 90
    a = rnd_mm((k, m) if ta else (m, k), dt, 3)
    b = rnd_mm((n, k) if tb else (k, n), dt, 4)
    A = dev(a).t() if ta else dev(a)
    B = dev(b).t() if tb else dev(b)
    ref = (a.t() if ta else a).double() @ (b.t() if tb else b).double()
    gemm_check(torch.mm(A, B), ref, dt, k)


def test_mm_on_sliced_views_with_offset():
    a, b = rnd_mm((20, 30), torch.float32, 5), rnd_mm((30, 25), torch.float32, 6)
    out = torch.mm(dev(a)[3:15, 4:20], dev(b)[4:20, 2:22])
    gemm_check(out, a[3:15, 4:20].double() @ b[4:20, 2:22].double(), torch.float32, 16)


@pytest.mark.parametrize("dt", DTYPES)
def test_bmm(dt):
    a, b = rnd_mm((5, 37, 29), dt, 1), rnd_mm((5, 29, 41), dt, 2)
    ref = torch.bmm(a.double(), b.double())
    gemm_check(torch.bmm(dev(a), dev(b)), ref, dt, 29)
    gemm_check(torch.bmm(dev(a), dev(b).transpose(1, 2).contiguous().transpose(1, 2)), ref, dt, 29)


@pytest.mark.parametrize("bias_shape", [(40,), (1, 40), (30, 1), (30, 40), ()])
@pytest.mark.parametrize("dt", DTYPES)
def test_addmm_bias_broadcast_alpha_beta(_lib, bias_shape, dt):
    a, b = rnd_mm((30, 20), dt, 1), rnd_mm((20, 40), dt, 2)
    bias = rnd_mm(bias_shape, dt, 3)
    for alpha, beta in [(1.0, 1.0), (0.5, 2.0), (2.0, 0.0)]:
        out = torch.addmm(dev(bias), dev(a), dev(b), alpha=alpha, beta=beta)
        gemm_check(out, oracle.addmm(bias, a, b, alpha, beta).expand(30, 40), dt, 20)
    assert _lib.kernel_counts().get("aten::addmm") == 3


def test_baddbmm():
    a, b = rnd_mm((3, 10, 8), torch.float32, 1), rnd_mm((3, 8, 12), torch.float32, 2)
    bias = rnd_mm((3, 1, 12), torch.float32, 3)
    out = torch.baddbmm(dev(bias), dev(a), dev(b), alpha=0.5, beta=1.5)
    ref = 1.5 * bias.double() + 0.5 * torch.bmm(a.double(), b.double())
    gemm_check(out, ref.expand(3, 10, 12), torch.float32, 8)


def test_mixed_dtype_raises_and_empty_k():
    with pytest.raises(RuntimeError):
        torch.mm(dev(rnd_mm((4, 5), torch.float32)), dev(rnd_mm((5, 6), torch.bfloat16)))
    z = torch.mm(torch.zeros(3, 0, device="cuda"), torch.zeros(0, 4, device="cuda"))
    assert torch.equal(z.cpu(), torch.zeros(3, 4))


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_linear_forward_backward_matches_cpu(dt):
    torch.manual_seed(0)
    lin = torch.nn.Linear(48, 32).to(dt)
    x = rnd_mm((2, 10, 48), dt, 5)
    xc = x.clone().requires_grad_(True)
    lin(xc).float().pow(2).mean().backward()
    gw, gb, gx = lin.weight.grad.clone(), lin.bias.grad.clone(), xc.grad.clone()
    lin_d = torch.nn.Linear(48, 32).to(dt)
    lin_d.load_state_dict(lin.state_dict())
    lin_d.cuda()
    xd = dev(x).requires_grad_(True)
    lin_d(xd).float().pow(2).mean().backward()
    tol = dict(rtol=2e-4, atol=1e-5) if dt == torch.float32 else dict(rtol=3e-2, atol=3e-3)
    assert torch.allclose(lin_d.weight.grad.cpu().float(), gw.float(), **tol)
    assert torch.allclose(lin_d.bias.grad.cpu().float(), gb.float(), **tol)
    assert torch.allclose(xd.grad.cpu().float(), gx.float(), **tol)


# ---- tcgen05 tensor-core path -------------------------------------------------------------------

@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n", [(128, 64, 128), (256, 128, 256), (1024, 2048, 2048), (65, 72, 200), (300, 136, 520),
                                   (1024, 16, 2048), (1024, 2048, 16), (33, 8, 64)])
def test_tc_matches_reference_and_is_selected(_lib, dt, m, k, n):
    a, b = rnd_mm((m, k), dt, 1), rnd_mm((k, n), dt, 2)
    A, B = dev(a), dev(b)
    # one output dimension <= 64 (a multiple of 8) with 256 <= K <= 1024 and the other <= 2048 goes to the
    # skinny kernel instead
    skinny = 256 <= k <= 1024 and max(m, n) <= 2048 and min(m, n) <= 64 and min(m, n) % 8 == 0
    assert _lib.gemm_path(A, B) == ("skinny" if skinny else "tcgen05")
    gemm_check(torch.mm(A, B), a.double() @ b.double(), dt, k)
    assert _lib.validation_errors() == 0


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_tc_operand_majors_and_bias(_lib, ta, tb):
    dt = torch.bfloat16
    m, k, n = 192, 320, 272
    a = rnd_mm((k, m) if ta else (m, k), dt, 3)
    b = rnd_mm((n, k) if tb else (k, n), dt, 4)
    A = dev(a).t() if ta else dev(a)
    B = dev(b).t() if tb else dev(b)
    assert _lib.gemm_path(A, B) == "tcgen05"
    ref = (a.t() if ta else a).double() @ (b.t() if tb else b).double()
    gemm_check(torch.mm(A, B), ref, dt, k)
    bias = rnd_mm((n,), dt, 5)
    gemm_check(torch.addmm(dev(bias), A, B, alpha=0.5, beta=2.0), 2.0 * bias.double() + 0.5 * ref, dt, k)


def test_tc_bmm_and_agreement_with_simt(_lib):
    a, b = rnd_mm((4, 136, 200), torch.bfloat16, 1), rnd_mm((4, 200, 72), torch.bfloat16, 2)
    ref = torch.bmm(a.double(), b.double())
    out_tc = torch.bmm(dev(a), dev(b))
    gemm_check(out_tc, ref, torch.bfloat16, 200)
    _lib.set_coop_enabled(False)
    try:
        out_simt = torch.bmm(dev(a), dev(b))
    finally:
        _lib.set_coop_enabled(True)
    assert torch.allclose(out_tc.float().cpu(), out_simt.float().cpu(), rtol=1.5e-2, atol=3e-2)


def test_tc_dit_shapes():
    """The DiT block's projections: x[1024,2048] @ W^T for W [2048,2048], [8192,2048]
    and the MLP down-projection [1024,8192] @ [8192,2048]^T, plus the LoRA skinny GEMMs."""
    for (m, k, n) in [(1024, 2048, 2048), (1024, 2048, 8192), (1024, 8192, 2048), (1024, 2048, 16), (1024, 16, 2048)]:
        x = rnd_mm((m, k), torch.bfloat16, 7)
        w = rnd_mm((n, k), torch.bfloat16, 8) * 0.02
        out = torch.nn.functional.linear(dev(x), dev(w))
        gemm_check(out, x.double() @ w.double().t(), torch.bfloat16, k)


@pytest.mark.parametrize("m,k,n,ta,bias", [(4096, 2048, 16, False, False), (2048, 4096, 16, True, False),
                                           (16, 4096, 2048, True, True), (200, 3000, 24, False, True)])
def test_tc_split_k_skinny(_lib, m, k, n, ta, bias):
    """Few output tiles and a long K (the LoRA projections): split-K partials in a scratch buffer and
    a reduction kernel; same result as the oracle, alpha/beta/bias applied once."""
    dt = torch.bfloat16
    a = rnd_mm((k, m) if ta else (m, k), dt, 21)
    b = rnd_mm((k, n), dt, 22)
    ad = dev(a).t() if ta else dev(a)
    ac = a.t() if ta else a
    if bias:
        c = rnd_mm((n,), dt, 23)
        out = torch.addmm(dev(c), ad, dev(b), beta=0.5, alpha=2.0)
        ref = oracle.addmm(c, ac, b, alpha=2.0, beta=0.5)
    else:
        out = torch.mm(ad, dev(b))
        ref = oracle.mm(ac, b)
    gemm_check(out, ref, dt, k)
    assert _lib.fallback_counts() == {}
