"""int8 dequant (bit-exact vs the oracle, cases of the reference tests/test_dequant_int8.py:36-75) and
the fused int8-weight linear on the tcgen05 kernel."""

import pytest
import torch

import oracle
from tests.helpers import gemm_check, make_int8, rnd_mm

pytestmark = pytest.mark.gpu
OUT_DTYPES = [torch.float32, torch.bfloat16, torch.float16]
SHAPES = [(1, 64), (1, 36), (3, 100), (5, 4608), (2, 63), (7, 65), (4, 1), (1, 1), (320, 2880), (1280, 5120),
          (2048, 8192), (640, 1280), (33, 130)]


@pytest.fixture(autouse=True)
def tv():
    import torch_vulkan_b200 as tv

    tv.reset_counts()
    return tv


def bits(t):
    return t.view(torch.int16) if t.dtype != torch.float32 else t.view(torch.int32)


@pytest.mark.parametrize("dt", OUT_DTYPES)
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_dequant_matches_reference_bitwise(tv, dt, rows, cols):
    q, scale = make_int8(rows, cols, seed=rows * 1000 + cols)
    out = tv.dequant_int8(q.cuda(), scale.cuda(), dt)
    assert out.is_cuda and out.dtype == dt and out.shape == (rows, cols)
    assert torch.equal(bits(out.cpu()), bits(oracle.dequant_int8(q, scale, dt)))
    assert tv.kernel_counts().get("b2::dequant_int8", 0) >= 1


def test_dequant_extreme_values_and_zero_scale(tv):
    q = torch.tensor([[-128, -127, 0, 1, 127] * 13], dtype=torch.int8)
    scale = torch.tensor([[0.5, 0.0]], dtype=torch.bfloat16)
    for dt in OUT_DTYPES:
        assert torch.equal(bits(tv.dequant_int8(q.cuda(), scale.cuda(), dt).cpu()), bits(oracle.dequant_int8(q, scale, dt)))


def test_dequant_noncontiguous_and_offset_views(tv):
    q, scale = make_int8(8, 200, 3)
    out = tv.dequant_int8(q.cuda()[:, :128], scale[:, :2].cuda(), torch.bfloat16)
    assert torch.equal(bits(out.cpu()), bits(oracle.dequant_int8(q[:, :128].contiguous(), scale[:, :2].contiguous(), torch.bfloat16)))
    q, scale = make_int8(9, 64, 5)
    out = tv.dequant_int8(q.cuda()[1:8], scale[1:8].contiguous().cuda(), torch.float32)
    assert torch.equal(out.cpu(), oracle.dequant_int8(q[1:8], scale[1:8].contiguous(), torch.float32))
    odd = torch.arange(3 * 64 + 1, dtype=torch.int64).to(torch.int8)[1:].view(3, 64)
    sc = (torch.rand(3, 1) + 0.1).to(torch.bfloat16)
    full = torch.arange(3 * 64 + 1, dtype=torch.int64).to(torch.int8).cuda()
    got = tv.dequant_int8(full[1:].view(3, 64), sc.cuda(), torch.bfloat16)
    assert torch.equal(bits(got.cpu()), bits(oracle.dequant_int8(odd, sc, torch.bfloat16)))


def test_dequant_per_row_fp32_scale_config1(tv):
    g = torch.Generator().manual_seed(0)
    q = torch.randint(-127, 128, (6144, 2048), generator=g, dtype=torch.int8)
    s = torch.rand(6144, generator=g) * 9e-3 + 1e-3
    out = tv.dequant_int8(q.cuda(), s.cuda(), torch.bfloat16)
    assert torch.equal(bits(out.cpu()), bits(oracle.dequant_int8(q, s, torch.bfloat16)))


def config1(seed=0, M=1024, N=6144, K=2048):
    """x ~N(0,1) [M,K] bf16 seed 0; W int8 uniform [-127,127]; per-row fp32 scale
    U[1e-3,1e-2]; bias ~N(0,0.02)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 9e-3 + 1e-3
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    return x, q, s, b


@pytest.mark.parametrize("M,N,K", [(1024, 6144, 2048), (200, 384, 320), (64, 256, 64), (1000, 520, 144)])
def test_int8_linear_forward(tv, M, N, K):
    x, q, s, b = config1(1, M, N, K)
    out = tv.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda())
    gemm_check(out, oracle.int8_linear(x, q, s, b), torch.bfloat16, K)
    assert tv.validation_errors() == 0


@pytest.mark.parametrize("M,N,K", [(1024, 2048, 2048), (200, 384, 320), (130, 96, 272)])
def test_int8_linear_backward_dx(tv, M, N, K):
    x, q, s, b = config1(2, M, N, K)
    xd = x.cuda().requires_grad_(True)
    out = tv.int8_linear(xd, q.cuda(), s.cuda(), b.cuda())
    gy = rnd_mm((M, N), torch.bfloat16, 9)
    out.backward(gy.cuda())
    gemm_check(xd.grad, oracle.int8_linear_dx(gy, q, s), torch.bfloat16, N)


def test_int8_linear_block64_scales(tv):
    q, s = make_int8(384, 320, 11)
    x = rnd_mm((200, 320), torch.bfloat16, 12)
    out = tv.int8_linear(x.cuda(), q.cuda(), s.cuda())
    gemm_check(out, oracle.int8_linear(x, q, s), torch.bfloat16, 320)
    gy = rnd_mm((200, 384), torch.bfloat16, 13)
    dx = torch.ops.b2.int8_linear_dx(gy.cuda(), q.cuda(), s.cuda())
    gemm_check(dx, oracle.int8_linear_dx(gy, q, s), torch.bfloat16, 384)


def test_int8_linear_equals_dequant_then_linear(tv):
    """The fused kernel uses bit-identical weights: equal (up to accumulation order) to dequant + mm."""
    x, q, s, b = config1(3, 256, 512, 256)
    fused = tv.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda()).float()
    w = tv.dequant_int8(q.cuda(), s.cuda(), torch.bfloat16)
    two_step = torch.nn.functional.linear(x.cuda(), w, b.cuda()).float()
    assert torch.allclose(fused, two_step, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M,N,K,layout,bias", [(1, 18432, 2048, 1, True), (1, 100, 16, 1, False), (2, 384, 320, 0, True),
                                               (3, 520, 144, 1, True), (5, 96, 2048, 0, False), (8, 2048, 4096, 1, True)])
def test_int8_linear_few_rows_weight_stream(tv, M, N, K, layout, bias):
    """x with at most 8 rows (the DiT adaLN modulation: one conditioning vector against an int8 [18432,
    2048] weight) takes the weight-stream kernel instead of a 128-row tensor-core tile: same dequantised
    weights, fp32 accumulation, against the float64 oracle in the GEMM tolerance; block-64 bf16 scales
    and per-row fp32 scales, ragged N, K down to one 16-column chunk, x a column slice of a wider tensor."""
    if layout == 1:
        x, q, s, b = config1(20 + M, M, N, K)
    else:
        q, s = make_int8(N, K, 30 + M)
        x = rnd_mm((M, K), torch.bfloat16, 31 + M)
        b = (0.02 * rnd_mm((N,), torch.float32, 32)).to(torch.bfloat16)
    b = b if bias else None
    xs = torch.zeros(M, K + 64, dtype=torch.bfloat16)
    xs[:, 8:8 + K] = x
    tv.profile_enable(True)
    try:
        out = tv.int8_linear(xs.cuda()[:, 8:8 + K], q.cuda(), s.cuda(), None if b is None else b.cuda())
        torch.cuda.synchronize()
        kernels = [ln.split("\t")[0] for ln in tv.profile().splitlines() if ln]
    finally:
        tv.profile_enable(False)
    assert "int8_gemv" in kernels
    gemm_check(out, oracle.int8_linear(x, q, s, b), torch.bfloat16, K)
    assert tv.validation_errors() == 0
