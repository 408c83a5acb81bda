"""The DiT block's MLP fc2(gelu_tanh(fc1(x))) with the GELU fused into the int8 GEMM epilogues
(b2::int8_linear_gelu_fwd writes h and gelu(h) from one GEMM; b2::int8_linear_dx_gelu returns
(dY @ W2~) * gelu'(h) from one GEMM) against float64 restatements. The reference runs GELU and its
backward as separate elementwise kernels (csrc/ops_ew.cpp:321-326, :352); the expected values here are
the same mathematics (the tanh approximation of F.gelu(approximate="tanh")) in float64."""

import math

import pytest
import torch

import oracle
from tests.helpers import gemm_check, rel_err

pytestmark = pytest.mark.gpu
K0, K1 = math.sqrt(2.0 / math.pi), 0.044715


def gelu64(h):
    return 0.5 * h * (1.0 + torch.tanh(K0 * (h + K1 * h ** 3)))


def gelu_grad64(h):
    t = torch.tanh(K0 * (h + K1 * h ** 3))
    return 0.5 * (1.0 + t) + 0.5 * h * (1.0 - t * t) * K0 * (1.0 + 3.0 * K1 * h * h)


def linear_weights(n_out, n_in, g):
    """int8 [n_out, n_in] uniform in [-127, 127], per-row fp32 scale U[1e-3, 1e-2], bias ~N(0, 0.02)."""
    q = torch.randint(-127, 128, (n_out, n_in), generator=g, dtype=torch.int8)
    s = torch.rand(n_out, generator=g) * 9e-3 + 1e-3
    b = (torch.randn(n_out, generator=g) * 0.02).to(torch.bfloat16)
    return q, s, b


@pytest.mark.parametrize("M,H,F", [(256, 512, 1024), (300, 256, 512), (1024, 2048, 8192)])
def test_fused_gelu_epilogues_match_float64(M, H, F):
    g = torch.Generator().manual_seed(M + H + F)
    q1, s1, b1 = linear_weights(F, H, g)
    q2, s2, _ = linear_weights(H, F, g)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    act, h = torch.ops.b2.int8_linear_gelu_fwd(x.cuda(), q1.cuda(), s1.cuda(), b1.cuda())
    gemm_check(h, oracle.int8_linear(x, q1, s1, b1), torch.bfloat16, H)
    # the epilogue applies GELU to the bf16-rounded h it stores
    h_dev = h.cpu().double()
    assert rel_err(act, gelu64(h_dev)) < 4e-3
    dy = torch.randn(M, H, generator=g).to(torch.bfloat16)
    dh = torch.ops.b2.int8_linear_dx_gelu(dy.cuda(), q2.cuda(), s2.cuda(), h)
    dh64 = oracle.int8_linear_dx(dy, q2, s2) * gelu_grad64(h_dev)
    assert rel_err(dh, dh64) < 8e-3


def test_int8_mlp_forward_and_backward_match_float64_autograd():
    """configs[3]'s MLP (1024 tokens, 2048 -> 8192 -> 2048) through tv.int8_mlp and autograd."""
    import torch_vulkan_b200 as tv

    M, H, F = 1024, 2048, 8192
    g = torch.Generator().manual_seed(5)
    q1, s1, b1 = linear_weights(F, H, g)
    q2, s2, b2 = linear_weights(H, F, g)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    gy = torch.randn(M, H, generator=g).to(torch.bfloat16)
    tv.reset_counts()
    xd = x.cuda().requires_grad_(True)
    y = tv.int8_mlp(xd, q1.cuda(), s1.cuda(), b1.cuda(), q2.cuda(), s2.cuda(), b2.cuda())
    y.backward(gy.cuda())
    kc = tv.kernel_counts()
    assert kc.get("b2::int8_linear_gelu", 0) == 1 and kc.get("b2::int8_linear_dx_gelu", 0) == 1, kc

    torch.set_num_threads(max(1, torch.get_num_threads()))
    x64 = x.double().requires_grad_(True)
    w1 = oracle.dequant_int8(q1, s1, torch.bfloat16).double()
    w2 = oracle.dequant_int8(q2, s2, torch.bfloat16).double()
    y64 = gelu64(x64 @ w1.t() + b1.double()) @ w2.t() + b2.double()
    y64.backward(gy.double())
    assert rel_err(y, y64.detach()) < 1e-2
    assert rel_err(xd.grad, x64.grad) < 2e-2
    assert tv.validation_errors() == 0
