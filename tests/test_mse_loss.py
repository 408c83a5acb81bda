"""The DiT step's MSE loss kernels (b2::mse_loss_fwd / b2::mse_loss_bwd through tv.mse_loss) against
F.mse_loss in float64 on the CPU: the mean of squared differences in fp32 from 16-bit operands, and the
gradient 2 (x - t) g / n in x's dtype. Sizes cover the vector path (n a multiple of 8), the scalar path
(odd n, an unaligned view), one element, empty input and the DiT step's [4096, 2048] activation; the loss
is the same bits on every call (fixed summation order)."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _pair(n, dt, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g).to(dt)
    t = (0.5 * torch.randn(n, generator=g)).to(dt)
    return x, t


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("n", [1, 7, 8, 1000, 4099, 65536, 4096 * 2048])
def test_forward_backward_vs_float64(dt, n):
    import torch_vulkan_b200 as tv

    x, t = _pair(n, dt, 11 + n)
    ref = F.mse_loss(x.double(), t.double())
    xd = x.cuda().requires_grad_(True)
    loss = tv.mse_loss(xd, t.cuda())
    assert loss.dtype == torch.float32 and loss.dim() == 0
    # fp32 accumulation of n squared differences: relative error a few ulp times log(n)
    assert abs(loss.item() - ref.item()) <= 1e-5 * abs(ref.item()) + 1e-7
    loss.backward(torch.tensor(1.5, device="cuda"))
    gref = (2.0 * 1.5 / n) * (x.double() - t.double())
    tol = {torch.float32: 1e-6, torch.float16: 1e-3, torch.bfloat16: 8e-3}[dt]
    # at large n the f16 gradient falls into f16's subnormal range (steps of 2^-24): one step absolute
    tiny = 2.0 ** -24 if dt == torch.float16 else 0.0
    assert xd.grad.dtype == dt
    torch.testing.assert_close(xd.grad.cpu().double(), gref, rtol=tol, atol=tol * gref.abs().max().item() + tiny + 1e-30)


def test_unaligned_view_takes_scalar_path():
    import torch_vulkan_b200 as tv

    x, t = _pair(4097, torch.bfloat16, 5)
    xs, ts = x.cuda()[1:], t.cuda()[1:]  # 2-byte offset: not 16-byte aligned
    ref = F.mse_loss(x[1:].double(), t[1:].double()).item()
    assert abs(tv.mse_loss(xs, ts).item() - ref) <= 1e-5 * ref


def test_empty_and_target_gradient():
    import torch_vulkan_b200 as tv

    e = torch.empty(0, 16, device="cuda", dtype=torch.bfloat16)
    assert torch.isnan(tv.mse_loss(e, e)).item()  # F.mse_loss's mean over no elements
    x, t = _pair(2048, torch.bfloat16, 3)
    xd, td = x.cuda().requires_grad_(True), t.cuda().requires_grad_(True)
    tv.mse_loss(xd, td).backward()
    torch.testing.assert_close(td.grad, -xd.grad, rtol=0, atol=0)


def test_deterministic_and_matches_reshape():
    import torch_vulkan_b200 as tv

    x, t = _pair(4 * 1024 * 2048, torch.bfloat16, 9)
    xd, td = x.cuda().view(4, 1024, 2048), t.cuda().view(4, 1024, 2048)
    a = tv.mse_loss(xd, td)
    b = tv.mse_loss(xd, td)
    c = tv.mse_loss(xd.reshape(-1), td.reshape(-1))
    assert a.item() == b.item() == c.item()


def test_mismatched_inputs_raise():
    import torch_vulkan_b200 as tv

    x = torch.zeros(8, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        tv.mse_loss(x, torch.zeros(8, device="cuda", dtype=torch.float16))
    with pytest.raises(RuntimeError):
        tv.mse_loss(x, torch.zeros(9, device="cuda", dtype=torch.bfloat16))
