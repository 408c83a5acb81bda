"""addcmul / addcdiv / lerp (+ in-place) vs the oracle (reference tests/test_ops_ew.py:291-345) and
the AdamW(foreach=False) loss curve against the CPU."""

import pytest
import torch
import torch.nn.functional as F

import oracle
from tests.helpers import ew_close, rnd_range

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]


@pytest.fixture(autouse=True)
def tv():
    import torch_vulkan_b200 as tv

    tv.reset_counts()
    return tv


@pytest.mark.parametrize("dt", DTYPES)
def test_addcmul_addcdiv_lerp(tv, dt):
    a, b, c = rnd_range((6, 9), dt, seed=1), rnd_range((6, 9), dt, seed=2), rnd_range((6, 9), dt, 0.5, 3.0, seed=3)
    ad = a.cuda()
    ew_close(torch.addcmul(ad, b.cuda(), c.cuda(), value=0.3), oracle.addcmul(a, b, c, 0.3), dt, scale=2.0)
    ew_close(torch.addcdiv(ad, b.cuda(), c.cuda(), value=-0.7), oracle.addcdiv(a, b, c, -0.7), dt, scale=2.0)
    ew_close(torch.lerp(ad, b.cuda(), 0.1), oracle.lerp(a, b, 0.1), dt, scale=2.0)
    x, xd = a.clone(), a.cuda()
    xd.addcmul_(b.cuda(), c.cuda(), value=0.3); x.addcmul_(b, c, value=0.3)
    xd.addcdiv_(b.cuda(), c.cuda(), value=2.0); x.addcdiv_(b, c, value=2.0)
    xd.lerp_(b.cuda(), 0.25); x.lerp_(b, 0.25)
    xd.lerp_(b.cuda(), 0.75); x.lerp_(b, 0.75)
    ew_close(xd, x.double(), dt, scale=4.0)
    kc = tv.kernel_counts()
    for op in ("aten::addcmul", "aten::addcdiv", "aten::lerp.Scalar", "aten::addcmul_", "aten::addcdiv_", "aten::lerp_.Scalar"):
        assert kc.get(op, 0) >= 1, (op, kc)
    assert tv.fallback_counts() == {}


@pytest.mark.parametrize("n", [1, 3, 4, 5, 1023, 1024, 1025, 4097, 100_003])
@pytest.mark.parametrize("dt", DTYPES)
def test_awkward_sizes_and_broadcast(n, dt):
    a, b, c = rnd_range((n,), dt, seed=1), rnd_range((n,), dt, 0.5, 3.0, seed=2), rnd_range((n,), dt, 0.5, 3.0, seed=3)
    ew_close(torch.addcmul(a.cuda(), b.cuda(), c.cuda(), value=1.5), oracle.addcmul(a, b, c, 1.5), dt, scale=2.0)
    m = rnd_range((4, 1, 7), dt, seed=4)
    r = rnd_range((1, 5, 7), dt, seed=5)
    s = rnd_range((7,), dt, 0.5, 2.0, seed=6)
    ew_close(torch.addcdiv(m.cuda(), r.cuda(), s.cuda(), value=0.5), oracle.addcdiv(m, r, s, 0.5), dt, scale=2.0)
    base = rnd_range((8, 6), dt, seed=7)
    ew_close(torch.lerp(base.cuda().t(), rnd_range((6, 8), dt, seed=8).cuda(), 0.3),
             oracle.lerp(base.t(), rnd_range((6, 8), dt, seed=8), 0.3), dt, scale=2.0)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_adamw_matches_cpu(tv, dt):
    def run(device):
        torch.manual_seed(0)
        m = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.GELU(), torch.nn.Linear(32, 4)).to(dt).to(device)
        x, y = torch.randn(32, 16).to(dt).to(device), torch.randn(32, 4).to(dt).to(device)
        opt = torch.optim.AdamW(m.parameters(), lr=1e-2, weight_decay=0.01, foreach=False)
        ls = []
        for _ in range(10):
            opt.zero_grad()
            loss = F.mse_loss(m(x).float(), y.float())
            loss.backward()
            opt.step()
            ls.append(loss.item())
        return ls

    cpu = run("cpu")
    tv.reset_counts()
    gpu = run("cuda")
    tol = 1e-4 if dt == torch.float32 else 5e-2
    assert max(abs(a - b) / max(abs(a), 1e-6) for a, b in zip(cpu, gpu)) < tol, (cpu, gpu)
    kc = tv.kernel_counts()
    assert kc.get("aten::addcmul_", 0) > 0 and kc.get("aten::addcdiv_", 0) > 0 and kc.get("aten::lerp_.Scalar", 0) > 0, kc


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_fused_adamw_matches_foreach_false(tv, dt):
    """FusedAdamW (one b2_adamw_step launch per 48 tensors) against torch.optim.AdamW(foreach=False)
    running on this library's addcmul_/addcdiv_/lerp_, over 10 steps of the same gradients."""
    from torch_vulkan_b200.optim import FusedAdamW

    g = torch.Generator().manual_seed(3)
    shapes = [(16, 2048), (2048, 16), (7,), (3, 5, 9)] * 13  # 52 tensors: more than one launch chunk
    init = [torch.randn(s, generator=g).to(dt) for s in shapes]
    grads = [[torch.randn(s, generator=g).to(dt) for s in shapes] for _ in range(10)]

    def run(make):
        ps = [torch.nn.Parameter(t.clone().cuda()) for t in init]
        opt = make(ps)
        for step in range(10):
            for p, gr in zip(ps, grads[step]):
                p.grad = gr.cuda()
            opt.step()
        return [p.detach().cpu().float() for p in ps]

    ref = run(lambda ps: torch.optim.AdamW(ps, lr=1e-2, weight_decay=0.01, foreach=False))
    tv.reset_counts()
    got = run(lambda ps: FusedAdamW(ps, lr=1e-2, weight_decay=0.01))
    assert tv.kernel_counts().get("b2::adamw_step_", 0) == 10  # one call (two launches: 48 + 4 tensors) per step
    tol = 1e-6 if dt == torch.float32 else 1e-2
    for a, b in zip(got, ref):
        assert torch.allclose(a, b, rtol=tol, atol=tol), (a - b).abs().max()


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_addcmul_broadcast_row(tv, dt):
    """x + g * y with g one broadcast row (the DiT residual update): the [rows, C] vectorised path."""
    x = rnd_range((2, 96, 256), dt, seed=31)
    g = rnd_range((1, 1, 256), dt, seed=32)
    y = rnd_range((2, 96, 256), dt, seed=33)
    ew_close(torch.addcmul(x.cuda(), g.cuda(), y.cuda()), oracle.addcmul(x, g, y, 1.0), dt, scale=2.0)
    ew_close(torch.addcmul(x.cuda(), y.cuda(), g.cuda(), value=0.5), oracle.addcmul(x, y, g, 0.5), dt, scale=2.0)
