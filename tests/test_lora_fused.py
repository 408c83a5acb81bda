"""The LoRA side path inside the int8 GEMM (b2::int8_lora_fwd / b2::int8_lora_dx and tv.int8_lora_linear)
against float64 restatements. The reference computes a LoRA linear as separate linears (module layout of
tests/anima_on_vk.py:43-48): y = x W^T + b + (x A^T) B^T * alpha / r. Here the up-projection is one more
64-wide reduction block of the int8 GEMM, and the backward's dX = dY W + (dY B s) A is one GEMM too. The
cases cover the DiT block's stacked groups (q/k/v: r = 48 over 6144 outputs; cross k/v: r = 32 on the
512 text tokens), a single module (r = 16) and ragged edges, in both int8 kernel forms (single CTAs and
CTA pairs, pinned per child process by B2_INT8_CG)."""

import json
import os
import subprocess
import sys

import pytest
import torch

import oracle
from tests.helpers import rel_err

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys
sys.path.insert(0, ROOT)
import torch
import oracle
import torch_vulkan_b200 as tv
from tests.helpers import make_int8

def rel(a, b):
    a = a.cpu().double()
    return ((a - b).norm() / b.norm()).item()

g = torch.Generator().manual_seed(3)
out = []
for M, N, K, r, lay in [(1024, 6144, 2048, 48, "row"), (512, 4096, 1024, 32, "row"), (300, 520, 272, 16, "row"),
                        (256, 384, 320, 16, "block64"), (4096, 2048, 2048, 16, "row")]:
    if lay == "row":
        q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
        s = torch.rand(N, generator=g) * 9e-3 + 1e-3
    else:
        q, s = make_int8(N, K, seed=N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    a = (torch.randn(r, K, generator=g) / K ** 0.5).to(torch.bfloat16)     # down-projection [r, K]
    b = (torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16)         # up-projection * alpha / r
    h = (x.double() @ a.double().t()).to(torch.bfloat16)                    # as the caller computes it
    y = torch.ops.b2.int8_lora_fwd(x.cuda(), q.cuda(), s.cuda(), bias.cuda(), h.cuda(), b.cuda())
    w = oracle.dequant_int8(q, s, torch.bfloat16).double()
    y64 = x.double() @ w.t() + bias.double() + h.double() @ b.double().t()
    dy = torch.randn(M, N, generator=g).to(torch.bfloat16)
    dh = (dy.double() @ b.double()).to(torch.bfloat16)
    dx = torch.ops.b2.int8_lora_dx(dy.cuda(), q.cuda(), s.cuda(), dh.cuda(), a.cuda())
    dx64 = dy.double() @ w + dh.double() @ a.double()
    out.append([M, N, K, r, lay, rel(y, y64), rel(dx, dx64)])
torch.cuda.synchronize()
print("RESULT " + json.dumps({"cases": out, "validation_errors": tv.validation_errors()}))
"""


@pytest.mark.parametrize("cg", ["1", "2"])
def test_int8_lora_ops_match_float64(cg):
    env = dict(os.environ, B2_INT8_CG=cg)
    r = subprocess.run([sys.executable, "-c", CHILD.replace("ROOT", repr(ROOT))], capture_output=True, text=True,
                       timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads([l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["validation_errors"] == 0
    for M, N, K, rk, lay, e_f, e_d in res["cases"]:
        assert e_f < 4e-3 and e_d < 4e-3, (cg, M, N, K, rk, lay, e_f, e_d)


def test_int8_lora_linear_autograd_matches_float64():
    """tv.int8_lora_linear forward and the gradients of x, A and B (the stacked q/k/v group of configs[3])."""
    import torch_vulkan_b200 as tv

    M, N, K, r = 1024, 6144, 2048, 48
    g = torch.Generator().manual_seed(9)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 9e-3 + 1e-3
    bias = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    a = (torch.randn(r, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    b = (torch.randn(N, r, generator=g) * 0.05).to(torch.bfloat16)
    gy = torch.randn(M, N, generator=g).to(torch.bfloat16)
    tv.reset_counts()
    xd, ad, bd = (t.cuda().requires_grad_(True) for t in (x, a, b))
    y = tv.int8_lora_linear(xd, q.cuda(), s.cuda(), bias.cuda(), ad, bd)
    y.backward(gy.cuda())
    kc = tv.kernel_counts()
    assert kc.get("b2::int8_lora_fwd", 0) == 1 and kc.get("b2::int8_lora_dx", 0) == 1, kc

    w = oracle.dequant_int8(q, s, torch.bfloat16).double()
    x64, a64, b64 = (t.double().requires_grad_(True) for t in (x, a, b))
    y64 = x64 @ w.t() + bias.double() + (x64 @ a64.t()) @ b64.t()
    y64.backward(gy.double())
    assert rel_err(y, y64.detach()) < 1e-2
    for name, got, ref in (("dx", xd.grad, x64.grad), ("dA", ad.grad, a64.grad), ("dB", bd.grad, b64.grad)):
        e = rel_err(got, ref)
        assert e < 2e-2, (name, e)
