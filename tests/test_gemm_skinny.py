"""The skinny GEMM kernel (one output dimension <= 64, K >= 256: the shape of the DiT block's LoRA
projections and weight gradients) through torch.mm / addmm against the float64 oracle, in the tolerance
of the reference's tests/test_mm.py:31-38. A child process pins B2_GEMM_SKINNY=1 so that every supported
shape takes the kernel (by default only 256 <= K <= 1024 with a wide dimension <= 2048 does): all four
operand-major combinations (K- or M-major A, K- or N-major B), the narrow dimension as N or as M (computed
as C^T = B^T A^T), ranks 8-64 (padded to 16-column tiles), ragged wide dimensions, bias with alpha/beta,
bf16 and f16, and the four LoRA GEMMs of the stacked q/k/v group at 1024 and 4096 tokens."""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import json, sys
sys.path.insert(0, ROOT)
import torch
import oracle
import torch_vulkan_b200 as tv
from tests.helpers import gemm_check, rnd_mm

out = []

def case(name, ad, bd, y, ref, dt, k):
    try:
        gemm_check(y, ref, dt, k)
        ok = True
    except AssertionError as e:
        ok = False
    out.append([name, tv.gemm_path(ad, bd), ok])

def run(m, k, n, ta, tb, dt, bias, seed):
    a = rnd_mm((k, m) if ta else (m, k), dt, seed + 1)
    b = rnd_mm((n, k) if tb else (k, n), dt, seed + 2)
    ad = a.cuda().t() if ta else a.cuda()
    bd = b.cuda().t() if tb else b.cuda()
    ac = a.t() if ta else a
    bc = b.t() if tb else b
    if bias:
        c = rnd_mm((n,), dt, seed + 3)
        y = torch.addmm(c.cuda(), ad, bd, beta=0.5, alpha=2.0)
        ref = oracle.addmm(c, ac, bc, alpha=2.0, beta=0.5)
    else:
        y, ref = torch.mm(ad, bd), oracle.mm(ac, bc)
    case(f"{m}x{k}x{n} ta={ta} tb={tb} {dt} bias={bias}", ad, bd, y, ref, dt, k)

for (m, k, n) in [(1024, 2048, 48), (1000, 512, 16), (2048, 1024, 64), (40, 3000, 24), (16, 4096, 2048), (520, 264, 8)]:
    for ta in (False, True):
        for tb in (False, True):
            run(m, k, n, ta, tb, torch.bfloat16, False, 0)
for dt in (torch.bfloat16, torch.float16):
    for (m, k, n, ta, tb) in [(1024, 2048, 32, False, True), (48, 1024, 6144, True, False), (3000, 704, 56, False, False)]:
        run(m, k, n, ta, tb, dt, True, 5)
dt = torch.bfloat16
for T in (1024, 4096):
    x = rnd_mm((T, 2048), dt, 11).cuda()
    A = (rnd_mm((48, 2048), dt, 12) * 0.05).cuda()
    Bm = (rnd_mm((6144, 48), dt, 13) * 0.05).cuda()
    gy = rnd_mm((T, 6144), dt, 14).cuda()
    h = torch.mm(x, A.t())
    dh = torch.mm(gy, Bm)
    for name, lhs, rhs in (("h", x, A.t()), ("dh", gy, Bm), ("dA", dh.t(), x), ("dB", gy.t(), h)):
        y = torch.mm(lhs, rhs)
        case(f"lora {name} T={T}", lhs, rhs, y, lhs.cpu().double() @ rhs.cpu().double(), dt, lhs.shape[1])
torch.cuda.synchronize()
print("RESULT " + json.dumps({"cases": out, "validation_errors": tv.validation_errors(),
                              "fallbacks": tv.fallback_counts()}))
"""


def test_skinny_kernel_matches_float64():
    r = subprocess.run([sys.executable, "-c", CHILD.replace("ROOT", repr(ROOT))], capture_output=True, text=True,
                       timeout=600, cwd=ROOT, env=dict(os.environ, B2_GEMM_SKINNY="1"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["validation_errors"] == 0 and res["fallbacks"] == {}
    bad = [c for c in res["cases"] if c[1] != "skinny" or not c[2]]
    assert not bad, bad
    assert len(res["cases"]) == 24 + 6 + 8


def test_default_region():
    """Without the pin: the LoRA dA shape at 1024 tokens (K = 1024, wide dimension 2048) takes the skinny
    kernel; the down-projection (K = 2048) and the 4096-token gradients stay on the tcgen05 kernel."""
    import torch_vulkan_b200 as tv

    if os.environ.get("B2_GEMM_SKINNY"):
        pytest.skip("B2_GEMM_SKINNY pins the choice in this process")
    dt = torch.bfloat16
    dh = torch.zeros(1024, 48, dtype=dt, device="cuda")
    x = torch.zeros(1024, 2048, dtype=dt, device="cuda")
    A = torch.zeros(48, 2048, dtype=dt, device="cuda")
    x4 = torch.zeros(4096, 2048, dtype=dt, device="cuda")
    dh4 = torch.zeros(4096, 48, dtype=dt, device="cuda")
    assert tv.gemm_path(dh.t(), x) == "skinny"
    assert tv.gemm_path(x, A.t()) == "tcgen05"
    assert tv.gemm_path(dh4.t(), x4) == "tcgen05"
