"""Fused SDPA forward + backward through F.scaled_dot_product_attention vs the float64 oracle
(cases of the reference tests/test_fused_attention.py:29-169) and at BASELINE config 2."""

import math

import pytest
import torch
import torch.nn.functional as F

import oracle
from tests.helpers import ATTN_REL, rel_err, rnd_unit

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
OVR = "aten::_scaled_dot_product_fused_attention_overrideable"
SHAPES = [(1, 1, 32, 32, 64), (1, 2, 40, 50, 64), (2, 3, 33, 33, 40), (1, 4, 100, 77, 64), (1, 2, 64, 64, 128),
          (1, 2, 17, 5, 20), (1, 2, 130, 130, 96), (1, 2, 35, 37, 30), (1, 1, 48, 48, 36)]


@pytest.fixture(autouse=True)
def tv():
    import torch_vulkan_b200 as tv

    tv.set_fused_attention("on")
    tv.reset_counts()
    yield tv
    tv.set_fused_attention("auto")


def run_dev(q, k, v, g):
    qv, kv, vv = [t.cuda().requires_grad_(True) for t in (q, k, v)]
    o = F.scaled_dot_product_attention(qv, kv, vv)
    o.backward(g.cuda())
    return o.detach().cpu(), qv.grad.cpu(), kv.grad.cpu(), vv.grad.cpu()


def dev_lse(q, k, v):
    """logsumexp [B,H,Sq] fp32 as the fused forward returns it (the op F.scaled_dot_product_attention reaches)."""
    return torch.ops.aten._scaled_dot_product_fused_attention_overrideable(q.cuda(), k.cuda(), v.cuda())[1].cpu()


def check_all(q, k, v, g, dtype, got):
    o64, lse64 = oracle.sdpa_fwd(q, k, v)
    dq64, dk64, dv64 = oracle.sdpa_bwd(q, k, v, g)
    for name, x, ref in zip(("out", "dq", "dk", "dv"), got, (o64, dq64, dk64, dv64)):
        assert x.dtype == dtype and x.shape == ref.shape, name
        e = rel_err(x, ref)
        assert e < ATTN_REL[dtype], f"{name}: rel err {e}"
    # logsumexp is an fp32 statistic: 1e-3 relative (of max(1, |lse|)) whatever the input dtype
    lse = dev_lse(q, k, v)
    assert lse.dtype == torch.float32 and lse.shape == lse64.shape
    err = (lse.double() - lse64).abs().max().item()
    assert err <= 1e-3 * max(1.0, lse64.abs().max().item()), f"lse: max err {err}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_fused_matches_oracle(tv, shape, dtype):
    B, H, Sq, Sk, D = shape
    q, k, v = rnd_unit((B, H, Sq, D), dtype, 1), rnd_unit((B, H, Sk, D), dtype, 2), rnd_unit((B, H, Sk, D), dtype, 3)
    g = rnd_unit((B, H, Sq, D), dtype, 4)
    check_all(q, k, v, g, dtype, run_dev(q, k, v, g))
    kc = tv.kernel_counts()
    assert kc.get(OVR, 0) >= 1 and kc.get(OVR + "_backward", 0) >= 1, kc
    assert not any("softmax" in n or "bmm" in n for n in kc), kc


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_strided_bshd_inputs(tv, dtype):
    B, H, S, D = 2, 4, 70, 64
    qb, kb, vb, gb = (rnd_unit((B, S, H, D), dtype, 5 + i) for i in range(4))
    q, k, v, g = (t.transpose(1, 2) for t in (qb, kb, vb, gb))
    qv, kv, vv = (t.cuda().transpose(1, 2).detach().requires_grad_(True) for t in (qb, kb, vb))
    o = F.scaled_dot_product_attention(qv, kv, vv)
    o.backward(gb.cuda().transpose(1, 2))
    check_all(q, k, v, g, dtype, (o.detach().cpu(), qv.grad.cpu(), kv.grad.cpu(), vv.grad.cpu()))
    assert o.transpose(1, 2).is_contiguous()


def test_large_logits_stay_fp32(tv):
    B, H, S, D = 1, 2, 256, 64
    q = rnd_unit((B, H, S, D), torch.bfloat16, 11, 6.0)
    k = rnd_unit((B, H, S, D), torch.bfloat16, 12, 6.0)
    v = rnd_unit((B, H, S, D), torch.bfloat16, 13)
    got = F.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    assert rel_err(got, oracle.sdpa_fwd(q, k, v)[0]) < 6e-3


def test_unsupported_cases_leave_the_fused_kernel(tv):
    B, H, S = 1, 2, 24
    q, k, v = (rnd_unit((B, H, S, 160), torch.float32, 21 + i) for i in range(3))
    got = F.scaled_dot_product_attention(q.cuda(), k.cuda(), v.cuda()).cpu()
    assert rel_err(got, oracle.sdpa_fwd(q, k, v)[0]) < 3e-5
    mask = torch.zeros(S, S)
    mask[:, S // 2:] = float("-inf")
    q2, k2, v2 = (t[..., :64].contiguous() for t in (q, k, v))
    ref2 = F.scaled_dot_product_attention(q2, k2, v2, attn_mask=mask)
    got2 = F.scaled_dot_product_attention(q2.cuda(), k2.cuda(), v2.cuda(), attn_mask=mask.cuda()).cpu()
    assert rel_err(got2, ref2) < 3e-5
    assert tv.kernel_counts().get(OVR, 0) == 0


def test_auto_policy(tv):
    tv.set_fused_attention("auto")
    q = rnd_unit((1, 2, 64, 64), torch.float32, 41)
    F.scaled_dot_product_attention(q.cuda(), q.cuda(), q.cuda())
    assert tv.kernel_counts().get(OVR, 0) == 0  # small fp32: not fused under auto
    qb = q.to(torch.bfloat16).cuda()
    F.scaled_dot_product_attention(qb, qb, qb)
    assert tv.kernel_counts().get(OVR, 0) == 1
    tv.set_fused_attention("off")
    tv.reset_counts()
    F.scaled_dot_product_attention(qb, qb, qb)
    assert tv.kernel_counts().get(OVR, 0) == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_unaligned_views(tv, dtype):
    B, H, S, D = 1, 2, 45, 64
    n = B * H * S * D
    flats = [rnd_unit((n + 3,), dtype, 10 + i) for i in range(3)]
    gflat = rnd_unit((n + 3,), dtype, 20)
    views = [f[3:].reshape(B, H, S, D) for f in flats]
    gv = gflat[3:].reshape(B, H, S, D)
    q, k, v = (f.cuda()[3:].view(B, H, S, D).detach().requires_grad_(True) for f in flats)
    o = F.scaled_dot_product_attention(q, k, v)
    o.backward(gv.cuda())
    check_all(*views, gv, dtype, (o.detach().cpu(), q.grad.cpu(), k.grad.cpu(), v.grad.cpu()))


def test_config2_attention_and_tc_vs_simt(tv):
    """B1 H16 S1024 D128 bf16, q/k/v/dO ~N(0,1), scale 1/sqrt(128)."""
    g = torch.Generator().manual_seed(0)
    q, k, v, do = (torch.randn(1, 16, 1024, 128, generator=g).to(torch.bfloat16) for _ in range(4))
    got = run_dev(q, k, v, do)
    check_all(q, k, v, do, torch.bfloat16, got)
    tv.set_tc_attention_enabled(False)
    try:
        simt = run_dev(q, k, v, do)
    finally:
        tv.set_tc_attention_enabled(True)
    for a, b in zip(got, simt):
        assert rel_err(a, b) < 2e-2


PAIR_CHILD = r"""
import json, sys
sys.path.insert(0, ROOT)
import torch
import oracle
import torch_vulkan_b200 as tv

OVR = torch.ops.aten._scaled_dot_product_fused_attention_overrideable
g = torch.Generator().manual_seed(11)
out = []
tv.profile_enable(True)
for B, H, Sq, Sk, dt in [(1, 16, 1024, 1024, torch.bfloat16), (1, 2, 4096, 512, torch.bfloat16),
                         (2, 3, 300, 200, torch.float16), (1, 2, 129, 77, torch.bfloat16)]:
    q, k, v = (torch.randn(B, H, S, 128, generator=g).to(dt) for S in (Sq, Sk, Sk))
    o, lse = OVR(q.cuda(), k.cuda(), v.cuda())[:2]
    o64, lse64 = oracle.sdpa_fwd(q, k, v)
    e = ((o.cpu().double() - o64).norm() / o64.norm()).item()
    le = (lse.cpu().double() - lse64).abs().max().item() / max(1.0, lse64.abs().max().item())
    out.append([B, H, Sq, Sk, str(dt), e, le])
torch.cuda.synchronize()
kernels = [ln.split("\t")[0] for ln in tv.profile().splitlines() if ln]
print("RESULT " + json.dumps({"cases": out, "kernels": kernels, "validation_errors": tv.validation_errors()}))
"""


def test_pair_forward_opt_in_matches_oracle():
    """The CTA-pair forward (B2_ATTN_FWD_PAIRS=1, D = 128): O and logsumexp against the float64 oracle at the
    config-2 shape, a 4096 x 512 cross-attention and ragged query/key counts (odd tile counts leave the
    second CTA of the last pair without rows)."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", PAIR_CHILD.replace("ROOT", repr(root))], capture_output=True,
                       text=True, timeout=600, cwd=root, env=dict(os.environ, B2_ATTN_FWD_PAIRS="1"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["validation_errors"] == 0
    assert "attn_fwd_tc_pair" in res["kernels"], res["kernels"]
    for B, H, Sq, Sk, dt, e, le in res["cases"]:
        assert e < 2e-2 and le <= 1e-3, (B, H, Sq, Sk, dt, e, le)


BWD_CHILD = r"""
import json, sys
sys.path.insert(0, ROOT)
import torch
import torch.nn.functional as F
import oracle
import torch_vulkan_b200 as tv

tv.set_fused_attention("on")
tv.profile_enable(True)
g = torch.Generator().manual_seed(12)
out = []
for B, H, Sq, Sk in [(1, 2, 200, 77), (2, 3, 65, 300), (1, 1, 1, 129), (1, 16, 1024, 1024), (2, 2, 333, 512)]:
    q, k, v, do = (torch.randn(B, H, S, 128, generator=g).to(torch.bfloat16) for S in (Sq, Sk, Sk, Sq))
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    F.scaled_dot_product_attention(qd, kd, vd).backward(do.cuda())
    refs = oracle.sdpa_bwd(q, k, v, do)
    errs = [((x.grad.cpu().double() - r).norm() / r.norm()).item() for x, r in zip((qd, kd, vd), refs)]
    out.append([B, H, Sq, Sk] + errs)
torch.cuda.synchronize()
kernels = [ln.split("\t")[0] for ln in tv.profile().splitlines() if ln]
print("RESULT " + json.dumps({"cases": out, "kernels": kernels, "validation_errors": tv.validation_errors()}))
"""


@pytest.mark.parametrize("dsout,fusedq", [("1", "1"), ("1", "0"), ("0", "1")])
def test_tc_backward_forms_ragged(dsout, fusedq):
    """The forms of the tcgen05 backward at ragged D = 128 shapes (query and key counts off the 64 / 128
    tiles, B > 1), each pinned by B2_ATTN_BWD_DSOUT / B2_ATTN_BWD_FUSEDQ and compared with float64: dS^T
    stored to L2 with dQ = scale dS K computed by the same kernel in a second phase (1, 1: the default
    whenever every key-tile CTA fits on the GPU at once) or by a GEMM after it (1, 0), and the in-kernel
    dQ^T with fp32 reductions into an L2 accumulator (0)."""
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", BWD_CHILD.replace("ROOT", repr(root))], capture_output=True,
                       text=True, timeout=600, cwd=root,
                       env=dict(os.environ, B2_ATTN_BWD_DSOUT=dsout, B2_ATTN_BWD_FUSEDQ=fusedq))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["validation_errors"] == 0
    ks = res["kernels"]
    assert ("attn_dq_convert" in ks) == (dsout == "0"), ks
    assert ("attn_bwd_tc_fusedq" in ks) == (dsout == "1" and fusedq == "1"), ks
    if dsout == "1" and fusedq == "0":
        assert "attn_bwd_tc" in ks and any(k.startswith("gemm_tc") for k in ks), ks
    for B, H, Sq, Sk, eq, ek, ev in res["cases"]:
        assert max(eq, ek, ev) < 2e-2, (dsout, B, H, Sq, Sk, eq, ek, ev)
