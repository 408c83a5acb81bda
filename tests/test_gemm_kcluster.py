"""Split-K GEMMs reduced inside a thread-block cluster (the LoRA projections and weight gradients of the
DiT block: one of M, N is 16-64, K is long): each CTA of a cluster computes one K slice of a 128x128 tile
and the cluster sums the fp32 partials through distributed shared memory, with no workspace and no second
kernel. Checked against float64 in both forms — the cluster reduction (the default, B2_GEMM_KCLUSTER=1) and
the workspace + gemm_splitk_reduce form (=0), each pinned in a child process with the skinny kernel (which
serves these shapes by default) switched off — over K-major and MN-major operands, ragged M/N, bias with
alpha/beta, and splits wider than a cluster (which keep the workspace form)."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import ctypes, json, sys
sys.path.insert(0, ROOT)
import torch
import oracle
import torch_vulkan_b200 as tv
from tests.helpers import rnd_mm

g_cases = [(1024, 2048, 48, False, False, False), (1000, 6144, 48, False, True, False),
           (48, 1024, 2048, True, False, True), (2048, 4096, 16, True, False, False),
           (6144, 1024, 48, True, True, False), (200, 3000, 24, False, False, True),
           (4096, 2048, 16, False, False, False), (128, 16384, 64, False, False, True)]
tv.profile_enable(True)
out = []
for m, k, n, ta, tb, bias in g_cases:
    dt = torch.bfloat16
    a = rnd_mm((k, m) if ta else (m, k), dt, 31)
    b = rnd_mm((n, k) if tb else (k, n), dt, 32)
    ad = a.cuda().t() if ta else a.cuda()
    bd = b.cuda().t() if tb else b.cuda()
    ac = a.t() if ta else a
    bc = b.t() if tb else b
    if bias:
        c = rnd_mm((n,), dt, 33)
        y = torch.addmm(c.cuda(), ad, bd, beta=0.5, alpha=2.0)
        ref = 2.0 * (ac.double() @ bc.double()) + 0.5 * c.double()
    else:
        y = torch.mm(ad, bd)
        ref = ac.double() @ bc.double()
    err = ((y.cpu().double() - ref).norm() / ref.norm()).item()
    out.append([m, k, n, ta, tb, bias, err])
torch.cuda.synchronize()
kernels = [ln.split("\t")[0] for ln in tv.profile().splitlines() if ln]
print("RESULT " + json.dumps({"cases": out, "kernels": kernels, "validation_errors": tv.validation_errors()}))
"""


@pytest.mark.parametrize("kcluster", ["1", "0"])
def test_split_k_forms_match_float64(kcluster):
    r = subprocess.run([sys.executable, "-c", CHILD.replace("ROOT", repr(ROOT))], capture_output=True, text=True,
                       timeout=600, cwd=ROOT, env=dict(os.environ, B2_GEMM_KCLUSTER=kcluster, B2_GEMM_SKINNY="0"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["validation_errors"] == 0
    # pinned off, every split runs the separate reduction kernel; on, the splits whose clusters all fit
    # on the GPU at once (the LoRA down-projection shapes among them) run the cluster form
    if kcluster == "0":
        assert "gemm_splitk_reduce" in res["kernels"] and "gemm_tc_bn128_kcluster" not in res["kernels"]
    else:
        assert "gemm_tc_bn128_kcluster" in res["kernels"], res["kernels"]
    for m, k, n, ta, tb, bias, err in res["cases"]:
        assert err < 4e-3, (kcluster, m, k, n, ta, tb, bias, err)


def test_workspace_only_for_tcgen05_splits():
    """A split-K tcgen05 GEMM asks for its fp32 partial scratch (1024 x 128 x 8192: 8 output tiles, 16 K
    slices of 8 blocks); the LoRA weight-gradient shape of the stacked q/k/v group at 1024 tokens
    (2048 x 48 x 1024) goes to the skinny kernel and asks for none."""
    import ctypes

    import torch_vulkan_b200  # noqa: F401

    class GemmArgs(ctypes.Structure):  # mirrors b2_gemm_args in include/b2rt.h
        _fields_ = ([(n, ctypes.c_void_p) for n in ("a", "b", "c", "bias")] +
                    [(n, ctypes.c_int64) for n in ("M", "N", "K", "batch", "a_sb", "a_sm", "a_sk", "b_sb", "b_sk",
                                                   "b_sn", "c_sb", "c_sm", "c_sn", "bias_sb", "bias_sm", "bias_sn")] +
                    [("alpha", ctypes.c_float), ("beta", ctypes.c_float)] +
                    [(n, ctypes.c_int32) for n in ("dtype", "has_bias", "force_simt", "pad_")] +
                    [("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_int64)])

    lib = ctypes.CDLL(os.path.join(ROOT, "torch_vulkan_b200", "libb2rt.so"))
    lib.b2_gemm_workspace_bytes.argtypes = [ctypes.POINTER(GemmArgs)]
    lib.b2_gemm_workspace_bytes.restype = ctypes.c_uint64
    assert lib.b2rt_init() == 0
    g = GemmArgs()
    g.a, g.b, g.c = 256, 256, 256  # only the layout matters here; nothing is launched
    g.M, g.N, g.K, g.batch = 1024, 128, 8192, 1
    g.a_sm, g.a_sk, g.b_sk, g.b_sn, g.c_sm, g.c_sn = 8192, 1, 128, 1, 128, 1
    g.alpha, g.dtype = 1.0, 1  # B2_BF16
    assert lib.b2_gemm_workspace_bytes(ctypes.byref(g)) == 16 * 1024 * 128 * 4
    g.M, g.N, g.K, g.a_sm, g.b_sk, g.c_sm = 2048, 48, 1024, 1024, 48, 48
    assert lib.b2_gemm_workspace_bytes(ctypes.byref(g)) == 0
