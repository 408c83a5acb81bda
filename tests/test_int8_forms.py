"""The two forms of the fused int8 GEMM against the float64 oracle: CTA pairs (cta_group::2, the two CTAs
of a cluster sharing each M = 256 MMA and each dequantising half of the B tile) and single CTAs. The
launch plan picks a form per shape; B2_INT8_CG=1|2 pins it for a whole process, so each form runs the
same cases in its own child process: forward with bias (per-row fp32 and block-64 bf16 scales), the
transposed dX form, ragged edges, and the split-K shapes of the DiT block (fc2 forward, fc1 dX). Two more
children pin one pair tile (B2_INT8_TILE) for every shape."""

import json
import os
import subprocess
import sys

import pytest

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

def row_weights(N, K, g):
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    return q, torch.rand(N, generator=g) * 9e-3 + 1e-3

g = torch.Generator().manual_seed(11)
out = []
# (M, N, K, scales): forward x[M,K] @ W~[N,K]^T + b, then dX = dY[M,N] @ W~
for M, N, K, lay in [(1024, 6144, 2048, "row"), (300, 520, 272, "row"), (512, 384, 320, "block64"),
                     (1024, 2048, 8192, "row"), (1024, 8192, 2048, "row"), (4096, 2048, 2048, "row"),
                     (130, 96, 64, "block64")]:
    q, s = row_weights(N, K, g) if lay == "row" else make_int8(N, K, seed=N + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    y = tv.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda())
    e_f = rel(y, oracle.int8_linear(x, q, s, b))
    dy = torch.randn(M, N, generator=g).to(torch.bfloat16)
    dx = torch.ops.b2.int8_linear_dx(dy.cuda(), q.cuda(), s.cuda())
    e_d = rel(dx, oracle.int8_linear_dx(dy, q, s))
    out.append([M, N, K, lay, e_f, e_d])
torch.cuda.synchronize()
print("RESULT " + json.dumps({"cases": out, "validation_errors": tv.validation_errors()}))
"""


@pytest.mark.parametrize("cg,tile", [("1", None), ("2", None), ("2", "128x1"), ("2", "256x1")])
def test_int8_kernel_form_matches_oracle(cg, tile):
    env = dict(os.environ, B2_INT8_CG=cg)
    if tile:  # every shape on one tile form (256 x 128 or 256 x 256 pair tiles, no split-K)
        env["B2_INT8_TILE"] = tile
    r = subprocess.run([sys.executable, "-c", CHILD.replace("ROOT", repr(ROOT))], capture_output=True, text=True,
                       timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads([l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1][len("RESULT "):])
    assert res["validation_errors"] == 0
    for M, N, K, lay, e_f, e_d in res["cases"]:
        # bf16 output rounding only (relative L2 ~1e-3): a wrong B half or a lost K slice is far above
        assert e_f < 4e-3 and e_d < 4e-3, (cg, tile, M, N, K, lay, e_f, e_d)
