"""The slab allocator on the device (the reference tests its runtime allocator on a real device,
vkrt/tests/basic.rs:14-182): use_slab_allocator() routes every CUDA tensor of a fresh process through
b2_malloc / b2_free, then a full-size configs[3] DiT block LoRA step runs on it. Checked: live bytes and
slab counts follow the allocations, a block freed on one stream is reused on another only behind a
cross-stream wait, and the training step computes the same loss as with PyTorch's caching allocator."""

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
import torch.nn.functional as F
import torch_vulkan_b200 as tv
use_slab = bool(USE_SLAB)
if use_slab:
    tv.use_slab_allocator()
torch.cuda.set_device(0)
out = {}
if use_slab:
    live0, blocks0 = tv.live_bytes(), tv.live_blocks()
    t = torch.empty(4 << 20, dtype=torch.uint8, device="cuda")
    out["live_delta"] = tv.live_bytes() - live0
    out["blocks_delta"] = tv.live_blocks() - blocks0
    out["slabs"] = tv.slab_count()
    # a block freed on stream s1 and requested again on s2 is the same memory, ordered by a wait
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(s1):
        a = torch.empty(3 << 20, dtype=torch.uint8, device="cuda")
        a.fill_(7)
    pa = a.data_ptr()
    waits0 = tv.stats()["cross_stream_waits"]
    del a
    with torch.cuda.stream(s2):
        b = torch.empty(3 << 20, dtype=torch.uint8, device="cuda")
        b.fill_(9)
    out["reused"] = b.data_ptr() == pa
    out["waits"] = tv.stats()["cross_stream_waits"] - waits0
    torch.cuda.synchronize()
    out["b_ok"] = bool((b == 9).all().item())
    del t, b
    torch.cuda.synchronize()
    out["live_after_free"] = tv.live_bytes() - live0
from torch_vulkan_b200.dit import DiTStack, LoRATrainer, synthetic_batch
model = DiTStack(blocks=1, seed=0)
tr = LoRATrainer(model, lr=1e-3, fused_optimizer=True)
batch = synthetic_batch(seed=1)
losses = [float(tr.step(*batch).item()) for _ in range(3)]
torch.cuda.synchronize()
out["losses"] = losses
if use_slab:
    out["peak"] = tv.peak_live_bytes()
    out["slabs_after_step"] = tv.slab_count()
    out["reserved"] = tv.reserved_bytes()
out["validation_errors"] = tv.validation_errors()
print("RESULT " + json.dumps(out))
"""


def run_child(use_slab):
    code = CHILD.replace("ROOT", repr(ROOT)).replace("USE_SLAB", "1" if use_slab else "0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def test_slab_allocator_serves_a_dit_step():
    slab = run_child(True)
    assert slab["live_delta"] == 4 << 20 and slab["blocks_delta"] == 1
    assert slab["slabs"] >= 1
    assert slab["reused"] and slab["waits"] >= 1 and slab["b_ok"]
    assert slab["live_after_free"] == 0
    assert slab["peak"] > 256 << 20  # the block's int8 weights (63 M), activations and gradients
    assert slab["slabs_after_step"] >= 1 and slab["reserved"] >= slab["peak"]
    assert slab["validation_errors"] == 0
    ref = run_child(False)
    for a, b in zip(slab["losses"], ref["losses"]):
        assert abs(a - b) <= 1e-3 * abs(b), (slab["losses"], ref["losses"])
    assert slab["losses"][-1] < slab["losses"][0]
