"""Parity at the full shapes the DiT LoRA step runs (BASELINE configs[3] at 1024 image tokens and configs[4] at
4096), against the float64 oracle. These are the code paths the small cases never reach:

* the int8 GEMM's split-K form (reductions of >= 4096 with few output tiles: the fc2 forward and the fc1 dX
  at M = 1024), and the 256x256-tile forms at M = 4096, forward and dX, each compared with
  oracle.int8_linear[_dx] (cases in the style of the reference's tests/test_dequant_int8.py:36-55);
* the fused in-mainloop dequant, checked bit for bit through an identity input: with x = I, each output
  is one product w * 1 accumulated in fp32, so int8_linear(I, q, s) must equal dequant_int8(q, s)^T exactly;
* attention at S = 4096 (configs[4] self-attention) and Sq = 4096 / 1024 against Sk = 512 (cross-attention),
  forward (O and logsumexp) and backward, like the reference's tests/test_fused_attention.py:29-60;
* one full-size configs[3] block: forward and LoRA gradients against a float64 restatement.
"""

import ctypes
import math
import os

import pytest
import torch
import torch.nn.functional as F

import oracle
from tests.helpers import gemm_check, make_int8, rel_err

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OVR = torch.ops.aten._scaled_dot_product_fused_attention_overrideable


class Int8Args(ctypes.Structure):
    # mirrors b2_int8_gemm_args in include/b2rt.h
    _fields_ = [("x", ctypes.c_void_p), ("q", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("x_ld", ctypes.c_int64), ("out_ld", ctypes.c_int64), ("scale_layout", ctypes.c_int32),
                ("transpose_w", ctypes.c_int32), ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_int64),
                ("epilogue", ctypes.c_int32), ("pad_", ctypes.c_int32), ("aux", ctypes.c_void_p), ("aux_ld", ctypes.c_int64),
                ("lora_h", ctypes.c_void_p), ("lora_b", ctypes.c_void_p), ("lora_h_ld", ctypes.c_int64),
                ("lora_b_ld", ctypes.c_int64), ("lora_r", ctypes.c_int32), ("pad2_", ctypes.c_int32)]


@pytest.fixture(scope="module")
def lib():
    import torch_vulkan_b200  # noqa: F401

    L = ctypes.CDLL(os.path.join(ROOT, "torch_vulkan_b200", "libb2rt.so"))
    L.b2_int8_gemm_workspace_bytes.argtypes = [ctypes.POINTER(Int8Args)]
    L.b2_int8_gemm_workspace_bytes.restype = ctypes.c_uint64
    assert L.b2rt_init() == 0
    return L


def int8_workspace_bytes(L, M, N, K, transpose, layout=1):
    a = Int8Args()
    a.M, a.N, a.K, a.x_ld = M, N, K, (N if transpose else K)
    a.out_ld = K if transpose else N
    a.scale_layout, a.transpose_w = layout, int(transpose)
    return int(L.b2_int8_gemm_workspace_bytes(ctypes.byref(a)))


def dit_weights(N, K, seed):
    """int8 weight [N, K] uniform in [-127, 127] with a per-row fp32 scale U[1e-3, 1e-2] (configs[0]'s recipe)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    s = torch.rand(N, generator=g) * 9e-3 + 1e-3
    return q, s


# (M, N, K, split): N = rows of q (output features of the forward), K = its input features.
# split = the plan must divide the reduction (fc2 forward: K = 8192; fc1 dX: N = 8192, both at M = 1024).
FWD = [(1024, 2048, 8192, True), (4096, 2048, 2048, False), (4096, 8192, 2048, False), (4096, 2048, 8192, False)]
DX = [(1024, 8192, 2048, True), (4096, 2048, 2048, False), (4096, 8192, 2048, False), (4096, 2048, 8192, False)]


@pytest.mark.parametrize("M,N,K,split", FWD)
def test_int8_forward_at_dit_shapes(lib, M, N, K, split):
    import torch_vulkan_b200 as tv

    q, s = dit_weights(N, K, seed=M + N + K)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.02).to(torch.bfloat16)
    assert (int8_workspace_bytes(lib, M, N, K, False) > 0) == split
    out = tv.int8_linear(x.cuda(), q.cuda(), s.cuda(), b.cuda())
    ref = oracle.int8_linear(x, q, s, b)
    gemm_check(out, ref, torch.bfloat16, K)
    assert rel_err(out, ref) < 4e-3  # bf16 output rounding only: a lost or doubled K slice is far above this
    assert tv.validation_errors() == 0


@pytest.mark.parametrize("M,N,K,split", DX)
def test_int8_dx_at_dit_shapes(lib, M, N, K, split):
    q, s = dit_weights(N, K, seed=M + N + K + 1)
    dy = torch.randn(M, N, generator=torch.Generator().manual_seed(8)).to(torch.bfloat16)
    assert (int8_workspace_bytes(lib, M, N, K, True) > 0) == split
    dx = torch.ops.b2.int8_linear_dx(dy.cuda(), q.cuda(), s.cuda())
    ref = oracle.int8_linear_dx(dy, q, s)
    gemm_check(dx, ref, torch.bfloat16, N)
    assert rel_err(dx, ref) < 4e-3


def same_values(a, b):
    """Bitwise equality of two bf16 tensors, treating +0 and -0 as the same value."""
    a, b = a.cpu().float(), b.cpu().float()
    return torch.equal(a, b)


@pytest.mark.parametrize("layout", ["row_f32", "block64_bf16"])
@pytest.mark.parametrize("M,N,K", [(2048, 6144, 2048), (1024, 2048, 8192)])
def test_fused_dequant_is_bit_exact(lib, layout, M, N, K):
    """int8_linear(I[:M], q, s) == dequant_int8(q, s)^T[:M]: every output is one product 1 * w~ (the rest
    are exact zeros), so any difference is a difference in the in-shared-memory dequantised weight."""
    import torch_vulkan_b200 as tv

    if layout == "row_f32":
        q, s = dit_weights(N, K, seed=N + K)
    else:
        q, s = make_int8(N, K, seed=N + K)
    eye = torch.eye(M, K, dtype=torch.bfloat16)
    w = oracle.dequant_int8(q, s, torch.bfloat16)
    y = tv.int8_linear(eye.cuda(), q.cuda(), s.cuda())
    assert same_values(y, w.t()[:M]), "forward: in-mainloop dequant differs from dequant_int8"
    # transposed (dX) form: I[:M, :N] @ W~ = the first M rows of W~
    Mt = min(M, N)
    dy = torch.eye(Mt, N, dtype=torch.bfloat16)
    dx = torch.ops.b2.int8_linear_dx(dy.cuda(), q.cuda(), s.cuda())
    assert same_values(dx, w[:Mt]), "dX: in-mainloop dequant differs from dequant_int8"
    assert tv.validation_errors() == 0


# ---- attention at the configs[3]/[4] sizes ---------------------------------------------------------

def attn_case(B, H, Sq, Sk, D, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda S: torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)  # noqa: E731
    return mk(Sq), mk(Sk), mk(Sk), mk(Sq)


@pytest.mark.parametrize("Sq,Sk", [(4096, 4096), (4096, 512), (1024, 512)])
def test_attention_at_dit_sizes(Sq, Sk):
    """B1 H16 D128 bf16 forward (O, logsumexp) and backward; the float64 oracle runs on heads 0 and 15."""
    import torch_vulkan_b200 as tv

    tv.set_fused_attention("on")
    try:
        q, k, v, do = attn_case(1, 16, Sq, Sk, 128, seed=Sq + Sk)
        qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
        o, lse = OVR(qd.detach(), kd.detach(), vd.detach())[:2]
        o2 = F.scaled_dot_product_attention(qd, kd, vd)
        o2.backward(do.cuda())
        assert torch.equal(o.cpu(), o2.detach().cpu())
        hs = [0, 15]
        sl = lambda t: t[:, hs].contiguous()  # noqa: E731
        o64, lse64 = oracle.sdpa_fwd(sl(q), sl(k), sl(v))
        dq64, dk64, dv64 = oracle.sdpa_bwd(sl(q), sl(k), sl(v), sl(do))
        assert rel_err(sl(o.cpu()), o64) < 2e-2
        lse_err = (sl(lse.cpu()).double() - lse64).abs().max().item()
        assert lse_err <= 1e-3 * max(1.0, lse64.abs().max().item()), lse_err
        for name, got, ref in (("dq", qd.grad, dq64), ("dk", kd.grad, dk64), ("dv", vd.grad, dv64)):
            e = rel_err(sl(got.cpu()), ref)
            assert e < 2e-2, (name, e)
        assert tv.validation_errors() == 0
    finally:
        tv.set_fused_attention("auto")


# ---- one full-size configs[3] block --------------------------------------------------------------

def test_config4_block_forward_and_lora_grads_match_float64():
    """BASELINE configs[3] at full size (hidden 2048, 16 heads, 1024 image + 512 text tokens, MLP 8192): the
    block's output and every LoRA gradient against a float64 CPU restatement with the same weights."""
    from tests.test_dit import ref_block, rel
    from torch_vulkan_b200.dit import DiTBlock, synthetic_batch

    blk = DiTBlock(seed=5)
    x, text, cond, target = synthetic_batch(seed=6)
    out = blk(x, text, cond)
    F.mse_loss(out.float(), target.float()).backward()
    ref_params = {n: p.detach().cpu().double().requires_grad_(True) for n, p in blk.named_parameters()}

    class View:
        pass

    def mkview(mod, prefix):
        v = View()
        for k2, sub in mod._modules.items():
            setattr(v, k2, mkview(sub, prefix + k2 + "."))
        for k2, b in mod._buffers.items():
            setattr(v, k2, b)
        for k2 in mod._parameters:
            setattr(v, k2, ref_params[prefix + k2])
        for k2 in ("scale", "h", "heads", "d"):
            if k2 in mod.__dict__:
                setattr(v, k2, mod.__dict__[k2])
        return v

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out64 = ref_block(mkview(blk, ""), x, text, cond)
    e_out = rel(out, out64)
    assert e_out < 2e-2, e_out
    F.mse_loss(out64, target.cpu().double()).backward()
    errs = {n: rel(p.grad, ref_params[n].grad) for n, p in blk.named_parameters() if "lora_" in n}
    assert len(errs) == 16
    worst = max(errs.items(), key=lambda kv: kv[1])
    assert worst[1] < 2e-2, (worst, errs)
    assert not math.isnan(sum(errs.values()))
