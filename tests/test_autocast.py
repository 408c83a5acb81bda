"""The autocast contract of the hot path (the reference's AutocastPrivateUse1 lists, csrc/shim.cpp:401-415):
under torch.autocast("cuda", torch.bfloat16), linear/mm/bmm/addmm/baddbmm/matmul and scaled-dot-product
attention reach their kernels in bf16, while layer_norm, softmax and mse_loss reach theirs in fp32. A
dispatch-mode recorder sees each ATen call after autocast has cast its inputs, i.e. the dtypes the CUDA
kernels registered by this package receive."""

import pytest
import torch
import torch.nn.functional as F
from torch.utils._python_dispatch import TorchDispatchMode
from torch.utils._pytree import tree_leaves

pytestmark = pytest.mark.gpu


class Recorder(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.calls = []

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        dts = [t.dtype for t in tree_leaves((args, kwargs)) if isinstance(t, torch.Tensor) and t.is_floating_point()]
        self.calls.append((func.__name__ if hasattr(func, "__name__") else str(func), str(func.overloadpacket), dts))
        return func(*args, **kwargs)


def seen(rec, packet):
    return [d for _, p, d in rec.calls if p == packet]


def test_autocast_lists_match_the_reference():
    import torch_vulkan_b200 as tv

    tv.reset_counts()
    tv.set_fused_attention("on")
    g = torch.Generator().manual_seed(0)
    mk = lambda *s: torch.randn(*s, generator=g).cuda()  # noqa: E731  (fp32 inputs)
    x, w, b = mk(64, 128), mk(256, 128), mk(256)
    a3, b3, c3 = mk(4, 64, 96), mk(4, 96, 32), mk(4, 64, 32)
    q, k, v = mk(1, 2, 128, 64), mk(1, 2, 128, 64), mk(1, 2, 128, 64)
    rec = Recorder()
    try:
        with torch.autocast("cuda", dtype=torch.bfloat16), rec:
            y_lin = F.linear(x, w, b)
            y_mm = torch.mm(x, w.t())
            y_bmm = torch.bmm(a3, b3)
            y_baddbmm = torch.baddbmm(c3, a3, b3)
            y_matmul = torch.matmul(a3, b3)
            y_attn = F.scaled_dot_product_attention(q, k, v)
            h = y_lin  # bf16 activation into the fp32 ops
            y_ln = F.layer_norm(h, (256,))
            y_sm = torch.softmax(h, -1)
            loss = F.mse_loss(h, torch.zeros_like(h))
    finally:
        tv.set_fused_attention("auto")
    for t in (y_lin, y_mm, y_bmm, y_baddbmm, y_matmul, y_attn):
        assert t.dtype == torch.bfloat16
    for t in (y_ln, y_sm, loss):
        assert t.dtype == torch.float32
    for packet in ("aten.addmm", "aten.mm", "aten.bmm", "aten.baddbmm",
                   "aten._scaled_dot_product_fused_attention_overrideable"):
        calls = seen(rec, packet)
        assert calls, (packet, [c[1] for c in rec.calls])
        assert all(d == torch.bfloat16 for dts in calls for d in dts), (packet, calls)
    for packet in ("aten.native_layer_norm", "aten._softmax", "aten.mse_loss"):
        calls = seen(rec, packet)
        assert calls, (packet, [c[1] for c in rec.calls])
        assert all(d == torch.float32 for dts in calls for d in dts), (packet, calls)
    kc = tv.kernel_counts()
    for op in ("aten::addmm", "aten::mm", "aten::bmm", "aten::baddbmm",
               "aten::_scaled_dot_product_fused_attention_overrideable", "aten::native_layer_norm", "aten::_softmax"):
        assert kc.get(op, 0) >= 1, (op, kc)
    assert tv.fallback_counts() == {}
