"""The synthetic DiT LoRA block on the hot-path kernels vs a float64 CPU restatement of
the same block built from the oracle (dequantised int8 weights, float64 attention/LayerNorm)."""

import math

import pytest
import torch
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu


def ref_block(blk, x, text, cond):
    """float64 CPU restatement of DiTBlock.forward with the same weights."""
    def d(t):  # float64 CPU copy; float64 CPU leaves (the gradient test's parameters) pass through
        return t if (t.device.type == "cpu" and t.dtype == torch.float64) else t.detach().cpu().double()

    def lin(mod, t):
        w = oracle.dequant_int8(mod.q.cpu(), mod.scale.cpu(), torch.bfloat16).double()
        y = t @ w.t()
        return y + d(mod.bias) if mod.bias is not None else y

    def lora(mod, t):
        return lin(mod.base, t) + (t @ d(mod.lora_down).t()) @ d(mod.lora_up).t() * mod.scale

    def attn(tq, tk, tv, qp, kp, vp, op):
        B, S, _ = tq.shape
        Skv = tk.shape[1]
        q = lora(qp, tq).view(B, S, blk.heads, blk.d).transpose(1, 2)
        k = lora(kp, tk).view(B, Skv, blk.heads, blk.d).transpose(1, 2)
        v = lora(vp, tv).view(B, Skv, blk.heads, blk.d).transpose(1, 2)
        o, _ = oracle.sdpa_fwd(q, k, v)
        return lora(op, o.transpose(1, 2).reshape(B, S, blk.h))

    x, text, cond = d(x), d(text), d(cond)
    mod = lin(blk.ada, F.silu(cond)).unsqueeze(1).chunk(9, dim=-1)
    sh1, sc1, g1, sh2, sc2, g2, sh3, sc3, g3 = mod

    def modln(t, sh, sc):
        return oracle.layer_norm(t, (blk.h,), eps=1e-6)[0] * (1 + sc) + sh

    h = modln(x, sh1, sc1)
    x = x + g1 * attn(h, h, h, blk.q, blk.k, blk.v, blk.o)
    h = modln(x, sh2, sc2)
    x = x + g2 * attn(h, text, text, blk.cq, blk.ck, blk.cv, blk.co)
    h = modln(x, sh3, sc3)
    return x + g3 * lin(blk.fc2, F.gelu(lin(blk.fc1, h), approximate="tanh"))


def small_block():
    from torch_vulkan_b200.dit import DiTBlock, synthetic_batch

    blk = DiTBlock(hidden=256, heads=2, text_dim=128, mlp=512, seed=3)
    x, text, cond, target = synthetic_batch(tokens=128, text_tokens=64, hidden=256, text_dim=128, seed=4)
    return blk, x, text, cond, target


def rel(a, b):
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return ((a - b).norm() / (b.norm() + 1e-30)).item()


def test_block_forward_matches_float64_restatement():
    import torch_vulkan_b200 as tv

    blk, x, text, cond, _ = small_block()
    tv.reset_counts()
    out = blk(x, text, cond)
    assert rel(out, ref_block(blk, x, text, cond)) < 2e-2
    kc = tv.kernel_counts()
    for op in ("b2::int8_linear", "aten::_scaled_dot_product_fused_attention_overrideable", "aten::native_layer_norm", "aten::mm"):
        assert kc.get(op, 0) > 0, (op, kc)


def test_block_lora_gradients_match_float64_autograd():
    blk, x, text, cond, target = small_block()
    out = blk(x, text, cond)
    F.mse_loss(out.float(), target.float()).backward()
    # float64 reference gradients through the restated block
    names = [n for n, _ in blk.named_parameters() if "lora_" in n]
    ref_params = {}
    for n, p in blk.named_parameters():
        ref_params[n] = p.detach().cpu().double().requires_grad_(True)
    saved = {n: p.data for n, p in blk.named_parameters()}
    # swap in float64 leaves on a CPU view of the module for the reference pass
    import types

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

    rb = mkview(blk, "")
    out64 = ref_block(rb, x, text, cond)
    F.mse_loss(out64, target.cpu().double()).backward()
    for n in names:
        p = dict(blk.named_parameters())[n]
        e = rel(p.grad, ref_params[n].grad)
        assert e < 5e-2, (n, e)
    del saved, types


def test_config4_training_step_runs_and_learns():
    """full-size block, 1024 tokens; AdamW(foreach=False) over the LoRA parameters."""
    import torch_vulkan_b200 as tv
    from torch_vulkan_b200.dit import DiTStack, make_optimizer, synthetic_batch

    model = DiTStack(blocks=1, seed=0)
    x, text, cond, target = synthetic_batch(seed=1)
    opt = make_optimizer(model.lora_parameters(), lr=1e-3)
    tv.reset_counts()
    losses = []
    for _ in range(4):
        opt.zero_grad(set_to_none=True)
        loss = F.mse_loss(model(x, text, cond).float(), target.float())
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert all(math.isfinite(v) for v in losses)
    assert losses[-1] < losses[0], losses
    kc = tv.kernel_counts()
    # the block's attention backward writes into the stacked projection gradients (b2::sdpa_bwd_into)
    for op in ("aten::addcmul_", "aten::addcdiv_", "aten::lerp_.Scalar", "b2::int8_linear_dx", "b2::sdpa_bwd_into"):
        assert kc.get(op, 0) > 0, (op, kc)


def test_graphed_step_matches_eager_step():
    """LoRATrainer.graphed (forward + backward replayed as a CUDA graph) produces the same loss and LoRA
    parameters as the eager step from identical starting states."""
    from torch_vulkan_b200.dit import DiTStack, LoRATrainer, synthetic_batch

    def run(graphed):
        model = DiTStack(blocks=2, seed=0, hidden=256, heads=2, text_dim=128, mlp=512)
        tr = LoRATrainer(model, lr=1e-3, fused_optimizer=True)
        batch = synthetic_batch(tokens=128, text_tokens=64, hidden=256, text_dim=128, seed=7)
        step = tr.graphed(*batch, warmup=2) if graphed else None
        if not graphed:
            for _ in range(2):
                tr.step(*batch)
        losses = [float((step() if graphed else tr.step(*batch)).item()) for _ in range(3)]
        return losses, torch.cat([p.detach().float().flatten() for p in tr.params]).cpu()

    le, pe = run(False)
    lg, pg = run(True)
    assert max(abs(a - b) / abs(a) for a, b in zip(le, lg)) < 1e-3, (le, lg)
    assert rel(pg, pe) < 1e-3


def test_stacked_lora_storage_follows_parameter_updates():
    """The stacked q/k/v and text k/v groups keep their LoRA matrices in stacked storage (each module's
    Parameter a view of it) and refresh the block-diagonal up-projection every forward: in-place updates of
    the Parameters (as an optimizer makes them) and fused-AdamW steps reach the next forward of the group,
    which matches a float64 restatement (dequantised base + x A^T B^T) built from the same Parameters."""
    from torch_vulkan_b200.dit import DiTStack, LoRATrainer

    def ref_proj(mod, t):
        t = t.detach().cpu().double()
        w = oracle.dequant_int8(mod.base.q.cpu(), mod.base.scale.cpu(), torch.bfloat16).double()
        y = t @ w.t() + mod.base.bias.detach().cpu().double()
        lo = (t @ mod.lora_down.detach().cpu().double().t()) @ mod.lora_up.detach().cpu().double().t()
        return y + lo * mod.scale

    def check(b, text, h):
        for name, inp, mods in (("qkv", h, (b.q, b.k, b.v)), ("ckv", text, (b.ck, b.cv))):
            outs = b._stacked(name, inp, mods)
            for o, m in zip(outs, mods):
                assert rel(o, ref_proj(m, inp)) < 1e-2, name
        return [o.detach().clone() for o in b._stacked("ckv", text, (b.ck, b.cv))]

    blk, x, text, cond, target = small_block()
    grp = blk._lora_groups["qkv"]
    assert blk.k.lora_up.data_ptr() == grp.b[grp.n:].data_ptr() and blk.k.lora_up.is_contiguous()
    with torch.no_grad():
        before = check(blk, text, x)
        for m in (blk.k, blk.cv):
            m.lora_up.add_(0.2 * torch.randn_like(m.lora_up))
            m.lora_down.mul_(2.0)
        after = check(blk, text, x)
    assert rel(after[1], before[1]) > 1e-2  # the update reached the text-side v projection

    model = DiTStack(blocks=1, seed=3, hidden=256, heads=2, text_dim=128, mlp=512)
    tr = LoRATrainer(model, lr=1e-2, fused_optimizer=True)
    with torch.no_grad():
        start = check(model.blocks[0], text, x)
    for _ in range(2):
        tr.step(x, text, cond, target)
    with torch.no_grad():
        moved = check(model.blocks[0], text, x)
    assert rel(moved[0], start[0]) > 1e-4  # the optimizer's updates reached the next forward


def test_stacked_attention_gradients_match_split_views():
    """The DiT block's attention over column blocks of the stacked projection outputs (self-attention: one
    [B, S, 3 H D] q/k/v tensor; cross-attention: q [B, S, H D] and a stacked [B, Sk, 2 H D] k/v tensor)
    writes dq, dk, dv straight into blocks of one gradient buffer; output and gradients equal those of
    F.scaled_dot_product_attention over split views (the same kernels, gradients concatenated by autograd)."""
    from torch_vulkan_b200.dit import _StackedSDPA

    g = torch.Generator().manual_seed(12)
    B, S, Sk, H, D = 1, 384, 192, 2, 128
    hd = H * D

    def heads(t, S_):
        return t.view(B, S_, H, D).transpose(1, 2)

    # self-attention: q, k, v = blocks 0, 1, 2 of one tensor
    qkv = torch.randn(B, S, 3 * hd, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    o = _StackedSDPA.apply(qkv, qkv, H, hd, 0, hd, 2 * hd)
    go = torch.randn(o.shape, generator=g).to(torch.bfloat16).cuda()
    o.backward(go)
    ref = qkv.detach().clone().requires_grad_(True)
    q, k, v = (heads(t, S) for t in ref.split(hd, dim=-1))
    o_ref = F.scaled_dot_product_attention(q, k, v)
    o_ref.backward(go)
    assert rel(o, o_ref) < 1e-3 and rel(qkv.grad, ref.grad) < 1e-3

    # cross-attention: q from its own tensor, k and v from one stacked tensor
    qt = torch.randn(B, S, hd, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    kv = torch.randn(B, Sk, 2 * hd, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    o = _StackedSDPA.apply(qt, kv, H, hd, 0, 0, hd)
    go = torch.randn(o.shape, generator=g).to(torch.bfloat16).cuda()
    o.backward(go)
    qr, kvr = qt.detach().clone().requires_grad_(True), kv.detach().clone().requires_grad_(True)
    kr, vr = (heads(t, Sk) for t in kvr.split(hd, dim=-1))
    o_ref = F.scaled_dot_product_attention(heads(qr, S), kr, vr)
    o_ref.backward(go)
    assert rel(o, o_ref) < 1e-3 and rel(qt.grad, qr.grad) < 1e-3 and rel(kv.grad, kvr.grad) < 1e-3
