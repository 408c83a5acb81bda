"""Synthetic DiT block with LoRA on frozen int8 base weights — the training workload of BASELINE configs[3]
(one block, 1024 image tokens) and configs[4] (a 28-block stack at 4096 tokens, data-parallel).

Built from the BASELINE description (the Anima model code of the reference's sd-scripts fork is not part of
the reference repository): hidden 2048, 16 heads x 128, self-attention + cross-attention to 512 text tokens
of width 1024, GELU MLP 2048 -> 8192 -> 2048, adaLN-modulated (affine-free) LayerNorm, LoRA rank 16 /
alpha 16 on the q/k/v/o linears of both attentions (the module layout of tests/anima_on_vk.py:43-48 of the
reference), every base linear frozen as int8 with a per-output-row fp32 scale. The hot operators run on
this package's kernels: int8 linears on the fused dequant GEMM (`b2::int8_linear_fwd/dx`) with the LoRA
up-projection as one more reduction block of it (`tv.int8_lora_linear`; the rank-r down-projection and the
LoRA weight gradients on `mm`), the MLP with GELU and its derivative in the int8 GEMM epilogues
(`tv.int8_mlp`), attention on the fused tcgen05 SDPA, LayerNorm on the row kernels, AdamW(foreach=False) on
`addcmul_/addcdiv_/lerp_` or the multi-tensor AdamW kernel. `DiTStack.enable_block_swap` streams the frozen
weights of the last blocks from pinned host memory (torch_vulkan_b200.offload).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.utils.checkpoint
import torch.nn.functional as F

import torch_vulkan_b200 as tv


class Int8Linear(nn.Module):
    """Frozen int8 weight [out, in] with a per-output-row fp32 scale; y = x (W*s)^T + b."""

    def __init__(self, in_f, out_f, bias=True, std=0.02, generator=None, device="cuda"):
        super().__init__()
        # random init std 0.02, quantised per output row (the set-up runs on the device; it is not timed)
        w = torch.randn(out_f, in_f, generator=generator, device=generator.device if generator else device) * std
        w = w.to(device)
        scale = w.abs().amax(1).clamp_min(1e-8) / 127.0
        q = torch.round(w / scale[:, None]).clamp_(-127, 127).to(torch.int8)
        del w
        self.register_buffer("q", q)
        self.register_buffer("scale", scale.float())
        self.register_buffer("bias", torch.zeros(out_f, dtype=torch.bfloat16, device=device) if bias else None)

    def forward(self, x):
        return tv.int8_linear(x, self.q, self.scale, self.bias)


class LoRAInt8Linear(nn.Module):
    """Frozen int8 base + trainable LoRA: y = base(x) + (x A^T) B^T * alpha / r."""

    def __init__(self, in_f, out_f, rank=16, alpha=16.0, generator=None, device="cuda", dtype=torch.bfloat16):
        super().__init__()
        self.base = Int8Linear(in_f, out_f, bias=True, generator=generator, device=device)
        gdev = generator.device if generator else device
        self.lora_down = nn.Parameter((torch.randn(rank, in_f, generator=generator, device=gdev) / math.sqrt(in_f)).to(dtype).to(device))
        # non-zero up-projection so the LoRA path carries gradient and signal from the first step
        self.lora_up = nn.Parameter((torch.randn(out_f, rank, generator=generator, device=gdev) * 0.02).to(dtype).to(device))
        self.scale = alpha / rank

    def forward(self, x):
        # the up-projection (h B^T) * alpha / r is one more reduction block of the int8 GEMM
        b = self.lora_up if self.scale == 1.0 else self.lora_up * self.scale
        return tv.int8_lora_linear(x, self.base.q, self.base.scale, self.base.bias, self.lora_down, b)


class LoRAGroup:
    """The LoRA matrices of several LoRAInt8Linear modules that read the same input, kept in stacked storage:
    the modules' lora_down Parameters are row blocks of one [G*r, in] matrix and their lora_up Parameters
    row blocks of one [G*N, r] matrix (every Parameter stays contiguous, so optimizers see nothing new),
    plus the block-diagonal [G*N, G*r] up-projection the int8 GEMM's LoRA block reads, refreshed in place
    from the stacked up matrices by one copy per forward. No per-step cat / block_diag / gradient copies."""

    def __init__(self, mods):
        self.mods = list(mods)
        self.g = len(mods)
        self.r = mods[0].lora_down.shape[0]
        self.n = mods[0].lora_up.shape[0]
        self.scale = mods[0].scale
        assert all(m.lora_down.shape[0] == self.r and m.lora_up.shape == (self.n, self.r) and m.scale == self.scale
                   and m.lora_down.shape[1] == mods[0].lora_down.shape[1] for m in mods)
        with torch.no_grad():
            self.a = torch.cat([m.lora_down.detach() for m in mods], 0)   # [G*r, in]
            self.b = torch.cat([m.lora_up.detach() for m in mods], 0)     # [G*N, r]
            self.b_bd = torch.zeros(self.g * self.n, self.g * self.r, dtype=self.b.dtype, device=self.b.device)
        for i, m in enumerate(mods):
            m.lora_down = nn.Parameter(self.a[i * self.r:(i + 1) * self.r])
            m.lora_up = nn.Parameter(self.b[i * self.n:(i + 1) * self.n])

    def diag_blocks(self, full: torch.Tensor) -> torch.Tensor:
        """[G*N, r] stack of the diagonal [N, r] blocks of a [G*N, G*r] matrix (one strided copy)."""
        out = torch.empty(self.g * self.n, self.r, dtype=full.dtype, device=full.device)
        out.view(self.g, self.n, self.r).copy_(full.view(self.g, self.n, self.g, self.r).diagonal(dim1=0, dim2=2).permute(2, 0, 1))
        return out

    def refresh(self):
        """b_bd's diagonal blocks <- B_i * alpha / r (one strided copy; the off-diagonal blocks stay zero)."""
        with torch.no_grad():
            diag = self.b_bd.view(self.g, self.n, self.g, self.r).diagonal(dim1=0, dim2=2)  # [N, r, G]
            diag.copy_(self.b.view(self.g, self.n, self.r).permute(1, 2, 0))
            if self.scale != 1.0:
                diag.mul_(self.scale)


class _StackedInt8LoRA(torch.autograd.Function):
    """y = x W~^T + bias + (x A^T) B_bd^T for a LoRAGroup (W~ the stacked frozen int8 bases); gradients for x
    and for every module's lora_down / lora_up, the latter as contiguous row blocks of two stacked GEMM
    results (one strided copy pulls the diagonal blocks out of dB)."""

    @staticmethod
    def forward(ctx, x, q, scale, bias, grp, *params):
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        h = torch.mm(x2, grp.a.t())  # the rank-r down-projections of every module, one GEMM
        y = torch.ops.b2.int8_lora_fwd(x2, q, scale, bias, h, grp.b_bd)
        ctx.save_for_backward(x2, q, scale, h)
        ctx.grp, ctx.x_shape = grp, x.shape
        return y.view(*x.shape[:-1], q.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, q, scale, h = ctx.saved_tensors
        grp = ctx.grp
        gy2 = gy.reshape(-1, gy.shape[-1])
        if not gy2.is_contiguous():
            gy2 = gy2.contiguous()
        dh = torch.mm(gy2, grp.b_bd)  # [rows, G*r] (alpha / r included)
        gx = None
        if ctx.needs_input_grad[0]:  # dy W~ + dh A in one GEMM
            gx = torch.ops.b2.int8_lora_dx(gy2, q, scale, dh, grp.a).view(ctx.x_shape)
        ga = torch.mm(dh.t(), x2)  # [G*r, in]: row block i is module i's lora_down gradient
        gb = grp.diag_blocks(torch.mm(gy2.t(), h))  # [G*N, G*r] product: only the diagonal blocks are used
        if grp.scale != 1.0:
            gb.mul_(grp.scale)
        gdown = [ga[i * grp.r:(i + 1) * grp.r] for i in range(grp.g)]
        gup = [gb[i * grp.n:(i + 1) * grp.n] for i in range(grp.g)]
        return (gx, None, None, None, None, *gdown, *gup)


def stacked_lora_forward(x, q, scale, bias, grp: LoRAGroup, whole=False):
    """LoRAInt8Linear.forward of the modules of a LoRAGroup (they read the same input x), with their frozen
    int8 bases stacked in (q, scale, bias): one down-projection GEMM over the stacked A_i, then one int8
    GEMM whose last reduction block adds the up-projection over the block-diagonal B_i (backward: one dX
    GEMM that also adds dh @ A, and one GEMM each for dh, dA and dB, instead of one of each per module).
    Returns one [..., out_i] view per module, or (whole=True) the stacked [..., sum out_i] output."""
    grp.refresh()
    params = [m.lora_down for m in grp.mods] + [m.lora_up for m in grp.mods]
    out = _StackedInt8LoRA.apply(x, q, scale, bias, grp, *params)
    if whole:
        return out
    return out.split([m.base.q.shape[0] for m in grp.mods], dim=-1)


class _StackedSDPA(torch.autograd.Function):
    """softmax(q k^T / sqrt(d)) v with q, k, v taken as hd-wide column blocks (at q_off, k_off, v_off) of
    projection outputs [B, S, *] (the stacked q/k/v output for self-attention; the q output and the stacked
    k/v output for cross-attention), on the fused attention kernels. The backward writes dq, dk, dv straight
    into the matching column blocks of one gradient buffer per input (b2::sdpa_bwd_into), so the stacked
    projections receive their gradient without a concatenation."""

    @staticmethod
    def _view(t, off, heads, hd):
        B, S, _ = t.shape
        return t[..., off:off + hd].view(B, S, heads, hd // heads).transpose(1, 2)

    @staticmethod
    def forward(ctx, qt, kvt, heads, hd, q_off, k_off, v_off):
        vw = _StackedSDPA._view
        q, k, v = vw(qt, q_off, heads, hd), vw(kvt, k_off, heads, hd), vw(kvt, v_off, heads, hd)
        o, lse = torch.ops.aten._scaled_dot_product_fused_attention_overrideable(q, k, v)[:2]
        ctx.save_for_backward(qt, kvt, o, lse)
        ctx.geom, ctx.same = (heads, hd, q_off, k_off, v_off), qt is kvt
        return o

    @staticmethod
    def backward(ctx, go):
        qt, kvt, o, lse = ctx.saved_tensors
        heads, hd, q_off, k_off, v_off = ctx.geom
        vw = _StackedSDPA._view
        gq = torch.empty_like(qt)  # every column block is written: q/k/v (self) or q and k/v (cross)
        gkv = gq if ctx.same else torch.empty_like(kvt)
        torch.ops.b2.sdpa_bwd_into(go, vw(qt, q_off, heads, hd), vw(kvt, k_off, heads, hd), vw(kvt, v_off, heads, hd),
                                   o, lse, 0.0, vw(gq, q_off, heads, hd), vw(gkv, k_off, heads, hd),
                                   vw(gkv, v_off, heads, hd))
        return gq, (None if ctx.same else gkv), None, None, None, None, None


class DiTBlock(nn.Module):
    def __init__(self, hidden=2048, heads=16, text_dim=1024, mlp=8192, rank=16, alpha=16.0, seed=0, device="cuda"):
        super().__init__()
        g = torch.Generator(device=device).manual_seed(seed)
        self.h, self.heads, self.d = hidden, heads, hidden // heads
        mk = lambda i, o: LoRAInt8Linear(i, o, rank, alpha, generator=g, device=device)  # noqa: E731
        self.q, self.k, self.v, self.o = mk(hidden, hidden), mk(hidden, hidden), mk(hidden, hidden), mk(hidden, hidden)
        self.cq, self.ck, self.cv, self.co = mk(hidden, hidden), mk(text_dim, hidden), mk(text_dim, hidden), mk(hidden, hidden)
        self.fc1 = Int8Linear(hidden, mlp, generator=g, device=device)
        self.fc2 = Int8Linear(mlp, hidden, generator=g, device=device)
        # adaLN modulation: (shift, scale, gate) for self-attn, cross-attn and MLP from the conditioning vector
        self.ada = Int8Linear(hidden, 9 * hidden, generator=g, device=device)
        # projections that read the same input keep their frozen int8 bases in one stacked weight
        # (each module's base buffers are views of it): one GEMM forward and one dX GEMM backward
        self._stack_bases("qkv", (self.q, self.k, self.v))
        self._stack_bases("ckv", (self.ck, self.cv))
        # and their LoRA matrices in stacked storage (the modules' Parameters are views of it)
        self._lora_groups = {"qkv": LoRAGroup((self.q, self.k, self.v)), "ckv": LoRAGroup((self.ck, self.cv))}

    def _stack_bases(self, name, mods):
        for part in ("q", "scale", "bias"):
            full = torch.cat([getattr(m.base, part) for m in mods], 0)
            self.register_buffer(f"{name}_{part}", full)
            o = 0
            for m in mods:
                n = getattr(m.base, part).shape[0]
                setattr(m.base, part, full[o:o + n])
                o += n

    def _stacked(self, name, x, mods, whole=False):
        grp = self._lora_groups[name]
        assert all(a is b for a, b in zip(grp.mods, mods))
        return stacked_lora_forward(x, getattr(self, f"{name}_q"), getattr(self, f"{name}_scale"),
                                    getattr(self, f"{name}_bias"), grp, whole=whole)

    def _attn(self, xq, xkv_k, xkv_v, qp, kp, vp, op, kv=None):
        B, S, _ = xq.shape
        Skv = xkv_k.shape[1]
        # projections that read the same input run as one stacked group (stacked_lora_forward)
        hd = self.heads * self.d
        if kv is not None or (xkv_k is xkv_v and kp is self.ck):  # q, and the stacked text-side k/v output
            q = qp(xq)
            if kv is not None:  # projected ahead on the side stream
                torch.cuda.current_stream(xq.device).wait_stream(self._side)
            else:
                kv = self._stacked("ckv", xkv_k, (kp, vp), whole=True)
            o = _StackedSDPA.apply(q, kv, self.heads, hd, 0, 0, hd)
            return op(o.transpose(1, 2).reshape(B, S, self.h))
        if xq is xkv_k and xkv_k is xkv_v and qp is self.q:  # the stacked q/k/v output
            qkv = self._stacked("qkv", xq, (qp, kp, vp), whole=True)
            o = _StackedSDPA.apply(qkv, qkv, self.heads, hd, 0, hd, 2 * hd)
            return op(o.transpose(1, 2).reshape(B, S, self.h))
        q, k, v = qp(xq), kp(xkv_k), vp(xkv_v)
        q = q.view(B, S, self.heads, self.d).transpose(1, 2)
        k = k.view(B, Skv, self.heads, self.d).transpose(1, 2)
        v = v.view(B, Skv, self.heads, self.d).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v)
        return op(o.transpose(1, 2).reshape(B, S, self.h))

    # the text-side k/v projection depends only on the text embeddings: it runs on a side stream, beside the
    # modulation, the first LayerNorm and the self-attention branch, and autograd runs its backward (the
    # LoRA gradients of ck/cv) on the same side stream, beside the rest of the block's backward
    overlap_text_kv = True
    _side = None

    def _text_kv_ahead(self, text):
        if not (self.overlap_text_kv and text.is_cuda):
            return None
        main = torch.cuda.current_stream(text.device)
        if self._side is None or self._side.device != text.device:
            self._side = torch.cuda.Stream(text.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            kv = self._stacked("ckv", text, (self.ck, self.cv), whole=True)
        kv.record_stream(main)  # consumed on the main stream: keep the allocator from reusing it early
        return kv

    def forward(self, x, text, cond):
        kv = self._text_kv_ahead(text)
        ada = self.ada(F.silu(cond))
        sh1, sc1, g1, sh2, sc2, g2, sh3, sc3, g3 = ada.unsqueeze(1).chunk(9, dim=-1)
        # one sample: the modulation is the LayerNorm's own affine (one kernel), its three weights 1 + scale
        # computed by one kernel from the scale chunks (1, 4 and 7 of the nine)
        ln_w = (1 + ada.view(9, self.h)[1::3]) if x.shape[0] == 1 else None

        def modln(t, sh, sc, i):
            if ln_w is not None:
                return F.layer_norm(t, (self.h,), weight=ln_w[i], bias=sh.view(self.h), eps=1e-6)
            return F.layer_norm(t, (self.h,), eps=1e-6) * (1 + sc) + sh

        # residual updates x + g * branch as one addcmul kernel
        h = modln(x, sh1, sc1, 0)
        x = torch.addcmul(x, g1, self._attn(h, h, h, self.q, self.k, self.v, self.o))
        h = modln(x, sh2, sc2, 1)
        x = torch.addcmul(x, g2, self._attn(h, text, text, self.cq, self.ck, self.cv, self.co, kv=kv))
        h = modln(x, sh3, sc3, 2)
        # MLP fc2(gelu(fc1(h))) with the GELU (and its backward) in the int8 GEMM epilogues
        mlp = tv.int8_mlp(h, self.fc1.q, self.fc1.scale, self.fc1.bias, self.fc2.q, self.fc2.scale, self.fc2.bias)
        x = torch.addcmul(x, g3, mlp)
        return x


class DiTStack(nn.Module):
    def __init__(self, blocks=1, seed=0, device="cuda", checkpoint=False, **kw):
        super().__init__()
        self.blocks = nn.ModuleList([DiTBlock(seed=seed + i, device=device, **kw) for i in range(blocks)])
        self.checkpoint = checkpoint
        self.offloader = None

    def forward(self, x, text, cond):
        for b in self.blocks:
            if self.checkpoint:
                x = torch.utils.checkpoint.checkpoint(b, x, text, cond, use_reentrant=False)
            else:
                x = b(x, text, cond)
        return x

    def enable_block_swap(self, blocks_to_swap, ring_size=2):
        """Keep the frozen int8 weights of the last `blocks_to_swap` blocks in pinned host memory and stream
        them through `ring_size` device slots (torch_vulkan_b200.offload); turns on activation checkpointing,
        which the swap needs for the backward."""
        from .offload import BlockSwapConfig, create_offloader

        dev = next(self.parameters()).device
        cfg = BlockSwapConfig(device=dev, supports_backward=True, h2d_only=True, ring_size=ring_size)
        self.checkpoint = True
        self.offloader = create_offloader("block", self.blocks, len(self.blocks), blocks_to_swap, cfg)
        self.offloader.prepare_block_devices_before_forward(self.blocks)
        return self.offloader

    def lora_parameters(self):
        return [p for n, p in self.named_parameters() if "lora_" in n]


def synthetic_batch(tokens=1024, text_tokens=512, hidden=2048, text_dim=1024, batch=1, seed=0, device="cuda"):
    """Latent tokens (64x64 latent, patch 2 -> 1024 tokens at 512 px; 4096 at 1024 px), text embeddings,
    conditioning vector and a regression target, all seeded N(0, 1) in bf16."""
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).to(device)  # noqa: E731
    return mk(batch, tokens, hidden), mk(batch, text_tokens, text_dim), mk(batch, hidden), mk(batch, tokens, hidden)


def block_flops(tokens=1024, text_tokens=512, hidden=2048, text_dim=1024, mlp=8192, heads=16):
    """Forward and backward FLOPs of one block (dX only for frozen weights, no dX into the text context,
    attention backward = 2.5x forward), excluding LoRA and elementwise work."""
    lin_f = 2 * tokens * hidden * hidden * 6 + 2 * text_tokens * text_dim * hidden * 2 + 2 * tokens * hidden * mlp * 2
    attn_f = 4 * tokens * tokens * hidden + 4 * tokens * text_tokens * hidden
    lin_b = 2 * tokens * hidden * hidden * 6 + 2 * tokens * hidden * mlp * 2  # dX of the frozen linears (no text dX)
    return lin_f + attn_f, lin_b + 2.5 * attn_f


def make_optimizer(params, lr=1e-4, fused=False):
    """AdamW(foreach=False): the per-tensor addcmul_/addcdiv_/lerp_ path the reference's trainer uses;
    fused=True: the same arithmetic as one multi-tensor launch per 48 parameters (FusedAdamW)."""
    if fused:
        from torch_vulkan_b200.optim import FusedAdamW

        return FusedAdamW(params, lr=lr, betas=(0.9, 0.999), weight_decay=0.01)
    return torch.optim.AdamW(params, lr=lr, betas=(0.9, 0.999), weight_decay=0.01, foreach=False)


class LoRATrainer:
    """One LoRA training step of a DiTStack: forward, MSE loss against the target (F.mse_loss(out.float(),
    target.float()) on the fused loss kernels, tv.mse_loss; target in the output's dtype), backward, data-parallel
    gradient averaging (bucketed per block, overlapped with the backward when torch.distributed is
    initialised), AdamW on the LoRA parameters (per-tensor foreach=False ops, or fused_optimizer=True for
    the multi-tensor kernel)."""

    def __init__(self, model: DiTStack, lr=1e-4, fused_optimizer=False):
        from torch_vulkan_b200.dp import BucketedGradAllReduce

        self.model = model
        buckets = [[p for n, p in b.named_parameters() if "lora_" in n] for b in model.blocks]
        self.params = [p for bk in buckets for p in bk]
        self.reducer = BucketedGradAllReduce(buckets)
        self.opt = make_optimizer(self.params, lr=lr, fused=fused_optimizer)

    def step(self, x, text, cond, target):
        loss = tv.mse_loss(self.model(x, text, cond), target)
        loss.backward()
        self.reducer.wait()
        self.opt.step()
        self.reducer.zero_grad()
        return loss.detach()

    def graphed(self, x, text, cond, target, warmup=3):
        """Step with forward + backward captured once as a CUDA graph (the inputs are the graph's static
        buffers: copy new data into them before each call) and the optimizer launched after each replay.
        With several ranks the bucket all-reduces that the gradient hooks launch during the captured
        backward are captured too (NCCL collectives replay inside the graph, still overlapping the
        backward of earlier blocks); every rank captures the same collectives in the same order. Warm-up
        steps run first so that NCCL's communicators exist before the capture. Returns a callable
        performing one step and returning the loss tensor."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self.step(x, text, cond, target)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        self.reducer.zero_grad()  # re-arm the hooks so the captured backward launches every bucket
        # with NCCL, the process group's watchdog thread queries events while this thread captures; the
        # thread-local capture mode keeps those queries from invalidating the capture
        mode = "thread_local" if self.reducer.world > 1 else "global"
        with torch.cuda.graph(graph, capture_error_mode=mode):
            for flat in self.reducer.flats:  # gradients accumulate into the bucket buffers
                flat.zero_()
            loss = tv.mse_loss(self.model(x, text, cond), target)
            loss.backward()
            self.reducer.wait()  # the captured collectives join the capture stream before it ends
        self._graph = graph  # kept alive with its memory pool (release it before destroying the group)

        def run():
            graph.replay()
            self.opt.step()
            return loss.detach()

        return run
