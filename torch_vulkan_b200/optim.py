"""Multi-tensor AdamW on the library's kernel (`b2_adamw_step`).

torch.optim.AdamW(foreach=False) — what torch-vulkan's trainer runs (its addcmul_/addcdiv_/lerp_ path,
csrc/ops_ew.cpp:432-451) — issues about six kernels per parameter tensor per step. `FusedAdamW` applies
the same arithmetic, rounded to the parameter dtype after each of those in-place ops, to up to 48
tensors per launch. Parameters, gradients and state must be contiguous CUDA tensors of one dtype
(float32 or bfloat16).
"""

from __future__ import annotations

import torch


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-2):
        if lr < 0 or eps < 0 or weight_decay < 0 or not (0 <= betas[0] < 1 and 0 <= betas[1] < 1):
            raise ValueError("FusedAdamW: invalid hyper-parameter")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            by_step = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("FusedAdamW does not support sparse gradients")
                st = self.state[p]
                if not st:
                    st["step"] = 0
                    st["exp_avg"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                    st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.contiguous_format)
                st["step"] += 1
                g = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
                by_step.setdefault((st["step"], p.dtype), []).append((p, g, st["exp_avg"], st["exp_avg_sq"]))
            b1, b2 = group["betas"]
            for (step, _), items in by_step.items():
                ps, gs, ms, vs = (list(t) for t in zip(*items))
                torch.ops.b2.adamw_step_(ps, gs, ms, vs, group["lr"], b1, b2, group["eps"], group["weight_decay"], step)
        return loss
