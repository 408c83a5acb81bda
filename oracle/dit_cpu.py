"""CPU restatement of the synthetic DiT LoRA training step — TEST INFRASTRUCTURE / CPU BASELINE ONLY.

The reference's path for this workload is its CPU fallback: every operator the block uses runs as stock
PyTorch CPU ATen (csrc/shim.cpp:70-131), and its LoRA module layout is tests/anima_on_vk.py:43-48.
This module states the same block (BASELINE configs[3]/[4]: adaLN-modulated LayerNorm, self-attention,
cross-attention to the text tokens, GELU(tanh) MLP, LoRA rank 16 / alpha 16 on the q/k/v/o linears of
both attentions over frozen int8 weights with a per-row scale, AdamW(foreach=False)) with plain CPU
PyTorch ops in bf16, so that bench.py can time the reference's CPU path on the host cores. Only
bench.py's cpu_baseline leg and tests/ use it.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

_LORA = ("q", "k", "v", "o", "cq", "ck", "cv", "co")


def _int8_weight(n_out, n_in, g, std=0.02):
    """Random init std 0.02, quantised per output row to int8, returned dequantised (bf16) as the
    reference's CPU path computes it (torch_vulkan/__init__.py:203-205, per-row variant)."""
    w = torch.randn(n_out, n_in, generator=g) * std
    s = w.abs().amax(1).clamp_min(1e-8) / 127.0
    q = torch.round(w / s[:, None]).clamp_(-127, 127)
    return (q * s[:, None]).to(torch.bfloat16)


def make_block(hidden=2048, heads=16, text_dim=1024, mlp=8192, rank=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    p = {"hidden": hidden, "heads": heads, "scale": 16.0 / rank}
    ins = {"q": hidden, "k": hidden, "v": hidden, "o": hidden, "cq": hidden, "ck": text_dim, "cv": text_dim, "co": hidden}
    for n in _LORA:
        p[n + ".w"] = _int8_weight(hidden, ins[n], g)
        p[n + ".b"] = torch.zeros(hidden, dtype=torch.bfloat16)
        p[n + ".A"] = (torch.randn(rank, ins[n], generator=g) / math.sqrt(ins[n])).to(torch.bfloat16).requires_grad_(True)
        p[n + ".B"] = (torch.randn(hidden, rank, generator=g) * 0.02).to(torch.bfloat16).requires_grad_(True)
    p["fc1.w"], p["fc1.b"] = _int8_weight(mlp, hidden, g), torch.zeros(mlp, dtype=torch.bfloat16)
    p["fc2.w"], p["fc2.b"] = _int8_weight(hidden, mlp, g), torch.zeros(hidden, dtype=torch.bfloat16)
    p["ada.w"], p["ada.b"] = _int8_weight(9 * hidden, hidden, g), torch.zeros(9 * hidden, dtype=torch.bfloat16)
    return p


def lora_params(p):
    return [p[n + s] for n in _LORA for s in (".A", ".B")]


def _lora(p, n, x):
    return F.linear(x, p[n + ".w"], p[n + ".b"]) + F.linear(F.linear(x, p[n + ".A"]), p[n + ".B"]) * p["scale"]


def block_forward(p, x, text, cond):
    h_, heads = p["hidden"], p["heads"]
    d = h_ // heads
    mod = F.linear(F.silu(cond), p["ada.w"], p["ada.b"]).unsqueeze(1).chunk(9, dim=-1)
    sh1, sc1, g1, sh2, sc2, g2, sh3, sc3, g3 = mod

    def modln(t, sh, sc):
        return F.layer_norm(t, (h_,), eps=1e-6) * (1 + sc) + sh

    def attn(tq, tkv, pre):
        B, S, _ = tq.shape
        Skv = tkv.shape[1]
        q = _lora(p, pre + "q", tq).view(B, S, heads, d).transpose(1, 2)
        k = _lora(p, pre + "k", tkv).view(B, Skv, heads, d).transpose(1, 2)
        v = _lora(p, pre + "v", tkv).view(B, Skv, heads, d).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v)
        return _lora(p, pre + "o", o.transpose(1, 2).reshape(B, S, h_))

    h = modln(x, sh1, sc1)
    x = x + g1 * attn(h, h, "")
    h = modln(x, sh2, sc2)
    x = x + g2 * attn(h, text, "c")
    h = modln(x, sh3, sc3)
    m = F.linear(F.gelu(F.linear(h, p["fc1.w"], p["fc1.b"]), approximate="tanh"), p["fc2.w"], p["fc2.b"])
    return x + g3 * m


def synthetic_batch(tokens=1024, text_tokens=512, hidden=2048, text_dim=1024, seed=0):
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
    return mk(1, tokens, hidden), mk(1, text_tokens, text_dim), mk(1, hidden), mk(1, tokens, hidden)


def make_step(p, lr=1e-4):
    """One LoRA training step of the block on the CPU: forward, MSE, backward, AdamW(foreach=False)."""
    opt = torch.optim.AdamW(lora_params(p), lr=lr, betas=(0.9, 0.999), weight_decay=0.01, foreach=False)

    def step(x, text, cond, target):
        opt.zero_grad(set_to_none=True)
        loss = F.mse_loss(block_forward(p, x, text, cond).float(), target.float())
        loss.backward()
        opt.step()
        return loss.item()

    return step
