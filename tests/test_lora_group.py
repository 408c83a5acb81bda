"""Host logic of the stacked LoRA storage of the DiT block (torch_vulkan_b200.dit.LoRAGroup), on CPU tensors:
the modules' Parameters become contiguous views of the stacked matrices, the block-diagonal up-projection
the int8 GEMM reads is refreshed from them (times alpha / r), and dB's diagonal blocks come out in the
stacked layout, one block per module."""

import torch
import torch.nn as nn

from torch_vulkan_b200.dit import LoRAGroup


class _Mod(nn.Module):
    def __init__(self, n, k, r, scale, seed):
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.lora_down = nn.Parameter(torch.randn(r, k, generator=g))
        self.lora_up = nn.Parameter(torch.randn(n, r, generator=g))
        self.scale = scale


def test_parameters_become_views_and_refresh_builds_block_diagonal():
    mods = [_Mod(6, 5, 2, 0.5, s) for s in range(3)]
    ups = [m.lora_up.detach().clone() for m in mods]
    downs = [m.lora_down.detach().clone() for m in mods]
    grp = LoRAGroup(mods)
    for i, m in enumerate(mods):
        assert torch.equal(m.lora_up, ups[i]) and torch.equal(m.lora_down, downs[i])
        assert m.lora_up.is_contiguous() and m.lora_up.data_ptr() == grp.b[6 * i:].data_ptr()
        assert m.lora_down.data_ptr() == grp.a[2 * i:].data_ptr()
    grp.refresh()
    assert torch.equal(grp.b_bd, torch.block_diag(*ups) * 0.5)
    with torch.no_grad():  # an optimizer's in-place update reaches the next refresh
        mods[1].lora_up.add_(1.0)
    grp.refresh()
    assert torch.equal(grp.b_bd, torch.block_diag(ups[0], ups[1] + 1.0, ups[2]) * 0.5)
    assert torch.equal(grp.a, torch.cat(downs, 0))


def test_diag_blocks_picks_each_modules_block():
    mods = [_Mod(4, 3, 2, 1.0, s) for s in range(3)]
    grp = LoRAGroup(mods)
    full = torch.arange(12 * 6, dtype=torch.float32).view(12, 6)
    out = grp.diag_blocks(full)
    ref = torch.cat([full[4 * i:4 * (i + 1), 2 * i:2 * (i + 1)] for i in range(3)], 0)
    assert out.shape == (12, 2) and torch.equal(out, ref)
