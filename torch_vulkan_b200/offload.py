"""H2D-only block swap: the frozen weights of the last `blocks_to_swap` blocks of a model live in pinned host
memory, and a ring of device slots holds the blocks that are about to run.

This is the device-side surface sd-scripts' block swap needs (the reference exercises it through
sd-scripts' `custom_offloading_utils` in tests/test_block_swap_vk.py:60-64 with
`BlockSwapConfig(device, supports_backward=True, h2d_only=True, ring_size=r)`), written for CUDA:

* each swapped block's frozen tensors (parameters with requires_grad=False, and buffers) are packed once
  into one pinned host buffer, so bringing a block in is a single `cudaMemcpyAsync` on a dedicated copy
  stream (the host link runs at full rate only with large pinned copies);
* the copy into a slot waits on an event recorded on the compute stream when the slot is taken (behind
  every kernel enqueued so far, the previous owner's included), and the compute stream waits on the
  copy's event before the block runs, so copies overlap the neighbouring blocks' kernels without a device
  synchronisation;
* tensors are re-pointed in place (`Tensor.set_`) at their slot, so modules, views that share storage (the
  stacked q/k/v bases of a DiT block) and tensors captured by other modules keep their identity;
* trainable parameters never move.

Nothing is ever copied device-to-host after set-up (h2d only): frozen weights do not change. A block's
weights are read in the forward and again in its backward, so swapped blocks must run under activation
checkpointing (`torch.utils.checkpoint.checkpoint(block, ..., use_reentrant=False)`): the recomputation in
the backward brings the block back through the same forward pre-hook, and autograd never keeps a saved
reference to a slot that has since been reused.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn

_ALIGN = 256  # bytes; every storage starts on a 256-byte boundary inside a slot (TMA wants 16)


@dataclass
class BlockSwapConfig:
    device: torch.device | str = "cuda"
    supports_backward: bool = True
    h2d_only: bool = True
    ring_size: int = 2


def _frozen_storages(block: nn.Module):
    """Distinct storages of the block's frozen tensors, and for each tensor (storage index, tensor)."""
    tensors = [p for p in block.parameters() if not p.requires_grad] + list(block.buffers())
    storages, index, refs = [], {}, []
    for t in tensors:
        key = t.untyped_storage().data_ptr()
        if key not in index:
            index[key] = len(storages)
            storages.append(t.untyped_storage())
        refs.append((index[key], t))
    return storages, refs


class _Swapped:
    """One swapped block: its pinned host image and the layout of its storages inside a slot."""

    def __init__(self, block: nn.Module, device: torch.device):
        storages, refs = _frozen_storages(block)
        offsets, total = [], 0
        for st in storages:
            offsets.append(total)
            total += (st.nbytes() + _ALIGN - 1) // _ALIGN * _ALIGN
        self.nbytes = total
        self.host = torch.empty(max(total, 1), dtype=torch.uint8, pin_memory=device.type == "cuda")
        for st, off in zip(storages, offsets):
            n = st.nbytes()
            src = torch.empty(0, dtype=torch.uint8, device=st.device).set_(st, 0, (n,), (1,))
            self.host[off:off + n].copy_(src)
        # (storage offset in the slot, tensor, element offset of the tensor inside its storage, size, stride)
        self.refs = [(offsets[si], t, t.storage_offset(), tuple(t.size()), tuple(t.stride())) for si, t in refs]
        self.device = device

    def point_at(self, slot: torch.Tensor) -> None:
        storage = slot.untyped_storage()
        base = slot.storage_offset()  # bytes (uint8)
        for off, t, elem_off, size, stride in self.refs:
            item = t.element_size()
            byte = base + off + elem_off * item
            assert byte % item == 0
            with torch.no_grad():
                if t.device != slot.device:  # a block built on the host: give the tensor a device first
                    t.data = torch.empty(0, dtype=t.dtype, device=slot.device)
                t.set_(storage, byte // item, size, stride)


class BlockSwapper:
    """Keeps the frozen weights of blocks[num_blocks - blocks_to_swap:] in pinned host memory and streams
    them into `ring_size` device slots in the order the forward (and the checkpointed backward) asks for
    them. Call `prepare_block_devices_before_forward` once, `wait_for_block(i)` before block i runs and
    `submit_move_blocks_forward(blocks, i)` after it (the method names of sd-scripts' offloader). A forward
    pre-hook on every swapped block makes the same calls by itself (they are idempotent), so a model that
    just calls its blocks works too, and it serves the recomputation inside the backward, which walks the
    blocks in reverse and prefetches block i - 1 while block i runs. A block whose backward reads its frozen
    weights after the next block's recomputation has started (a side branch, e.g. a gradient into a
    context input computed late) is outside this contract."""

    def __init__(self, blocks, num_blocks: int, blocks_to_swap: int, config: BlockSwapConfig):
        if not config.h2d_only:
            raise ValueError("only the h2d-only form is implemented (frozen weights are never written back)")
        if not 0 <= blocks_to_swap <= num_blocks:
            raise ValueError(f"blocks_to_swap must be in [0, {num_blocks}]")
        if config.ring_size < 1:
            raise ValueError("ring_size must be >= 1")
        self.blocks = list(blocks)
        self.num_blocks = num_blocks
        self.first_swapped = num_blocks - blocks_to_swap
        self.cfg = config
        self.device = torch.device(config.device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.copy_stream = None
        self.swapped: dict[int, _Swapped] = {}
        self.slots: list[torch.Tensor] = []
        self.owner: list[int | None] = []
        self.ready: list[torch.cuda.Event | None] = []
        self.last_use: list[int] = []
        self.where: dict[int, int] = {}  # block -> slot
        self.current: int | None = None
        self.clock = 0
        self.h2d_bytes = 0
        self.h2d_copies = 0
        self._hooks = []

    # ---- set-up ------------------------------------------------------------------------------------

    def prepare_block_devices_before_forward(self, blocks=None) -> None:
        blocks = self.blocks if blocks is None else list(blocks)
        self.copy_stream = torch.cuda.Stream(device=self.device)
        for i, b in enumerate(blocks):
            if i < self.first_swapped:
                b.to(self.device)
                continue
            # trainable parameters stay resident; the frozen ones are packed into pinned memory
            for p in b.parameters():
                if p.requires_grad:
                    p.data = p.data.to(self.device)
            if i not in self.swapped:
                self.swapped[i] = _Swapped(b, self.device)
        if self.swapped and not self.slots:
            nbytes = max(s.nbytes for s in self.swapped.values())
            for _ in range(min(self.cfg.ring_size, len(self.swapped))):
                self.slots.append(torch.empty(nbytes, dtype=torch.uint8, device=self.device))
                self.owner.append(None)
                self.ready.append(None)
                self.last_use.append(-1)
            # every swapped block points at slot 0 until it is loaded; its device copies are released here
            for s in self.swapped.values():
                s.point_at(self.slots[0])
            torch.cuda.synchronize(self.device)
        if not self._hooks:
            for i in self.swapped:
                self._hooks.append(blocks[i].register_forward_pre_hook(self._pre_hook(i)))

    def _pre_hook(self, i):
        def hook(module, args):
            self.wait_for_block(i)
            # the next block to run: i - 1 in the recomputation inside the backward, i + 1 otherwise
            self._prefetch(i - 1 if torch._C._current_graph_task_id() != -1 else i + 1)
        return hook

    def close(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []

    # ---- the sd-scripts call pattern ----------------------------------------------------------------

    def wait_for_block(self, i: int) -> None:
        """Block i's weights are resident and the current stream waits for their copy (idempotent)."""
        if i not in self.swapped:
            self.current = None
            return
        if self.current == i:
            return
        self.current = None
        s = self.where.get(i)
        if s is None:
            s = self._load(i)
        torch.cuda.current_stream(self.device).wait_event(self.ready[s])
        self.current = i
        self.clock += 1
        self.last_use[s] = self.clock

    def submit_move_blocks_forward(self, blocks, i: int) -> None:
        """Called after block i's forward: start bringing in the next swapped block."""
        self._prefetch(i + 1)

    # ---- internals ----------------------------------------------------------------------------------

    def _prefetch(self, j: int) -> None:
        if j in self.swapped and j not in self.where and (len(self.slots) > 1 or self.current is None):
            self._load(j)

    def _load(self, j: int) -> int:
        """Copy block j into the least recently used slot that the running block does not hold. The copy
        waits for everything the compute stream has enqueued so far (the previous owner's kernels)."""
        keep = self.where.get(self.current) if self.current is not None else None
        cands = [s for s in range(len(self.slots)) if s != keep]
        free = [s for s in cands if self.owner[s] is None]
        s = free[0] if free else min(cands, key=lambda k: self.last_use[k])
        old = self.owner[s]
        if old is not None:
            del self.where[old]
        sw = self.swapped[j]
        released = torch.cuda.Event()
        released.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(released)
            self.slots[s][:sw.nbytes].copy_(sw.host[:sw.nbytes], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        self.ready[s] = ev
        self.owner[s] = j
        self.where[j] = s
        self.clock += 1
        self.last_use[s] = self.clock
        sw.point_at(self.slots[s])
        self.h2d_bytes += sw.nbytes
        self.h2d_copies += 1
        return s

    def resident_bytes(self) -> int:
        """Device bytes held for swapped blocks (the slots)."""
        return sum(t.numel() for t in self.slots)


def create_offloader(kind: str, blocks, num_blocks: int, blocks_to_swap: int, config: BlockSwapConfig):
    """sd-scripts' factory name; only the per-block ("block") form exists."""
    if kind != "block":
        raise ValueError(f"unknown offloader kind {kind!r}")
    return BlockSwapper(blocks, num_blocks, blocks_to_swap, config)
