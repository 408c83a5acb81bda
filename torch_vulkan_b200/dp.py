"""Data parallelism for the LoRA step: bucketed gradient averaging overlapped with the backward pass.

New relative to the reference (torch-vulkan is single-device, csrc/shim.cpp:176-184)
shards the global batch one sample per GPU and averages the LoRA gradients with NCCL all-reduce over
NVLink every step, then every rank applies the same AdamW update, which keeps the replicas identical.

Each bucket (normally one transformer block's LoRA parameters) owns one flat gradient buffer; the
parameters' `.grad` are views into it, so autograd accumulates straight into the buffer and no packing
copy is needed. When the last gradient of a bucket has been accumulated (post-accumulate-grad hook, fired
on the autograd thread in backward order) the bucket's all-reduce is launched asynchronously, so the
collective for block n overlaps the backward of blocks n-1, n-2, ...; `wait()` blocks the host only at
the end of the backward. Every rank issues the same collectives in the same order (the hooks fire in the
deterministic autograd order of identical graphs).
"""

from __future__ import annotations

from typing import Iterable, Sequence

import torch
import torch.distributed as dist


class BucketedGradAllReduce:
    """With one process there is nothing to average: no flat buffers are bound, so autograd hands each
    parameter the gradient tensor it computed (no accumulation kernel per parameter) and `zero_grad`
    resets `.grad` to None."""

    def __init__(self, buckets: Sequence[Sequence[torch.nn.Parameter]], group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.buckets = [list(b) for b in buckets if len(b) > 0]
        self.flats = []
        self._owner = {}
        if self.world == 1:
            self._pending = [0] * len(self.buckets)
            self._streams = [set() for _ in self.buckets]
            self._handles = []
            return
        for bi, params in enumerate(self.buckets):
            dtype, dev = params[0].dtype, params[0].device
            if any(p.dtype != dtype or p.device != dev for p in params):
                raise ValueError("a bucket must hold parameters of one dtype and device")
            flat = torch.zeros(sum(p.numel() for p in params), dtype=dtype, device=dev)
            self.flats.append(flat)
            for p in params:
                self._owner[p] = bi
                p.register_post_accumulate_grad_hook(self._on_grad)
        self._pending = [len(b) for b in self.buckets]
        self._streams = [set() for _ in self.buckets]
        self._handles = []
        self._bind()

    def _bind(self):
        for params, flat in zip(self.buckets, self.flats):
            off = 0
            for p in params:
                n = p.numel()
                p.grad = flat[off:off + n].view_as(p)
                off += n

    def _on_grad(self, p):
        bi = self._owner[p]
        self._pending[bi] -= 1
        if p.is_cuda:  # the stream this gradient was accumulated on (autograd runs each op on its forward's)
            self._streams[bi].add(torch.cuda.current_stream(p.device))
        if self._pending[bi] == 0 and self.world > 1:
            flat = self.flats[bi]
            # the collective is ordered after the current stream only: make that stream wait for every other
            # stream that accumulated into this bucket (a block whose branches ran on two streams)
            if self._streams[bi]:
                cur = torch.cuda.current_stream(flat.device)
                for s in self._streams[bi]:
                    if s != cur:
                        cur.wait_stream(s)
            backend = dist.get_backend(self.group)
            if backend == "nccl":
                self._handles.append(dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=self.group, async_op=True))
            else:  # gloo has no AVG: sum, then scale after the wait
                self._handles.append((dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True), flat))

    def wait(self):
        """Completes every bucket's all-reduce (called once the backward has finished)."""
        if any(n != 0 for n in self._pending):
            raise RuntimeError(f"backward did not produce every bucketed gradient (pending {self._pending})")
        for h in self._handles:
            if isinstance(h, tuple):
                h[0].wait()
                h[1].div_(self.world)
            else:
                h.wait()
        self._handles = []

    def zero_grad(self):
        """Clears the flat buffers (one memset per bucket) and re-arms the hooks for the next step."""
        if self.world == 1:
            for params in self.buckets:
                for p in params:
                    p.grad = None
            return
        for flat in self.flats:
            flat.zero_()
        self._pending = [len(b) for b in self.buckets]
        self._streams = [set() for _ in self.buckets]
        self._bind()


def flat_grads(params: Iterable[torch.nn.Parameter]) -> torch.Tensor:
    return torch.cat([p.grad.reshape(-1).float() for p in params])
