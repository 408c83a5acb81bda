"""The DiT LoRA step data-parallel over NCCL on 2 GPUs (one process per GPU): the bucketed all-reduce
leaves every rank with the average of both ranks' LoRA gradients — equal to one process running both
samples — and the replicas stay identical after the optimizer step. Skipped with fewer than 2 GPUs."""

import datetime
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KW = dict(hidden=256, heads=2, text_dim=128, mlp=512)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _batch(rank, dev):
    from torch_vulkan_b200.dit import synthetic_batch

    return synthetic_batch(tokens=128, text_tokens=64, hidden=256, text_dim=128, seed=500 + rank, device=dev)


def _worker(rank, world, port, q):
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        import torch.nn.functional as F

        from torch_vulkan_b200.dit import DiTStack, LoRATrainer

        model = DiTStack(blocks=2, seed=0, device=dev, **KW)
        tr = LoRATrainer(model, lr=1e-3, fused_optimizer=True)
        x, text, cond, target = _batch(rank, dev)
        out = model(x, text, cond)
        F.mse_loss(out.float(), target.float()).backward()
        tr.reducer.wait()
        grads = torch.cat([p.grad.float().flatten() for p in tr.params]).cpu()
        tr.opt.step()
        params = torch.cat([p.detach().float().flatten() for p in tr.params]).cpu()
        ref = None
        if rank == 0:  # one process, both samples, gradients averaged by hand
            m2 = DiTStack(blocks=2, seed=0, device=dev, **KW)
            ps = m2.lora_parameters()
            for r in range(world):
                xb, tb, cb, yb = _batch(r, dev)
                F.mse_loss(m2(xb, tb, cb).float(), yb.float()).backward()
            ref = torch.cat([p.grad.float().flatten() / world for p in ps]).cpu()
        torch.cuda.synchronize()
        q.put((rank, grads.numpy(), params.numpy(), None if ref is None else ref.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_bucketed_average_matches_single_process():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, g, prm, ref = q.get(timeout=300)
        res[r] = (torch.from_numpy(g), torch.from_numpy(prm), None if ref is None else torch.from_numpy(ref))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    g0, p0, ref = res[0]
    g1, p1, _ = res[1]
    assert torch.equal(g0, g1)  # every rank holds the same averaged gradient
    assert torch.equal(p0, p1)  # replicas identical after the step
    rel = ((g0.double() - ref.double()).norm() / ref.double().norm()).item()
    assert rel < 2e-2, rel  # bf16 gradients, two summation orders
