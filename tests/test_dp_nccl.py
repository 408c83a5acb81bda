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


def _worker_graphed(rank, world, port, q):
    """Two identical trainers per rank: one steps eagerly, one replays its forward + backward (with the
    captured bucket all-reduces) as a CUDA graph; after three steps both hold the same LoRA parameters."""
    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from torch_vulkan_b200.dit import DiTStack, LoRATrainer

        batch = _batch(rank, dev)
        eager = LoRATrainer(DiTStack(blocks=2, seed=0, device=dev, **KW), lr=1e-3, fused_optimizer=True)
        le = [float(eager.step(*batch).item()) for _ in range(3)]
        pe = torch.cat([p.detach().float().flatten() for p in eager.params]).cpu()
        gtr = LoRATrainer(DiTStack(blocks=2, seed=0, device=dev, **KW), lr=1e-3, fused_optimizer=True)
        step = gtr.graphed(*batch, warmup=1)  # one eager warm-up step, then captured steps
        lg = [float(step().item()) for _ in range(2)]
        pg = torch.cat([p.detach().float().flatten() for p in gtr.params]).cpu()
        torch.cuda.synchronize()
        del step, gtr._graph  # graphs holding NCCL work go before the process group
        q.put((rank, le, lg, pe.numpy(), pg.numpy()))
    finally:
        dist.destroy_process_group()


def _spawn(target, world=2):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = [q.get(timeout=240) for _ in range(world)]
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:  # a rank that failed must not outlive the test (its peer would wait in NCCL)
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=30)
    return {o[0]: o[1:] for o in out}


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_nccl_graphed_step_matches_eager_step():
    res = _spawn(_worker_graphed)
    for r in range(2):
        le, lg, pe, pg = res[r]
        # graphed steps 2 and 3 against eager steps 2 and 3 (warm-up = eager step 1)
        assert max(abs(a - b) / abs(b) for a, b in zip(lg, le[1:])) < 1e-3, (le, lg)
        pe, pg = torch.from_numpy(pe).double(), torch.from_numpy(pg).double()
        assert ((pg - pe).norm() / pe.norm()).item() < 1e-3
    # replicas identical across ranks, eager and graphed
    assert torch.equal(torch.from_numpy(res[0][2]), torch.from_numpy(res[1][2]))
    assert torch.equal(torch.from_numpy(res[0][3]), torch.from_numpy(res[1][3]))


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
