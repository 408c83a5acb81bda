"""Data-parallel gradient averaging (torch_vulkan_b200.dp) with world size 2 on CPU (gloo): the averaged
bucketed gradients equal the single-process average over both ranks' samples, replicas stay identical after
the optimizer step, and a rank that fails makes its peer's collective end with an error (host-side failure,
no GPU involved)."""

import datetime
import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    torch.manual_seed(0)
    m = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.GELU(), torch.nn.Linear(16, 4), torch.nn.Linear(4, 3))
    return m


def _sample(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(5, 8, generator=g), torch.randn(5, 3, generator=g)


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
    from torch_vulkan_b200.dp import BucketedGradAllReduce, flat_grads

    try:
        m = _model()
        params = list(m.parameters())
        buckets = [params[0:2], params[2:4], params[4:6]]  # one bucket per linear
        red = BucketedGradAllReduce(buckets)
        opt = torch.optim.AdamW(params, lr=1e-2, foreach=False)
        x, y = _sample(rank)
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before its backward")
        for step in range(2):
            loss = torch.nn.functional.mse_loss(m(x), y)
            loss.backward()
            red.wait()
            g = flat_grads(params).clone()
            opt.step()
            red.zero_grad()
        q.put((rank, "ok", g.numpy().copy(), torch.cat([p.detach().reshape(-1) for p in params]).numpy().copy()))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(2):
        r, status, a, b = q.get(timeout=120)
        out[r] = (status, a, b)
    for p in ps:
        p.join(timeout=60)
    return out


def test_bucketed_average_matches_single_process_and_replicas_agree():
    out = _run("ok")
    assert out[0][0] == "ok" and out[1][0] == "ok", out
    # reference: the same two steps in one process with the gradients averaged over both samples
    m = _model()
    params = list(m.parameters())
    opt = torch.optim.AdamW(params, lr=1e-2, foreach=False)
    for step in range(2):
        opt.zero_grad()
        for r in range(2):
            x, y = _sample(r)
            (torch.nn.functional.mse_loss(m(x), y) / 2).backward()
        g = torch.cat([p.grad.reshape(-1) for p in params]).clone()
        opt.step()
    g0, g1 = torch.from_numpy(out[0][1]), torch.from_numpy(out[1][1])
    w0, w1 = torch.from_numpy(out[0][2]), torch.from_numpy(out[1][2])
    assert torch.allclose(g0, g, atol=1e-6, rtol=1e-5)
    assert torch.equal(g0, g1)
    assert torch.equal(w0, w1)  # identical replicas after the optimizer
    assert torch.allclose(w0, torch.cat([p.detach().reshape(-1) for p in params]), atol=1e-6)


def test_failing_rank_makes_peer_collective_error():
    out = _run("fail")
    assert out[1][0] == "error"
    assert out[0][0] == "error", out[0]  # its all-reduce / wait ends with an error instead of hanging
