"""Data-parallel plumbing on CPU ranks (gloo, world size 2): per-layer gradient buckets are
averaged by all-reduce hooks during backward, and a rank that fails before the collective makes
the other rank's collective end with an error instead of hanging."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class TwinModel(torch.nn.Module):
    """Two 'layers' with parameters named like the diffusion twins."""

    def __init__(self):
        super().__init__()
        torch.manual_seed(0)
        self.model = torch.nn.Module()
        self.model.layers = torch.nn.ModuleList()
        for _ in range(2):
            layer = torch.nn.Module()
            layer.self_attn = torch.nn.Module()
            layer.self_attn.q_proj_diff = torch.nn.Linear(4, 4, bias=False)
            layer.self_attn.k_proj_diff = torch.nn.Linear(4, 4, bias=False)
            self.model.layers.append(layer)

    def forward(self, x):
        for layer in self.model.layers:
            x = torch.tanh(layer.self_attn.k_proj_diff(layer.self_attn.q_proj_diff(x)))
        return x.sum()


def _bucket_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    from orthrus_training_b200.train_step import GradBuckets

    model = TwinModel()
    params = [p for p in model.parameters()]
    buckets = GradBuckets(model, params, world)
    buckets.zero()
    # two micro-batches; only the last one all-reduces
    for j, scale in enumerate((1.0, 2.0)):
        buckets.arm(j == 1)
        x = torch.full((3, 4), float(rank + 1) * scale)
        model(x).backward()
    buckets.wait()
    out[rank] = torch.cat([p.grad.flatten() for p in params]).clone()
    dist.destroy_process_group()


def _local_grads(rank):
    model = TwinModel()
    for scale in (1.0, 2.0):
        model(torch.full((3, 4), float(rank + 1) * scale)).backward()
    return torch.cat([p.grad.flatten() for p in model.parameters()])


def test_bucketed_allreduce_averages_twin_grads():
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.start_processes(_bucket_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    expect = (_local_grads(0) + _local_grads(1)) / 2
    assert torch.allclose(out[0], expect, atol=1e-6) and torch.allclose(out[1], expect, atol=1e-6)


def _failing_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        out[1] = "left"  # leaves between steps, before the collective, without joining it
        return
    try:
        dist.all_reduce(torch.ones(4))
        out[0] = "completed"
    except Exception as e:  # noqa: BLE001
        out[0] = f"error: {type(e).__name__}"


def test_missing_rank_ends_the_collective_with_an_error():
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.start_processes(_failing_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    assert out[1] == "left"
    assert out[0].startswith("error")


def _monitored_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    from orthrus_training_b200.train_step import PeerLost, PeerMonitor

    store = dist.distributed_c10d._get_default_store()
    mon = PeerMonitor(store, rank, world, timeout_s=5.0)
    model = TwinModel()
    steps_done = 0
    try:
        for step in range(3):
            if rank == 1 and step == 1:
                mon.leave()  # between steps, with nothing in flight
                out[1] = "left"
                return
            mon.beat(step)
            mon.check(step)  # before the step's collective
            x = torch.ones(2, 4)
            loss = model(x)
            loss.backward()
            for p in model.parameters():
                dist.all_reduce(p.grad)
            steps_done += 1
        out[rank] = "completed"
    except PeerLost as e:
        out[rank] = f"peer lost after {steps_done} steps: {e}"
    finally:
        if rank == 0:
            dist.destroy_process_group()


def test_peer_monitor_stops_before_the_collective_a_departed_rank_would_not_join():
    """The heartbeat check raises PeerLost on the surviving rank before it launches the next
    step's collective (no collective times out), after one step completed on both ranks."""
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.start_processes(_monitored_worker, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    assert out[1] == "left"
    assert out[0].startswith("peer lost after 1 steps"), out[0]
