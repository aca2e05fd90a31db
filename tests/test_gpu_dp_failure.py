"""A data-parallel rank that leaves between steps, on two GPUs with NCCL (NVLS off): the surviving
rank's host-side liveness check raises PeerLost before it launches the next step's all-reduce, so
no collective is left waiting for a peer that will never join it. The departing rank leaves with
none of its kernels or collectives in flight. Skipped on a box with fewer than two GPUs."""

import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from test_gpu_model import _bf16_tiny
    from test_gpu_train_step import _micro_batches

    from orthrus_training_b200.train_step import PeerLost, PeerMonitor, Trainer

    model, _ = _bf16_tiny(seed=3)
    monitor = PeerMonitor(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=20.0)
    trainer = Trainer(model, lr=1e-3, total_steps=10, num_anchors=8, kl_chunk_size=256, seed=9, world=world,
                      rank=rank, monitor=monitor)
    dev = torch.device("cuda", rank)
    done = 0
    try:
        for step in range(3):
            if rank == 1 and step == 1:
                torch.cuda.synchronize()  # nothing of this rank in flight when it leaves
                monitor.leave()
                out[1] = "left"
                return
            batches = [(i.to(dev), m.to(dev)) for i, m in _micro_batches(500 + 10 * step + rank, 1)]
            trainer.step(batches)
            torch.cuda.synchronize()
            done += 1
        out[rank] = "completed"
    except PeerLost as e:
        out[rank] = f"peer lost after {done} steps: {e}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_departed_rank_is_detected_before_the_next_all_reduce():
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    here = os.path.dirname(os.path.abspath(__file__))
    os.environ["PYTHONPATH"] = os.pathsep.join([here, os.path.dirname(here), os.environ.get("PYTHONPATH", "")])
    mp.start_processes(_rank, args=(2, port, out), nprocs=2, join=True, start_method="spawn")
    assert out[1] == "left"
    assert out[0].startswith("peer lost after 1 steps"), out[0]
