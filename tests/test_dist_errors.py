"""Cross-rank gather of per-layer error scalars on gloo CPU ranks (world size 2).

The patch path's only collective is the all-gather of each rank's per-layer measured errors
(deltakv_b200.metrics.gather_layer_errors); no KV crosses ranks.  These tests run it as two
CPU processes over gloo on 127.0.0.1, including a rank that leaves before the collective:
the surviving rank must get an error within the process group's short timeout, not hang.
"""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank: int, world: int, port: int, timeout_s: float) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _gather_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    from deltakv_b200.metrics import gather_layer_errors

    _init(rank, world, port, 30)
    local = torch.tensor([rank * 10.0 + i for i in range(5)], dtype=torch.float64)
    got = gather_layer_errors(local)
    torch.save(got, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_gather_layer_errors_two_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_gather_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    want = torch.tensor([[0.0, 1, 2, 3, 4], [10.0, 11, 12, 13, 14]], dtype=torch.float64)
    for r in range(2):
        assert torch.equal(torch.load(tmp_path / f"r{r}.pt"), want)


def _leaver_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    from deltakv_b200.metrics import gather_layer_errors

    _init(rank, world, port, 5)
    if rank == 1:
        os._exit(0)  # leaves between steps, with no collective in flight
    status = "no error"
    try:
        gather_layer_errors(torch.zeros(3, dtype=torch.float64))
    except Exception as e:  # gloo reports the lost peer or the timeout
        status = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(status)
    os._exit(0)


def test_gather_reports_a_lost_rank(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_leaver_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=60)
    alive = [p for p in ctx.processes if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung on the collective"
    assert (tmp_path / "rank0.txt").read_text().startswith("error")


def test_gather_single_process_is_identity():
    from deltakv_b200.metrics import gather_layer_errors

    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    x = torch.tensor([0.5, 0.25])
    assert torch.equal(gather_layer_errors(x), x.view(1, -1))


def _sharded_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    from deltakv_b200.metrics import gather_sharded_layer_errors

    _init(rank, world, port, 30)
    # 5 layers round-robin over 2 ranks (layer l on rank l mod 2): an uneven split
    mine = [l for l in range(5) if l % world == rank]
    local = torch.tensor([100.0 + l for l in mine], dtype=torch.float64)
    got = gather_sharded_layer_errors(local, mine, 5)
    torch.save(got, os.path.join(out_dir, f"s{rank}.pt"))
    status = "no error"
    try:  # both ranks claim layer 0: overlapping sets are rejected on every rank
        gather_sharded_layer_errors(torch.zeros(1, dtype=torch.float64), [0], 5)
    except ValueError:
        status = "rejected"
    with open(os.path.join(out_dir, f"s{rank}.txt"), "w") as f:
        f.write(status)
    dist.barrier()
    dist.destroy_process_group()


def test_gather_sharded_layer_errors_two_ranks(tmp_path):
    port = _free_port()
    mp.start_processes(_sharded_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    want = torch.tensor([100.0, 101, 102, 103, 104], dtype=torch.float64)
    for r in range(2):
        assert torch.equal(torch.load(tmp_path / f"s{r}.pt"), want)
        assert (tmp_path / f"s{r}.txt").read_text() == "rejected"
