"""The N > 1 host path of bench.py (torchrun, one process per GPU; rank 0 drives the model split over
every GPU, the other ranks report no work): two gloo ranks on the CPU combine their device and wall
times as the maximum over ranks and their positions as the sum, so the line is rank 0's stream; the
reference arm runs on rank 0 alone."""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out, idle_others=False):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    if idle_others:
        work = (1000.0, 2000.0, 256) if rank == 0 else (0.0, 0.0, 0)
    else:
        work = (1000.0 * (rank + 1), 2000.0 + rank, 256)
    t_dev, t_wall, total = bench.combine_ranks(dist, *work)
    out.put((rank, t_dev, t_wall, total))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_combine_max_time_and_sum_positions():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, t_dev, t_wall, total in got:
        assert (t_dev, t_wall, total) == (2000.0, 2001.0, 512.0), rank


def test_split_model_line_is_rank_zeros_stream():
    """bench.py --gpus 2: rank 0 drives the split model, rank 1 reports zeros; the combined line is
    rank 0's device time, wall time and positions."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q, True)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(2))
    for rank, t_dev, t_wall, total in got:
        assert (t_dev, t_wall, total) == (1000.0, 2000.0, 256.0), rank


def test_single_rank_is_identity():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.combine_ranks(None, 5.0, 6.0, 7) == (5.0, 6.0, 7)


def test_reference_arm_other_ranks_exit_quietly(monkeypatch, capsys):
    """Under torchrun only rank 0 runs the reference arm and prints; the others return at once."""
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("LOCAL_RANK", "1")

    class A:
        config, steps, warmup = "SmolLM2-135M-q8_0", 3, 3
    bench.bench_reference(A())
    assert capsys.readouterr().out == ""
