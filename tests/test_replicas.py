"""The multi-GPU path on CPU: replicas only, so the ranks share nothing but the job-level
reduction of bench.py (the slowest replica's time, the sum of every replica's rows) and
the rule that rank 0 alone reports.  Two gloo ranks stand in for two GPUs."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out) -> None:
    import datetime

    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        # rank r: step time 10 + r ms, 96 - r rows, r tokens
        got = bench.reduce_over_ranks([10.0 + rank], [96.0 - rank, float(rank)])
        # a reduction with no counts still takes both collective steps on every rank
        only_max = bench.reduce_over_ranks([1.0 + 2 * rank], [])
        out.put((rank, got, only_max))
    finally:
        dist.destroy_process_group()


def test_two_replicas_reduce_max_time_and_sum_counts():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, got, only_max = out.get(timeout=120)
        results[rank] = (got, only_max)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        (maxes, sums), (m2, s2) = results[rank]
        assert maxes == [11.0]
        assert sums == [96.0 + 95.0, 1.0]
        assert m2 == [3.0] and s2 == []


def test_single_process_reduction_is_the_identity():
    import bench
    assert bench.reduce_over_ranks([4.5], [7.0]) == ([4.5], [7.0])


@pytest.mark.parametrize("rank", [1, 3])
def test_reference_arm_runs_on_rank_zero_only(rank):
    """Under torchrun the reference arm's other ranks exit without work."""
    import bench
    assert bench.run_reference(None, rank) is None
