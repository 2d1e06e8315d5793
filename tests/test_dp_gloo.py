"""Data-parallel request partitioning and the off-path reductions, as world-size-2 gloo ranks on
the CPU (the same host logic bench.py runs over NCCL, one process per GPU)."""

import datetime
import os
import socket

import pytest
import torch.multiprocessing as mp

from fast_dllm_relax_b200 import dp


def test_request_range_partitions_contiguously():
    for n in (0, 1, 5, 8, 256, 1023):
        for world in (1, 2, 3, 4, 8):
            rs = [dp.request_range(n, world, r) for r in range(world)]
            assert [i for r in rs for i in r] == list(range(n))
            sizes = [len(r) for r in rs]
            assert max(sizes) - min(sizes) <= 1
    assert dp.request_range(256, 8, 3) == range(96, 128)  # 32 requests per GPU
    with pytest.raises(ValueError):
        dp.request_range(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_requests, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        requests = [[i, i + 1, i + 2] for i in range(n_requests)]  # stand-in prompts
        local = dp.serve(requests, lambda p: [t * 10 for t in p], world, rank)
        seconds = 1.0 + rank  # per-rank device time; the job time is the max over ranks
        mx, sm = dp.reduce_max_sum([seconds], [float(3 * len(local))])
        gathered = dp.gather_results(local, n_requests)
        q.put((rank, [i for i, _ in local], mx, sm, gathered))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_serve_disjoint_ranges_and_reduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port, world, n = _free_port(), 2, 5
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, idx, mx, sm, gathered = q.get(timeout=120)
        results[rank] = (idx, mx, sm, gathered)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results[0][0] == [0, 1, 2] and results[1][0] == [3, 4]
    for r in range(world):
        assert results[r][1] == [2.0]        # max over ranks
        assert results[r][2] == [15.0]       # 5 requests x 3 tokens
    assert results[0][3] == [[i * 10, i * 10 + 10, i * 10 + 20] for i in range(n)]
    assert results[1][3] is None


def test_single_process_fallbacks():
    local = dp.serve([[1], [2], [3]], lambda p: p[0] * 2, 1, 0)
    assert dp.gather_results(local, 3) == [2, 4, 6]
    assert dp.reduce_max_sum([1.5], [2.0]) == ([1.5], [2.0])
    assert dp.world_info()[0] >= 1
