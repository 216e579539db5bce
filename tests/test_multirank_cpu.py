"""The N > 1 host logic of bench.py on CPU: two gloo ranks (spawned
processes, 127.0.0.1) initialise through dist_init, agree on the max-over-ranks
time, and split the batch workload's requests so that every request is owned
by exactly one rank."""
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, total, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(ws),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import bench
    got_ws, got_rank, _ = bench.dist_init()
    assert (got_ws, got_rank) == (ws, rank)
    m = bench.max_over_ranks(10.0 + rank, ws)
    bench.barrier(ws)
    import torch
    mine = bench.rank_requests(total, ws, rank)
    everyone = [None] * ws
    dist.all_gather_object(everyone, mine)
    dist.destroy_process_group()
    q.put((rank, m, everyone))


def test_two_gloo_ranks():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.is_available():
        pytest.skip("the CPU path is tested where no GPU is visible")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ws, total = 2, 64
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, total, q)) for r in range(ws)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(ws)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, m, everyone in out:
        assert m == 10.0 + ws - 1  # the max over ranks
        owned = sorted(r for part in everyone for r in part)
        assert owned == list(range(total))  # each request on exactly one rank
        assert all(len(part) == total // ws for part in everyone)


def test_rank_requests_rejects_uneven_split():
    sys.path.insert(0, ROOT)
    import bench
    with pytest.raises(SystemExit):
        bench.rank_requests(63, 2, 0)
    assert bench.rank_requests(8, 4, 3) == [6, 7]
