"""The multi-GPU host logic of bench.py on CPU: two ranks over `gloo` (one
process per rank, rendezvous on 127.0.0.1, as torchrun sets it up).  The
data path has no collective -- ranks serve independent sequences -- so what
is shared is the barrier, the max-over-ranks timing, the summed counts and
the longest-prompt-first partition of the many-request workload."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench
    import torch.distributed as td

    r, w, local = bench.dist()
    assert (r, w, local) == (rank, world, rank)
    bench.barrier(w)
    mx = bench.allreduce([float(rank + 1), 10.0 * rank], w, "max")
    sm = bench.allreduce([1.0, float(rank)], w, "sum")
    reqs = bench.serve_requests()
    mine = bench.partition(reqs, w)[r]

    class Args:
        warmup, steps = 1, 1

    ref = bench.run_reference(Args(), r, w) if r != 0 else None  # rank != 0: no work, no output
    out.put((rank, mx, sm, sorted(mine), ref))
    bench.barrier(w)
    td.destroy_process_group()


def test_two_ranks_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, mx, sm, _, ref in res:
        assert mx == [2.0, 10.0] and sm == [2.0, 1.0]
        assert ref is None
    # the partition covers every request exactly once and balances the work
    import importlib
    sys.path.insert(0, ROOT)
    bench = importlib.import_module("bench")
    reqs = bench.serve_requests()
    parts = [set(r[3]) for r in res]
    assert parts[0].isdisjoint(parts[1]) and parts[0] | parts[1] == set(range(len(reqs)))
    work = [sum(len(reqs[i][0]) + bench.SERVE_GEN for i in p) for p in parts]
    assert abs(work[0] - work[1]) <= max(len(p) for p, _ in reqs) + bench.SERVE_GEN


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_partition_balance(world):
    sys.path.insert(0, ROOT)
    import bench
    reqs = bench.serve_requests()
    parts = bench.partition(reqs, world)
    assert sorted(i for p in parts for i in p) == list(range(len(reqs)))
    work = [sum(len(reqs[i][0]) + bench.SERVE_GEN for i in p) for p in parts]
    assert max(work) - min(work) <= max(len(p) for p, _ in reqs) + bench.SERVE_GEN
