"""The N>1 path of bench.py on CPU: two gloo ranks (world_size 2) join the
process group the way torchrun launches them, compile disjoint TU shards
(weak scaling: each rank its own seed), and combine bytes (sum) and step
times (max) with the same helpers the GPU run uses.  The data path has no
collective; these two reductions are the only cross-rank traffic."""
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    import bench
    r, w, _ = bench.dist_init("gloo")
    srcs = bench.workload(r, 6)
    nbytes = float(sum(len(s.encode()) for s in srcs))
    total = bench.allreduce(nbytes, w, "cpu", "sum")
    slowest = bench.allreduce(1.0 + r, w, "cpu", "max")
    bench.barrier(w)
    q.put((r, w, srcs[0], nbytes, total, slowest))
    dist.destroy_process_group()


def test_two_gloo_ranks_shard_and_reduce():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, w0, s0, b0, t0, m0), (r1, w1, s1, b1, t1, m1) = out
    assert (r0, r1, w0, w1) == (0, 1, 2, 2)
    assert s0 != s1                       # disjoint shards
    assert t0 == t1 == b0 + b1            # whole-job bytes
    assert m0 == m1 == 2.0                # max over ranks
