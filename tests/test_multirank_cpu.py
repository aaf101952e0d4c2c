"""The N>1 path of bench.py on CPU: two gloo ranks (world_size 2) join the
process group the way torchrun launches them, split every slice of a batch
across the ranks by bytes (greedy LPT: strong scaling, each TU on exactly one
rank), and combine bytes (sum) and step times (max) with the same helpers the
GPU run uses.  The data path has no collective; these reductions are the only
cross-rank traffic."""
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
    import numpy as np
    import torch.distributed as dist

    import bench
    from opencuda import synth
    r, w, _ = bench.dist_init("gloo")
    srcs = synth.lognormal_batch(64, seed=5678)
    buf, off = bench.c5_batch(r, w, n=64)   # rank 0 generates, rank 1 reads its file
    assert buf.tobytes() == "".join(srcs).encode()
    plan = bench.slice_plan(np.diff(off), 4, w)
    mine = [plan[j][r] for j in range(4)]
    shards = [bench.gather(buf, off, m) for m in mine]
    for m, (b, o) in zip(mine, shards):
        assert [bytes(b[int(o[k]):int(o[k + 1])]).decode() for k in range(len(m))] == \
            [srcs[i] for i in m]
    nbytes = float(sum(len(b) for b, _ in shards))
    total = bench.allreduce(nbytes, w, "cpu", "sum")
    slowest = bench.allreduce(1.0 + r, w, "cpu", "max")
    bench.barrier(w)
    q.put((r, w, [m.tolist() for m in mine], nbytes, total, slowest, len(buf)))
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
    (r0, w0, p0, b0, t0, m0, n0), (r1, w1, p1, b1, t1, m1, n1) = out
    assert (r0, r1, w0, w1) == (0, 1, 2, 2)
    every = sorted(i for j in range(4) for i in p0[j] + p1[j])
    assert every == list(range(64))       # every TU in one slice, on one rank
    for j in range(4):
        assert not set(p0[j]) & set(p1[j])
    assert t0 == t1 == b0 + b1 == n0      # whole-job bytes
    assert abs(b0 - b1) < 0.25 * n0       # balanced by bytes
    assert m0 == m1 == 2.0                # max over ranks


def test_slice_plans_cover_the_batch_once():
    sys.path.insert(0, str(ROOT))
    import numpy as np

    import bench
    rng = np.random.default_rng(3)
    sizes = rng.lognormal(8.0, 1.0, 5000).astype(np.int64) + 1
    for mode in ("sorted", "dealt"):
        for world in (1, 3):
            plan = bench.slice_plan(sizes, 7, world, mode)
            got = np.sort(np.concatenate([p for sl in plan for p in sl]))
            assert np.array_equal(got, np.arange(len(sizes)))
            per_slice = [int(sum(sizes[p].sum() for p in sl)) for sl in plan]
            assert abs(max(per_slice) - min(per_slice)) <= int(sizes.max())
    sorted_plan = bench.slice_plan(sizes, 7, 1, "sorted")
    assert int(sizes[sorted_plan[0][0]].min()) >= int(sizes[sorted_plan[1][0]].max())
    dealt = bench.slice_plan(sizes, 7, 1, "dealt")
    top7 = set(np.argsort(-sizes, kind="stable")[:7].tolist())
    assert {int(sl[0][0]) for sl in dealt} == top7    # one of the largest per slice
