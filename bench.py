#!/usr/bin/env python
"""Benchmark of the B200 batch compiler (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): compile 4,096 seeded random kernels (50-200 statements
each, ~4.6 KB, ~19 MB of CUDA C per GPU; 60% s32 / 40% f32 arithmetic,
if/else depth <= 3, unrollable for loops of trip 2-16, atomics and
__shfl_sync) to PTX: preprocess -> lex -> parse -> optimize -> register
allocation -> PTX text, with the arena reruns for TUs that outgrow their first
slice.  Each GPU compiles its own 4,096 kernels (another seed per rank: weak
scaling, TUs shard with no collective).  The working set of a step (arenas of
~13 GB) is far larger than L2, so no flush is needed between steps.

* ``value``      -- source MB/s over all GPUs with the batch resident in HBM
                    (``ocb_compile_device``), timed with CUDA events on the
                    context's stream, max over ranks.
* ``e2e``        -- the same metric through the public host API
                    (``Context.compile_batch``: pinned source -> device -> PTX
                    text, offsets and statuses back on the host).
* ``roofline``   -- the dominant kernel: end-to-end compile bytes (source +
                    PTX of the TUs of one launch) / its mean launch time,
                    against the measured HBM copy peak.
* ``cpu_baseline`` -- the reference compiler (pure Python, oracle/_ref/py) on
                    all host cores over a bounded sample of the same kernels.
* ``lexer``      -- the batch lexer over 1 GiB of lexer stress text per GPU
                    (GB/s of source and its HBM roofline fraction).
* ``latency_sgemm`` -- batch-1 latency of the tiled SGEMM kernel, end to end.

``--impl reference`` times only the reference compiler (rank 0; other ranks
exit without work).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "source MB/s compiled to byte-identical PTX at 1/2/4/8 B200; lexer GB/s vs HBM"
UNIT = "MB/s source"
N_KERNELS = 4096
SEED = 1234
RANK_SEED_STRIDE = 1_000_000
TOKEN_RECORD_BYTES = 12     # start u32 + kind<<24|len u32 + line u32
LEX_BYTES = 1 << 30
LEX_TU_BYTES = 16384
WORKLOAD = ("4,096 seeded random kernels (50-200 stmts, ~4.6 KB each) compiled to PTX "
            "per GPU")

# DRAM bytes (read + write) per TU of k_cc_opt from an ncu capture of one
# launch over the first 256 kernels of this workload (370.5 MB read + 760.2 MB
# written); the full 4,096-kernel launch is too large to capture under ncu,
# so the figure is scaled by the TUs of one launch.
NCU_OPT_DRAM_BYTES_PER_TU = (370.5e6 + 760.2e6) / 256


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        ok = [r for r in self.rows if len(r) >= 9]
        sm = [float(r[1]) for r in ok if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in ok if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in ok:
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init(backend: str = "nccl"):
    """Rank, world size and local rank from the torchrun environment; joins
    the process group when there is more than one rank (NCCL on the GPU box,
    gloo in the CPU tests of this logic)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allreduce(x, world, device, op="max"):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def workload(rank, n=N_KERNELS):
    """This rank's kernels: its own seed, so ranks compile disjoint TUs."""
    from opencuda_b200 import synth
    return synth.random_batch(n, seed=SEED + RANK_SEED_STRIDE * rank)


def cpu_sample_size(cores):
    # ~32 kernels per core: a few seconds of wall time, tens of CPU-seconds
    return min(N_KERNELS, 32 * cores)


def time_reference(srcs, cores, steps, warmup):
    """Wall seconds per step of the reference compiler over ``srcs``."""
    from oracle import ref_runner
    with ref_runner.RefPool(cores) as pool:
        for _ in range(warmup):
            pool.time_compile(srcs)
        return [pool.time_compile(srcs)[0] for _ in range(steps)]


def run_reference(args, rank, world):
    """The reference's own compiler (pure Python) on all host cores."""
    if rank != 0:
        return
    srcs_all = workload(0)
    cores = len(os.sched_getaffinity(0))
    k = cpu_sample_size(cores)
    srcs = srcs_all[:k]
    nbytes = sum(len(s.encode()) for s in srcs)
    ts = time_reference(srcs, cores, args.steps, args.warmup)
    t = float(np.mean(ts))
    v = nbytes / t / 1e6
    sample = (f"first {k} of the {N_KERNELS} kernels ({nbytes} bytes) per step, "
              f"reference preprocess->parse->optimize->ir_to_ptx in {cores} processes")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "n_kernels": N_KERNELS, "seed": SEED},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


class DevArray:
    """A device address as a CUDA-array-interface object (for torch.as_tensor)."""

    def __init__(self, ptr, n, typestr):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def count_launches(fn):
    """Kernels launched by one call of ``fn`` (CUPTI through torch.profiler)."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = {}
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        nm = e.name
        if nm.startswith("Memcpy") or nm.startswith("Memset") or "memcpy" in nm.lower() \
                or "memset" in nm.lower():
            continue
        short = nm.split("(")[0].split("<")[0].split("::")[-1] or nm[:40]
        names[short] = names.get(short, 0) + 1
    return sum(names.values()), names


def lexer_measure(ctx, api, synth, dev, rank, steps, warmup, peak, nbytes_req):
    """Lexer GB/s over the lexer stress text (resident in HBM)."""
    import torch
    buf, off = synth.lexstress_batch(total_bytes=nbytes_req, tu_bytes=LEX_TU_BYTES,
                                     seed=99 + 1000 * rank)
    n_tu = len(off) - 1
    nbytes = len(buf)
    d_src = torch.frombuffer(bytearray(buf), dtype=torch.uint8).to(dev)
    d_off = torch.from_numpy(off.astype(np.int64)).to(dev)
    cap = nbytes // 2 + n_tu + 1   # > 2x the measured token density of this text
    d_start = torch.empty(cap, dtype=torch.int32, device=dev)
    d_kl = torch.empty(cap, dtype=torch.int32, device=dev)
    d_line = torch.empty(cap, dtype=torch.int32, device=dev)
    d_tto = torch.empty(n_tu + 1, dtype=torch.int64, device=dev)
    d_status = torch.empty(n_tu, dtype=torch.int32, device=dev)
    d_n = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        ctx.lex_device(d_src.data_ptr(), nbytes, d_off.data_ptr(), n_tu, d_start.data_ptr(),
                       d_kl.data_ptr(), d_line.data_ptr(), cap, d_tto.data_ptr(),
                       d_status.data_ptr(), d_n.data_ptr(), stream.cuda_stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    n_tok = int(d_n.item())
    if n_tok > cap:
        raise SystemExit(f"token capacity {cap} < {n_tok}")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / steps
    alg = nbytes + TOKEN_RECORD_BYTES * n_tok
    del d_src, d_start, d_kl, d_line
    torch.cuda.empty_cache()
    return {"value": nbytes / t / 1e9, "unit": "GB/s source", "bytes": nbytes,
            "tokens": n_tok, "ms_per_step": t * 1e3,
            "workload": f"lexer stress text, {nbytes >> 20} MiB in 16 KiB TUs",
            "roofline": {"bound": "hbm", "achieved": alg / t / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": alg / t / 1e9 / peak,
                         "algorithmic_bytes": alg,
                         "scope": "whole lexer step (source + 12 B per token record)"}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernels", type=int, default=N_KERNELS,
                    help="kernels per GPU (default 4096; smaller only for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-lexer", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true",
                    help="skip the CUPTI launch count (for runs under ncu)")
    ap.add_argument("--lexer-bytes", type=int, default=LEX_BYTES)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank, world, local = dist_init()
    if args.impl == "reference":
        run_reference(args, rank, world)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch
    from opencuda_b200 import api, synth
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = api.Context(local)
    peak, peak_kind = measured_peak()

    srcs = workload(rank, args.kernels)
    buf, off = api.pack_sources(srcs)
    n_tu = len(srcs)
    nbytes = len(buf)
    host_src = torch.from_numpy(buf.copy()).pin_memory()
    d_src = host_src.to(dev)
    d_off = torch.from_numpy(off.astype(np.int64)).to(dev)
    stream = torch.cuda.ExternalStream(ctx.stream, device=dev)
    torch.cuda.synchronize()   # the batch is on the device before the context's stream reads it

    def step():
        return ctx.compile_device(d_src.data_ptr(), nbytes, d_off.data_ptr(), n_tu, 2)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    launches, launch_names = None, None
    if not args.no_launch_count:
        try:
            launches, launch_names = count_launches(step)
        except Exception as ex:  # noqa: BLE001
            launch_names = {"error": f"{type(ex).__name__}: {ex}"}

    ctx.kernel_profile(True)
    clocks = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        d_out, out_bytes, d_out_off, d_status = step()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ktimes = ctx.kernel_times()
    ctx.kernel_profile(False)
    barrier(world)
    t_step = e0.elapsed_time(e1) / 1e3 / args.steps
    t_max = allreduce(t_step, world, dev, "max")
    total_bytes = allreduce(float(nbytes), world, dev, "sum")
    value = total_bytes / t_max / 1e6

    # statuses of the device result (a view of the context's buffer)
    st_host = (torch.as_tensor(DevArray(d_status, n_tu, "<i4"), device=dev).cpu().numpy()
               if n_tu else np.zeros(0, np.int32))
    n_ok = int((st_host == 0).sum())
    n_unsup = int((st_host == api.TU_UNSUPPORTED).sum())
    n_over = int((st_host == api.TU_OVERFLOW).sum())
    n_raise = int(((st_host > 0) & (st_host < 0x100)).sum())
    ok_bytes = int(sum(int(off[i + 1] - off[i]) for i in range(n_tu) if st_host[i] == 0))

    # roofline of the dominant kernel: source + PTX bytes of the TUs it processed
    dom = max(ktimes, key=lambda k: ktimes[k][0])
    dom_ms, dom_n = ktimes[dom]
    tus_per_launch = n_tu * args.steps / max(dom_n, 1)
    alg_per_launch = (nbytes + out_bytes) * args.steps / max(dom_n, 1)
    t_launch = dom_ms / 1e3 / max(dom_n, 1)
    achieved = alg_per_launch / t_launch / 1e9
    traffic = (NCU_OPT_DRAM_BYTES_PER_TU * tus_per_launch
               if (NCU_OPT_DRAM_BYTES_PER_TU is not None and dom == "k_cc_opt") else None)
    ktot = sum(v[0] for v in ktimes.values())
    kernels = {k: {"ms_total": v[0], "launches": v[1],
                   "share_of_compile_kernels": (v[0] / ktot if ktot else None),
                   "share_of_step": v[0] / 1e3 / (t_step * args.steps)}
               for k, v in ktimes.items()}

    # end to end through the public host API (pinned source, PTX back on the host)
    e2e = None
    if not args.no_e2e:
        src_np = host_src.numpy()
        tb = ctx.compile_batch(buf=src_np, tu_off=off)
        barrier(world)
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            tb = ctx.compile_batch(buf=src_np, tu_off=off)
        f1.record(stream)
        torch.cuda.synchronize()
        t_e2e = f0.elapsed_time(f1) / 1e3 / args.steps
        t_e2e = allreduce(t_e2e, world, dev, "max")
        e2e = {"value": total_bytes / t_e2e / 1e6, "unit": UNIT,
               "ms_per_step": t_e2e * 1e3,
               "h2d_bytes_per_step": int(nbytes + 8 * (n_tu + 1)),
               "d2h_bytes_per_step": int(len(tb.data) + 8 * (n_tu + 1) + 4 * n_tu + 4 * n_tu)}

    # batch-1 latency of the tiled SGEMM kernel (public API, end to end)
    lat = None
    if rank == 0:
        for _ in range(3):
            ctx.compile_batch([synth.SGEMM_SRC])
        ts = []
        for _ in range(10):
            t0 = time.perf_counter()
            ctx.compile_batch([synth.SGEMM_SRC])
            ts.append(time.perf_counter() - t0)
        lat = {"ms": float(np.median(ts)) * 1e3, "source_bytes": len(synth.SGEMM_SRC)}

    lexer = None
    if not args.no_lexer:
        lexer = lexer_measure(ctx, api, synth, dev, rank, args.steps, args.warmup, peak,
                              args.lexer_bytes)
        lexer["value"] = allreduce(lexer["bytes"], world, dev, "sum") / \
            allreduce(lexer["ms_per_step"] / 1e3, world, dev, "max") / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cores = len(os.sched_getaffinity(0))
            k = cpu_sample_size(cores)
            sb = sum(len(s.encode()) for s in srcs[:k])
            tcpu = time_reference(srcs[:k], cores, 1, 1)[0]
            cpu = {"value": sb / tcpu / 1e6, "unit": UNIT, "cores": cores, "kind": "reference",
                   "sample": f"first {k} of the {n_tu} kernels ({sb} bytes), reference "
                             f"preprocess->parse->optimize->ir_to_ptx in {cores} processes"}
            if lat is not None:
                from oracle import ref_runner
                with ref_runner.RefPool(1) as pool:
                    pool.time_compile([synth.SGEMM_SRC])
                    tl = [pool.time_compile([synth.SGEMM_SRC])[0] for _ in range(5)]
                lat["reference_ms"] = float(np.median(tl)) * 1e3
        except Exception as ex:  # noqa: BLE001
            cpu = {"value": None, "error": f"{type(ex).__name__}: {ex}"}

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_max * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": WORKLOAD if n_tu == N_KERNELS
                       else f"{n_tu} of the {N_KERNELS} seeded random kernels",
                       "n_kernels": n_tu, "source_bytes_per_gpu": nbytes,
                       "ptx_bytes_per_gpu": int(out_bytes), "seed": SEED,
                       "tu_status": {"ok": n_ok, "reference_raises": n_raise,
                                     "unsupported": n_unsup, "overflow": n_over},
                       "ok_source_bytes": ok_bytes,
                       "l2": "working set (~13 GB of arenas) larger than L2, no flush",
                       "parallelism": f"tu-shard x{world}"},
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": alg_per_launch,
                         "tus_per_launch": tus_per_launch,
                         "mean_launch_ms": t_launch * 1e3,
                         "per_unit": "source bytes + PTX bytes of each TU"},
            "kernels": kernels,
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": (launches * args.steps if launches is not None else None),
            "gpu_launches_per_step": launch_names,
            "latency_sgemm": lat,
            "lexer": lexer,
            "clocks": clk,
        }), flush=True)
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
