#!/usr/bin/env python
"""Benchmark of the B200 batch compiler (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step"): the batch lexer over the lexer/preprocessor stress
text -- 1 GiB of seeded CUDA-C-like source per GPU in 16 KiB TUs (identifiers
Zipf(1.1) over 10k names, 5% #define lines, hex/float/suffixed literals, 10%
comments).  Each GPU lexes its own 1 GiB (weak scaling, no collective on the
data path); the batch is larger than L2, so no flush is needed between steps.

* ``value``      -- source GB/s over all GPUs with the batch resident in HBM
                    (``ocb_lex_device``), timed with CUDA events on the
                    launching stream, max over ranks.
* ``e2e``        -- the same metric through the public host API
                    (``Context.lex_batch``: pinned source -> device -> token
                    arrays back on the host), copies inside the timed region.
* ``roofline``   -- algorithmic bytes (source read once + one 12-byte token
                    record written) / step time, against measured HBM peak.
* ``cpu_baseline`` -- the reference's own lexer (oracle/_ref/py, pure Python)
                    on all host cores over a bounded sample of the same TUs.

``--impl reference`` times only the reference lexer (rank 0; other ranks exit).
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
TOKEN_RECORD_BYTES = 12     # start u32 + kind<<24|len u32 + line u32
BYTES_PER_GPU = 1 << 30
TU_BYTES = 16384


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
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            if len(r) >= 9:
                for nm, v in zip(names, r[5:9]):
                    if v.lower() == "active":
                        reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_init(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=None)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def allmax(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def allsum(x, world, device):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def reference_sample(buf, off, n_tu):
    return [buf[int(off[i]):int(off[i + 1])].decode() for i in range(n_tu)]


def run_reference(args, rank):
    """The reference's own lexer (pure Python) on all host cores."""
    if rank != 0:
        return
    from opencuda_b200 import synth
    from oracle import ref_runner
    buf, off = synth.lexstress_batch(total_bytes=BYTES_PER_GPU, tu_bytes=TU_BYTES, seed=99)
    cores = len(os.sched_getaffinity(0))
    n_tu = 8 * cores  # ~16 KiB each: a few seconds of work per step
    srcs = reference_sample(buf, off, n_tu)
    nbytes = sum(len(s) for s in srcs)
    with ref_runner.RefPool(cores) as pool:
        for _ in range(args.warmup):
            pool.time_lex(srcs)
        ts = [pool.time_lex(srcs)[0] for _ in range(args.steps)]
    t = float(np.mean(ts))
    v = nbytes / t / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s source (lexer)",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "config": {"workload": "lexer over lexstress text (16 KiB TUs)", "tu_bytes": TU_BYTES,
                   "bytes_per_gpu": BYTES_PER_GPU},
        "cpu_baseline": {"value": v, "unit": "GB/s source (lexer)", "cores": cores,
                         "kind": "reference",
                         "sample": f"{n_tu} TUs ({nbytes} bytes) of the 1 GiB batch per step"},
        "e2e": {"value": v, "unit": "GB/s source (lexer)", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--bytes", type=int, default=BYTES_PER_GPU,
                    help="source bytes per GPU (default 1 GiB)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank, world, local = dist_init(args.gpus)
    if args.impl == "reference":
        run_reference(args, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    import torch
    from opencuda_b200 import api, synth
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = api.Context(local)

    buf, off = synth.lexstress_batch(total_bytes=args.bytes, tu_bytes=TU_BYTES,
                                     seed=99 + 1000 * rank)
    n_tu = len(off) - 1
    nbytes = len(buf)
    host_src = torch.frombuffer(bytearray(buf), dtype=torch.uint8).pin_memory()
    host_off = torch.from_numpy(off.astype(np.int64))
    d_src = host_src.to(dev)
    d_off = host_off.to(dev)
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

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    n_tok = int(d_n.item())
    if n_tok > cap:
        raise SystemExit(f"token capacity {cap} < {n_tok}")
    bad = int((d_status != 0).sum().item())

    clocks = ClockSampler(local)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    barrier(world)
    t_step = e0.elapsed_time(e1) / 1e3 / args.steps
    t_max = allmax(t_step, world, dev)
    total_bytes = allsum(float(nbytes), world, dev)
    total_tok = allsum(float(n_tok), world, dev)
    value = total_bytes / t_max / 1e9

    # end to end through the public host API (pinned source, tokens to host)
    e2e = None
    if not args.no_e2e:
        src_np = host_src.numpy()
        ctx.lex_batch(buf=src_np, tu_off=off)
        barrier(world)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            tb = ctx.lex_batch(buf=src_np, tu_off=off)
        t_e2e = (time.perf_counter() - t0) / args.steps
        t_e2e = allmax(t_e2e, world, dev)
        e2e = {"value": total_bytes / t_e2e / 1e9, "unit": "GB/s source",
               "h2d_bytes_per_step": int(nbytes + 8 * (n_tu + 1)),
               "d2h_bytes_per_step": int(TOKEN_RECORD_BYTES * len(tb.start) +
                                         8 * (n_tu + 1) + 4 * n_tu + 8)}

    peak, peak_kind = measured_peak()
    alg = nbytes + TOKEN_RECORD_BYTES * n_tok
    achieved = alg / t_step / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from oracle import ref_runner
            cores = len(os.sched_getaffinity(0))
            k = 8 * cores
            srcs = reference_sample(buf, off, k)
            with ref_runner.RefPool(cores) as pool:
                pool.time_lex(srcs[:cores])
                tcpu, _ = pool.time_lex(srcs)
            sb = sum(len(s) for s in srcs)
            cpu = {"value": sb / tcpu / 1e9, "unit": "GB/s source (lexer)", "cores": cores,
                   "kind": "reference",
                   "sample": f"{k} of the {n_tu} TUs ({sb} bytes), reference lex() in "
                             f"{cores} processes"}
        except Exception as ex:  # noqa: BLE001
            cpu = {"value": None, "error": f"{type(ex).__name__}: {ex}"}

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": "GB/s source (lexer)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_max * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": f"lexer over lexstress text: {nbytes >> 20} MiB per GPU, "
                                   "16 KiB TUs",
                       "tu_bytes": TU_BYTES, "bytes_per_gpu": nbytes, "tokens": int(total_tok),
                       "l2": "inputs (1 GiB) larger than L2, no flush",
                       "tu_status_nonzero": bad, "parallelism": f"tu-shard x{world}"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": None,
                         "algorithmic_bytes_per_step": int(alg),
                         "scope": "whole lexer step (all kernels)"},
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": 8 * args.steps,
            "clocks": clk,
        }), flush=True)
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
