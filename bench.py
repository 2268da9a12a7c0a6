"""Benchmark: ZipGEMM on B200 (W 4096x4096 bf16 ~ N(0, 0.02)
TCA-TBE compressed, X N=128 tokens ~ N(0, 1), SplitK=1, fp32 accumulate).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one ZipGEMM launch over one weight matrix. Multi-GPU (torchrun):
column-parallel weak scaling -- rank r holds output rows [4096 r, 4096 (r+1))
of a (4096 N) x 4096 weight (its own compressed shard, seeded by r) and the
same X; there is no data-path collective. The timed region is K CUDA-graph
replayed steps bracketed by barrier + synchronize; time = max over ranks.

L2 policy: each rank rotates through enough distinct compressed weights that
the rotating set exceeds the 126 MB L2, so every step streams its weight from
HBM.

`value` is algorithmic bytes per second: compressed W bytes + X (2KN) + Y (2MN).
`e2e` repeats the step through the public API from pinned host memory (H2D of
X + ZipGEMM + D2H of Y inside the timed region). `cpu_baseline` times the CPU
path (CPU decode of W + fp32 GEMM) on a bounded sample on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M_, K_, N_ = 4096, 4096, 128
L2_BYTES = 126 * 1024 * 1024
PROFILE_TRAFFIC = os.path.join(ROOT, "profiles", "zipgemm_config2_traffic.json")
METRIC = "ZipGEMM compressed-byte HBM GB/s (config 2: 4096x4096 W, N=128)"
CONFIG = {"workload": "config2_zipgemm_4096x4096_N128", "M": M_, "K": K_, "N": N_, "split_k": 1,
          "l2": "rotating compressed weight sets larger than the 126 MB L2", "global_batch": N_}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.path = gpu, None, None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        num = lambda s: s.replace(".", "", 1).isdigit()  # noqa: E731
        sm = [float(r[1]) for r in rows if num(r[1])]
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        smax = max(float(r[2]) for r in rows if num(r[2]))
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        load = [s for s in sm if s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows)}


def make_weights(zs, torch, rank, count, dev, first=0):
    comps = []
    for i in range(first, first + count):
        g = torch.Generator(device=dev).manual_seed(1000 * rank + i)
        w = (torch.randn(M_, K_, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        comps.append(zs.compress(w))
        del w
    return comps


def cpu_step_sample(max_steps: int = 10, cap_s: float = 15.0):
    """CPU path of one config-2 step on all host cores: decode W with the
    oracle port of the reference CPU decoder (bench_kv_cache_zipserv_decompress_
    token_scaling.cu:2106, row bands in parallel threads) + fp32 GEMM in torch.
    Returns (bytes/s, seconds per step, cores, sample description)."""
    import concurrent.futures as cf
    import ctypes as C

    import numpy as np
    import torch

    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from oracle_bindings import Oracle
    orc = Oracle()
    rng = np.random.default_rng(0)
    w32 = rng.standard_normal((M_, K_), dtype=np.float32) * 0.02
    wb = torch.from_numpy(w32).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    xb = torch.randn(N_, K_).to(torch.bfloat16)
    enc = orc.encode(wb)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    out = np.zeros((M_, K_), np.uint16)
    gtk = K_ // 64
    band = (M_ // 64 + cores - 1) // cores
    p = lambda a, off=0: C.c_void_p(a.ctypes.data + off)  # noqa: E731

    def decode_band(b):
        g0, g1 = b * band, min(M_ // 64, (b + 1) * band)
        if g0 >= g1:
            return 0
        return orc.lib.oracle_decode(p(enc.sign_mantissa), enc.sign_mantissa.size, p(enc.full), enc.full.size,
                                     p(enc.bitmap1, g0 * gtk * 512), p(enc.bitmap2, g0 * gtk * 512),
                                     p(enc.bitmap3, g0 * gtk * 512), p(enc.gt_offsets, g0 * gtk * 8),
                                     enc.start_exp, (g1 - g0) * 64, K_, p(out, g0 * 64 * K_ * 2))

    times = []
    t_end = time.perf_counter() + cap_s
    with cf.ThreadPoolExecutor(cores) as ex:
        while len(times) < max_steps and (time.perf_counter() < t_end or not times):
            t0 = time.perf_counter()
            assert all(r == 0 for r in ex.map(decode_band, range(cores)))
            wf = torch.from_numpy(out.view(np.int16)).view(torch.bfloat16).float()
            (xb.float() @ wf.t()).to(torch.bfloat16)
            times.append(time.perf_counter() - t0)
    assert np.array_equal(out, wb)
    per = statistics.median(times)
    nbytes = enc.compressed_bytes() + 2 * K_ * N_ + 2 * M_ * N_
    desc = (f"median of {len(times)} full config-2 steps: CPU decode of the 4096x4096 TCA-TBE weight "
            f"({cores} threads) + fp32 torch GEMM N=128 ({cores} threads)")
    return nbytes / per, per, cores, desc


def run_reference(args):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    t0 = time.perf_counter()
    v, per, cores, desc = cpu_step_sample(max_steps=max(3, min(args.steps, 10)))
    value = v / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded W ~ N(0,0.02), X ~ N(0,1))", "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": desc + "; decoder = oracle port of the reference CPU decoder (its source "
                                          "needs nvCOMP headers, not buildable here)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0}), flush=True)


def run_ncu(args):
    """Profiling mode: plain launches over the same rotating weights and X."""
    import torch

    import zipserv_asplos26_b200 as zs
    dev = torch.device("cuda", 0)
    comps = make_weights(zs, torch, 0, 1, dev)
    n_sets = max(2, -(-int(1.5 * L2_BYTES) // comps[0].compressed_bytes()))
    comps += make_weights(zs, torch, 0, n_sets - 1, dev, first=1)
    x = torch.randn(N_, K_, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)
    y = torch.empty(N_, M_, dtype=torch.bfloat16, device=dev)
    for i in range(args.warmup + args.steps):
        zs.zipgemm(comps[i % n_sets], x, out=y)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_mode": True, "launches": args.warmup + args.steps, "sets": n_sets}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ncu", action="store_true", help="plain launches for ncu, no timing")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.ncu:
        return run_ncu(args)

    import torch
    import torch.distributed as dist

    import zipserv_asplos26_b200 as zs
    from zipserv_asplos26_b200._lib import lib

    lib()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    W = max(3, args.warmup)
    K = args.steps

    comps = make_weights(zs, torch, rank, 1, dev)
    cb = comps[0].compressed_bytes()
    n_sets = max(2, -(-int(1.5 * L2_BYTES) // cb))
    comps += make_weights(zs, torch, rank, n_sets - 1, dev, first=1)
    x = torch.randn(N_, K_, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)
    ys = [torch.empty(N_, M_, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    nbytes = cb + 2 * K_ * N_ + 2 * M_ * N_

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(W):
            zs.zipgemm(comps[i % n_sets], x, out=ys[i % 2])
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(K):
                zs.zipgemm(comps[i % n_sets], x, out=ys[i % 2])
        graph.replay()
        stream.synchronize()

        sampler = ClockSampler(local)
        sampler.start()
        t_soak = time.perf_counter()
        while time.perf_counter() - t_soak < 1.0:   # load the GPU while the sampler runs
            graph.replay()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms_total = e0.elapsed_time(e1)
        clocks = sampler.stop()

        # e2e through the public API from pinned host memory
        xh = x.cpu().pin_memory()
        yh = torch.empty(N_, M_, dtype=torch.bfloat16).pin_memory()
        xd = torch.empty_like(x)
        for i in range(W):
            xd.copy_(xh, non_blocking=True)
            zs.zipgemm(comps[i % n_sets], xd, out=ys[0])
            yh.copy_(ys[0], non_blocking=True)
        stream.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
        for i in range(K):
            ev[i][0].record(stream)
            xd.copy_(xh, non_blocking=True)
            zs.zipgemm(comps[i % n_sets], xd, out=ys[0])
            yh.copy_(ys[0], non_blocking=True)
            ev[i][1].record(stream)
        stream.synchronize()
        e2e_ms = sum(a.elapsed_time(b) for a, b in ev)

    t = torch.tensor([ms_total, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms = t.tolist()
    ms_step = ms_total / K
    peak, peak_kind = peaks()
    achieved = nbytes / (ms_step / 1e3) / 1e9
    traffic = None
    if os.path.exists(PROFILE_TRAFFIC):
        with open(PROFILE_TRAFFIC) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    if rank == 0:
        line = {
            "metric": METRIC, "value": world * nbytes * K / (ms_total / 1e3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_step, "us_per_gemm": ms_step * 1e3,
            "tflops": 2.0 * M_ * N_ * K_ / (ms_step / 1e3) / 1e12, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded W ~ N(0,0.02) per rank and set, X ~ N(0,1))",
            "config": dict(CONFIG, parallelism=f"column-parallel weak scaling, {world} shard(s)",
                           rotating_sets=n_sets, compressed_bytes=cb, ratio=round(2 * M_ * K_ / cb, 4)),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": nbytes},
            "e2e": {"value": world * nbytes * K / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": 2 * N_ * K_, "d2h_bytes_per_step": 2 * N_ * M_,
                    "ms_per_step": e2e_ms / K},
            "gpu_launches": K,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            v, per, cores, desc = cpu_step_sample()
            line["cpu_baseline"] = {"value": v / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                    "sample": desc, "ms_per_step": per * 1e3}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
