"""Benchmark: ZipGEMM on B200 (W 4096x4096 bf16 ~ N(0, 0.02)
TCA-TBE compressed, X N=128 tokens ~ N(0, 1), SplitK=1, fp32 accumulate).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one config-2 GEMM. Multi-GPU (torchrun): row-parallel strong
scaling, as a tensor-parallel O / down projection runs -- rank r holds columns
[K r / N, K (r+1) / N) of W (its own compressed shard, seeded by r) and of X,
and the all-reduce of the partial Ys is fused into the ZipGEMM (each CTA
stores its rows into every rank's exchange buffer over NVLink and sums the
ranks' rows once they have landed); `unfused_nccl_us_per_step` times the same
steps as ZipGEMM + NCCL all-reduce, as context. The timed region
is K CUDA-graph replayed steps bracketed by barrier + synchronize; time = max
over ranks. Before the headline line, the config-4 Llama-70B layer at tp = N
is printed (one line per token count); at N = 1 the other BASELINE
configurations are printed first as well (config 1 round trip, config 3
Llama-8B projections against cuBLAS, config 5 decode attention against stock
flash-attn), unless --headline-only is given.

L2 policy: each rank rotates through enough distinct compressed weights that
the rotating set exceeds the 126 MB L2, so every step streams its weight from
HBM.

`value` is algorithmic bytes per second summed over the ranks: compressed W
bytes + X (2KN) + Y (2MN) of each rank. The roofline is the ZipGEMM kernel's
own (its launches alone, replayed in a graph); `dense_bf16_us` times cuBLAS on
uncompressed weights at the same shape, as context.
`e2e` repeats the step through the public API from pinned host memory (H2D of
X + ZipGEMM + D2H of Y of every step inside the timed region, steps pipelined
on three streams as a serving loop would run them). `cpu_baseline` times the CPU
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
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded W ~ N(0,0.02), X ~ N(0,1))", "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": desc + "; decoder = oracle port of the reference CPU decoder (its source "
                                          "needs nvCOMP headers, not buildable here)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": time.perf_counter() - t0}), flush=True)


def run_ncu_attention(args):
    """Profiling mode for decode attention: B=32, T=4096 (config 5), plain launches."""
    import math

    import torch

    import zipserv_asplos26_b200 as zs
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(5)
    B, T, Hq, Hkv, D = 32, 4096, 32, 8, 128

    def kv():
        scale = torch.exp(torch.empty(Hkv, D, device=dev).uniform_(math.log(0.1), math.log(4.0), generator=gen))
        return (torch.randn(B, T, Hkv, D, device=dev, generator=gen) * scale).to(torch.bfloat16)

    kc, vc = zs.compress_kv(kv()), zs.compress_kv(kv())
    q = torch.randn(B, Hq, D, device=dev, generator=gen).to(torch.bfloat16)
    seq = torch.full((B,), T, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    for _ in range(args.warmup + args.steps):
        zs.decode_attention(q, kc, vc, seq, Hkv, max_seqlen=T, out=out)
    torch.cuda.synchronize()
    print(json.dumps({"ncu_mode": True, "workload": "attention", "launches": args.warmup + args.steps}))


def run_ncu(args):
    """Profiling mode: plain launches over the same rotating weights and X."""
    if args.workload == "attention":
        return run_ncu_attention(args)
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


# ----------------------------------------------------------------------------
# Other BASELINE configurations (not the driver's headline line): one JSON line
# per measured case, same timing rules (warm-up, CUDA-graph replay, inputs that
# rotate through more than L2, CUDA events on the launching stream).
# ----------------------------------------------------------------------------
def _graph_time_us(torch, fns, stream, reps=3):
    with torch.cuda.stream(stream):
        for f in fns[:3]:
            f()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for f in fns:
                f()
        g.replay()
        stream.synchronize()
        best = float("inf")
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            b.synchronize()
            best = min(best, a.elapsed_time(b) * 1e3 / len(fns))
    return best


_LINES = []   # the per-case lines printed so far (summarised in the headline line)


def _emit(line):
    print(json.dumps(line), flush=True)
    _LINES.append(line)


def run_llama8b(args):
    """Config 3: Llama-3.1-8B projection shapes, N in {1..256}; W ~ N(0, sigma),
    sigma ~ U[0.01, 0.04] per matrix; compared with dense bf16 torch.matmul (cuBLAS)."""
    import torch

    import zipserv_asplos26_b200 as zs
    dev = torch.device("cuda", 0)
    peak, kind = peaks()
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}
    g = torch.Generator().manual_seed(7)
    stream = torch.cuda.Stream(device=dev)
    for name, (M, K) in shapes.items():
        sigma = 0.01 + 0.03 * float(torch.rand(1, generator=g))
        one = zs.compress((torch.randn(M, K, device=dev) * sigma).to(torch.bfloat16))
        nsets = max(2, -(-int(1.5 * L2_BYTES) // one.compressed_bytes()))
        comps, dense = [one], []
        for i in range(nsets):
            w = (torch.randn(M, K, device=dev) * sigma).to(torch.bfloat16)
            if i:
                comps.append(zs.compress(w))
            dense.append(w)
        if args.weight_offload:
            _weight_offload_lines(torch, zs, name, M, K, comps[0], dense[0], stream, peak, kind)
            del comps, dense
            continue
        for N in (1, 8, 16, 32, 64, 128, 256):
            x = torch.randn(N, K, device=dev).to(torch.bfloat16)
            y = torch.empty(N, M, dtype=torch.bfloat16, device=dev)
            L = 40
            tz = _graph_time_us(torch, [(lambda c=comps[i % nsets]: zs.zipgemm(c, x, out=y)) for i in range(L)], stream)
            td = _graph_time_us(torch, [(lambda w=dense[i % nsets]: torch.matmul(x, w.t(), out=y)) for i in range(L)],
                                stream)
            cb = comps[0].compressed_bytes()
            nbytes = cb + 2 * N * K + 2 * M * N
            gbps = nbytes / tz / 1e3
            _emit({"workload": "config3_llama8b", "proj": name, "M": M, "K": K, "N": N, "sigma": round(sigma, 4),
                              "zipgemm_us": round(tz, 2), "dense_bf16_us": round(td, 2), "speedup_vs_dense": round(td / tz, 3),
                              "compressed_GBps": round(gbps, 1), "hbm_frac": round(gbps / peak, 4),
                              "tflops": round(2 * M * N * K / tz / 1e6, 2), "ratio": round(2 * M * K / cb, 4),
                   "peak": f"{peak} GB/s ({kind})",
                   "split_k": "the SplitK argument is accepted; the kernel picks its K split per shape"})
        del comps, dense


def _weight_offload_lines(torch, zs, name, M, K, comp, dense, stream, peak, kind):
    """Weight offload (reference kernel_benchmark/bench_zipserv_gemm_sweep.cu:608-661,
    680-684): the weight lives in pinned host memory and every step copies it to
    the device before the GEMM. Compressed: the TCA-TBE arrays cross PCIe, then
    ZipGEMM; dense: the bf16 matrix crosses PCIe, then torch.matmul."""
    from zipserv_asplos26_b200.codec import Compressed
    fields = ("sign_mantissa", "compressed_full", "bitmap1", "bitmap2", "bitmap3", "tile_offsets_median",
              "tile_offsets_global")
    n_used = {"sign_mantissa": comp.total_hf, "compressed_full": comp.total_full}
    host = {f: getattr(comp, f)[:n_used.get(f, getattr(comp, f).numel())].cpu().pin_memory() for f in fields}
    devb = {f: torch.empty_like(getattr(comp, f)) for f in fields}
    dc = Compressed(devb["sign_mantissa"], devb["compressed_full"], devb["bitmap1"], devb["bitmap2"], devb["bitmap3"],
                    None, devb["tile_offsets_median"], devb["tile_offsets_global"], comp.rows, comp.cols,
                    comp.max_high_freq_count, comp.max_full_count, comp.start_exp, comp.total_hf, comp.total_full)
    wh = dense.cpu().pin_memory()
    wd = torch.empty_like(dense)
    h2d_comp = sum(t.numel() * t.element_size() for t in host.values())
    for N in (1, 16, 64, 128):
        x = torch.randn(N, K, device=dense.device).to(torch.bfloat16)
        y = torch.empty(N, M, dtype=torch.bfloat16, device=dense.device)

        def comp_step():
            for f in fields:
                devb[f][:host[f].numel()].copy_(host[f], non_blocking=True)
            zs.zipgemm(dc, x, out=y)

        def dense_step():
            wd.copy_(wh, non_blocking=True)
            torch.matmul(x, wd.t(), out=y)
        tz = _graph_time_us(torch, [comp_step] * 10, stream)
        td = _graph_time_us(torch, [dense_step] * 10, stream)
        print(json.dumps({"workload": "config3_llama8b_weight_offload", "proj": name, "M": M, "K": K, "N": N,
                          "compressed_step_us": round(tz, 2), "dense_step_us": round(td, 2),
                          "speedup_vs_dense": round(td / tz, 3), "h2d_bytes_compressed": h2d_comp,
                          "h2d_bytes_dense": 2 * M * K, "ratio": round(2 * M * K / h2d_comp, 4),
                          "mode": "per step: H2D of the weight from pinned host memory, then the GEMM; "
                                  "10 steps in one CUDA graph"}), flush=True)


def run_attention(args):
    """Config 5: compressed-KV decode attention, Hq=32, Hkv=8, D=128, one query
    token; K/V = N(0,1) x per-channel scale log-uniform in [0.1, 4], compressed per
    64-token page (head-major layout); tok/s = B / latency."""
    import math

    import torch

    import zipserv_asplos26_b200 as zs
    dev = torch.device("cuda", 0)
    peak, kind = peaks()
    Hq, Hkv, D = 32, 8, 128
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(5)

    def kv(B, T):
        scale = torch.exp(torch.empty(Hkv, D, device=dev).uniform_(math.log(0.1), math.log(4.0), generator=gen))
        return (torch.randn(B, T, Hkv, D, device=dev, generator=gen) * scale).to(torch.bfloat16)

    for B in (1, 8, 32):
        for T in (1024, 4096, 16384, 32768):
            k0, v0 = kv(B, T), kv(B, T)
            kc, vc = zs.compress_kv(k0), zs.compress_kv(v0)
            del k0, v0
            cb = kc.compressed_bytes() + vc.compressed_bytes()
            nsets = max(1, min(16, -(-int(1.5 * L2_BYTES) // cb)))
            sets = [(kc, vc)]
            for _ in range(nsets - 1):
                k1, v1 = kv(B, T), kv(B, T)
                sets.append((zs.compress_kv(k1), zs.compress_kv(v1)))
                del k1, v1
            q = torch.randn(B, Hq, D, device=dev, generator=gen).to(torch.bfloat16)
            seq = torch.full((B,), T, dtype=torch.int32, device=dev)
            out = torch.empty_like(q)
            L = 20
            t = _graph_time_us(torch, [(lambda s=sets[i % nsets]: zs.decode_attention(q, s[0], s[1], seq, Hkv,
                                                                                       max_seqlen=T, out=out))
                                       for i in range(L)], stream)
            nbytes = cb + 2 * 2 * B * Hq * D
            dense = 2 * 2 * B * T * Hkv * D
            # yardstick: stock flash-attn decode on the uncompressed cache (rotating
            # beyond L2 where it fits), as the reference's dense baseline runs it
            # (kernel_benchmark/bench_zipserv_decode_attention.py:610-649)
            fa_us = None
            try:
                from flash_attn import flash_attn_with_kvcache
                nd = max(1, min(8, -(-int(1.5 * L2_BYTES) // dense)))
                dsets = [(kv(B, T), kv(B, T)) for _ in range(nd)]
                q4 = q.view(B, 1, Hq, D)
                fa_us = _graph_time_us(torch, [(lambda s=dsets[i % nd]: flash_attn_with_kvcache(
                    q4, s[0], s[1], cache_seqlens=seq)) for i in range(L)], stream)
                del dsets
            except ImportError:
                pass
            _emit({"workload": "config5_decode_attention", "B": B, "T": T, "Hq": Hq, "Hkv": Hkv, "D": D,
                              "us": round(t, 2), "tok_per_s": round(B / (t * 1e-6), 1),
                              "dense_flash_attn_us": round(fa_us, 2) if fa_us else None,
                              "speedup_vs_dense_flash_attn": round(fa_us / t, 3) if fa_us else None,
                              "compressed_GBps": round(nbytes / t / 1e3, 1), "hbm_frac": round(nbytes / t / 1e3 / peak, 4),
                              "dense_equiv_GBps": round((dense + 4 * B * Hq * D) / t / 1e3, 1),
                              "kv_ratio": round(dense / cb, 4), "rotating_sets": nsets,
                   "peak": f"{peak} GB/s ({kind})"})
            del sets, kc, vc
            torch.cuda.empty_cache()


def run_paged_kv(args):
    """Paged compressed KV (config 5 shapes): decode attention over a paged
    cache with a dense tail page, against the head-major kernel on the same
    tokens, and the online append rate (one page per sequence and KV head)."""
    import math

    import torch

    import zipserv_asplos26_b200 as zs
    from zipserv_asplos26_b200.kvcache import PagedZipKVCache
    dev = torch.device("cuda", 0)
    peak, kind = peaks()
    Hq, Hkv, D = 32, 8, 128
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(9)

    def kv(B, T):
        scale = torch.exp(torch.empty(Hkv, D, device=dev).uniform_(math.log(0.1), math.log(4.0), generator=gen))
        return (torch.randn(B, T, Hkv, D, device=dev, generator=gen) * scale).to(torch.bfloat16)

    for B, T in ((32, 4096), (8, 16384), (1, 32768)):
        k0, v0 = kv(B, T + 33), kv(B, T + 33)   # T + 33 tokens: the last page is a dense tail
        blocks = (T + 64) // 64
        cache = PagedZipKVCache(num_blocks=B * blocks, max_batch=B, max_blocks_per_seq=blocks, num_kv_heads=Hkv,
                                k_window=PagedZipKVCache.window_from(k0[0]),
                                v_window=PagedZipKVCache.window_from(v0[0]), full_elems_per_page=2048, device=dev)
        for b in range(B):
            cache.prefill(b, k0[b], v0[b])
        q = torch.randn(B, Hq, D, device=dev, generator=gen).to(torch.bfloat16)
        out = torch.empty_like(q)
        t_paged = _graph_time_us(torch, [lambda: cache.attention(q, out=out)] * 20, stream)
        kc, vc = zs.compress_kv(k0), zs.compress_kv(v0)
        seq = torch.full((B,), T + 33, dtype=torch.int32, device=dev)
        t_head = _graph_time_us(torch, [lambda: zs.decode_attention(q, kc, vc, seq, Hkv, max_seqlen=T + 33,
                                                                     out=out)] * 20, stream)
        cb = int(cache.k.cursor[0].item() + 2 * cache.k.cursor[1].item() + cache.v.cursor[0].item()
                 + 2 * cache.v.cursor[1].item()) + 2 * B * blocks * Hkv * (3 * 1024 + 64)
        # append: one full page per sequence (B x Hkv pages of K and of V per launch)
        xk, xv = kv(B, 64), kv(B, 64)
        app = PagedZipKVCache(num_blocks=B * 8, max_batch=B, max_blocks_per_seq=8, num_kv_heads=Hkv,
                              k_window=cache.k.top, v_window=cache.v.top, device=dev)
        dst = torch.arange(B * Hkv, dtype=torch.int32, device=dev)
        from zipserv_asplos26_b200.kvcache import _fn
        import ctypes as C
        f = _fn("zs_kv_append_pages")

        def append_once():
            app.k.cursor[:2].zero_()
            app.v.cursor[:2].zero_()
            for pool, x in ((app.k, xk), (app.v, xv)):
                f(torch.cuda.current_stream().cuda_stream, C.byref(pool.st), x.data_ptr(), B, 1, Hkv, D,
                  dst.data_ptr(), None)
        t_app = _graph_time_us(torch, [append_once] * 20, stream)
        print(json.dumps({"workload": "paged_kv", "B": B, "T": T + 33, "Hq": Hq, "Hkv": Hkv, "D": D,
                          "paged_attention_us": round(t_paged, 2), "head_major_attention_us": round(t_head, 2),
                          "paged_tok_per_s": round(B / (t_paged * 1e-6), 1),
                          "paged_compressed_GBps": round(cb / t_paged / 1e3, 1),
                          "paged_hbm_frac": round(cb / t_paged / 1e3 / peak, 4),
                          "append_us_per_token_page": round(t_app, 2),
                          "append_input_GBps": round(2 * 2 * B * 64 * Hkv * D / t_app / 1e3, 1),
                          "peak": f"{peak} GB/s ({kind})"}), flush=True)
        del cache, app, kc, vc, k0, v0
        torch.cuda.empty_cache()


def run_roundtrip(args):
    """Config 1: host TCA-TBE round trip of a 4096x4096 bf16 N(0, 0.02) matrix
    through the library's own host encoder and GPU decoder, plus GPU encode and
    decode throughput on the same matrix."""
    import numpy as np
    import torch

    import zipserv_asplos26_b200 as zs
    from zipserv_asplos26_b200.codec import compress_host
    rng = np.random.default_rng(0)
    w32 = rng.standard_normal((M_, K_), dtype=np.float32) * 0.02
    w = torch.from_numpy(w32).to(torch.bfloat16)
    cores = os.cpu_count() or 1
    t0 = time.perf_counter()
    reps = 5
    for _ in range(reps):
        hc = compress_host(w)
    t_enc = (time.perf_counter() - t0) / reps
    dev = torch.device("cuda", 0)
    wd = w.to(dev)
    gc = zs.compress(wd)
    torch.cuda.synchronize()
    same = all(torch.equal(getattr(hc, f).cpu(), getattr(gc, f).cpu()[:getattr(hc, f).numel()])
               for f in ("bitmap1", "bitmap2", "bitmap3", "tile_offsets_median", "tile_offsets_global"))
    rt = zs.decompress(gc)
    exact = torch.equal(rt.view(torch.int16).cpu(), w.view(torch.int16))
    stream = torch.cuda.Stream(device=dev)
    # GPU encode (not graph-capturable end to end: it sizes outputs on the host), events around eager calls
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for _ in range(3):
        zs.compress(wd)
    torch.cuda.synchronize()
    ev[0].record()
    for _ in range(10):
        zs.compress(wd)
    ev[1].record()
    ev[1].synchronize()
    t_genc = ev[0].elapsed_time(ev[1]) / 10 * 1e3
    t_gdec = _graph_time_us(torch, [lambda: zs.decompress(gc)] * 20, stream)
    cb = gc.compressed_bytes()
    _emit({"workload": "config1_roundtrip", "M": M_, "K": K_, "ratio": round(2 * M_ * K_ / cb, 4),
                      "compressed_bytes": cb, "host_encode_ms": round(t_enc * 1e3, 2), "host_cores": cores,
                      "gpu_encode_us": round(t_genc, 1), "gpu_decode_us": round(t_gdec, 2),
                      "gpu_decode_GBps": round((cb + 2 * M_ * K_) / t_gdec / 1e3, 1),
                      "host_gpu_bytes_identical": bool(same), "round_trip_bit_exact": bool(exact)})


def tp70b_lines(world, rank, dev, reps=20):
    """Config 4: one Llama-3.1-70B decoder layer's four weight GEMMs,
    tensor-parallel over the ranks (QKV / gate_up column-parallel, O / down
    row-parallel with the all-reduce fused into the ZipGEMM), captured in one
    CUDA graph per N; per-layer
    device time = max over ranks. Also times GPU compression of this rank's four
    shards. Returns one dict per N (printed by rank 0)."""
    import torch
    import torch.distributed as dist

    import zipserv_asplos26_b200 as zs
    from zipserv_asplos26_b200.tp import LLAMA70B_SHAPES, TPLayerGemms
    layer = TPLayerGemms(LLAMA70B_SHAPES, seed=0, device=dev, fused=world > 1)
    comp_ms, in_bytes = 0.0, 0
    for lin in layer.layers.values():
        w = (torch.randn(lin.out_features, lin.in_features, device=dev) * 0.02).to(torch.bfloat16)
        zs.compress(w)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        zs.compress(w)
        e1.record()
        e1.synchronize()
        comp_ms += e0.elapsed_time(e1)
        in_bytes += 2 * w.numel()
        del w
    cb = sum(l.weight.compressed_bytes() for l in layer.layers.values())
    stream = torch.cuda.Stream(device=dev)
    out = []
    for N in (1, 16, 64):
        xs = {n: torch.randn(*shp, device=dev).to(torch.bfloat16) for n, shp in layer.input_shapes(N).items()}
        ys = {n: torch.empty(N, lin.out_features, dtype=torch.bfloat16, device=dev) for n, lin in layer.layers.items()}
        with torch.cuda.stream(stream):
            for _ in range(3):
                for n, lin in layer.layers.items():
                    lin(xs[n], out=ys[n])
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(reps):
                    for n, lin in layer.layers.items():
                        lin(xs[n], out=ys[n])
            g.replay()
            stream.synchronize()
            if world > 1:
                dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            g.replay()
            b.record(stream)
            b.synchronize()
        t = torch.tensor([a.elapsed_time(b) * 1e3 / reps], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        out.append({"workload": "config4_tp70b_layer", "tp": world, "N": N, "layer_us": round(t.item(), 2),
                    "per_rank_compressed_MB": round(cb / 1e6, 2), "per_rank_GBps": round(cb / t.item() / 1e3, 1),
                    "hbm_frac": round(cb / t.item() / 1e3 / peaks()[0], 4),
                    "compress_layer_ms": round(comp_ms, 2),
                    "compress_GBps_bf16_in": round(in_bytes / comp_ms / 1e6, 1),
                    "note": "4 projections per layer" + (
                        ", O and down with the all-reduce fused into the ZipGEMM (NVLink peer stores)"
                        if world > 1 else "") + f", one CUDA graph of {reps} layers, max over ranks"})
        del g
    return out


def compress80_line(world, rank, dev, layers=80):
    """Whole-model GPU compression (config 4): all `layers` Llama-3.1-70B layers
    of this rank's shards, each layer's four matrices generated on the device
    (seeded per layer, outside the timed region) and compressed through the
    public API; the compressions' device times are summed (max over ranks).
    Reference: kernel_benchmark/bench_llama31_70b_compress.cu:923 ProcessTensor."""
    import torch
    import torch.distributed as dist

    import zipserv_asplos26_b200 as zs
    from zipserv_asplos26_b200.tp import LLAMA70B_SHAPES
    total_ms, in_bytes, out_bytes = 0.0, 0, 0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for layer in range(layers):
        for i, (name, (M, K)) in enumerate(LLAMA70B_SHAPES.items()):
            col = name in ("qkv", "gate_up")
            m, k = (M // world, K) if col else (M, K // world)
            g = torch.Generator(device=dev).manual_seed(layer * 64 + i * 8 + rank)
            w = (torch.randn(m, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            torch.cuda.synchronize()
            e0.record()
            c = zs.compress(w)
            e1.record()
            e1.synchronize()
            total_ms += e0.elapsed_time(e1)
            in_bytes += 2 * w.numel()
            out_bytes += c.compressed_bytes()
            del w, c
    t = torch.tensor([total_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    cpu = None
    if rank == 0:
        # CPU baseline (bounded sample): the library's host encoder (OpenMP, all
        # cores; the reference's host encoders produce the same bytes) on one O
        # shard, extrapolated by bf16 bytes to the rank's 80 layers
        from zipserv_asplos26_b200.codec import compress_host
        ko = LLAMA70B_SHAPES["o"][1] // world
        w = (torch.randn(LLAMA70B_SHAPES["o"][0], ko, generator=torch.Generator().manual_seed(3)) * 0.02).to(
            torch.bfloat16)
        compress_host(w)
        t0 = time.perf_counter()
        compress_host(w)
        dt = time.perf_counter() - t0
        cpu = {"seconds_extrapolated": round(dt * in_bytes / (2 * w.numel()), 2), "cores": os.cpu_count() or 1,
               "kind": "port", "sample": f"host encode of one {LLAMA70B_SHAPES['o'][0]}x{ko} O shard "
                                         f"({round(dt * 1e3, 1)} ms), scaled by bytes to {layers} layers"}
    return {"workload": "config4_whole_model_compression", "tp": world, "layers": layers,
            "cpu_baseline": cpu,
            "seconds": round(t.item() / 1e3, 4), "per_rank_bf16_GB": round(in_bytes / 1e9, 2),
            "per_rank_compressed_GB": round(out_bytes / 1e9, 2), "ratio": round(in_bytes / out_bytes, 4),
            "GBps_bf16_in": round(in_bytes / (t.item() / 1e3) / 1e9, 1),
            "note": "each matrix compressed by zs.compress (window analysis + GPU encoder + size read-back); "
                    "device time summed over the 320 matrices of the rank, max over ranks"}


def run_tp70b(args):
    """--workload tp70b: the config-4 layer lines (under torchrun for tp > 1) and
    the whole-model compression line."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    for line in tp70b_lines(world, rank, dev) + [compress80_line(world, rank, dev)]:
        if rank == 0:
            print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if world > 1:   # leave without tearing down the communicator (see main)
        dist.barrier()
        sys.stdout.flush()
        os._exit(0)


def _summarise(lines, layer_lines):
    """Compact summary of the per-case lines printed before the headline, kept
    in the headline line itself (the line a log reader parses)."""
    out = {}
    for d in lines:
        w = d.get("workload")
        if w == "config1_roundtrip":
            out["config1_roundtrip"] = {k: d[k] for k in ("ratio", "host_encode_ms", "host_cores", "gpu_encode_us",
                                                          "gpu_decode_us", "round_trip_bit_exact",
                                                          "host_gpu_bytes_identical")}
        elif w == "config3_llama8b":
            out.setdefault("config3_llama8b_us_zipgemm_vs_cublas", {})[f"{d['proj']} N={d['N']}"] = [
                d["zipgemm_us"], d["dense_bf16_us"]]
        elif w == "config5_decode_attention":
            out.setdefault("config5_attention_us_ours_vs_flash_attn_dense", {})[f"B={d['B']} T={d['T']}"] = [
                d["us"], d["dense_flash_attn_us"]]
    for d in layer_lines:
        out.setdefault("config4_tp70b_layer_us", {})[f"tp={d['tp']} N={d['N']}"] = d["layer_us"]
    return out


def dense_bf16_us(torch, dev, steps=40):
    """torch.matmul (cuBLAS) at the config-2 shape on uncompressed bf16 weights
    that rotate beyond L2: context for the ZipGEMM time, not a product path."""
    sets = [(torch.randn(M_, K_, device=dev) * 0.02).to(torch.bfloat16) for _ in range(6)]
    x = torch.randn(N_, K_, device=dev).to(torch.bfloat16)
    y = torch.empty(N_, M_, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.Stream(device=dev)
    return _graph_time_us(torch, [(lambda w=sets[i % 6]: torch.matmul(x, w.t(), out=y)) for i in range(steps)], stream)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="N = 1: skip the config 1 / 3 / 5 lines printed before the headline")
    ap.add_argument("--ncu", action="store_true", help="plain launches for ncu, no timing")
    ap.add_argument("--weight-offload", action="store_true",
                    help="with --workload llama8b: copy the weight H2D inside every timed step")
    ap.add_argument("--workload", default="config2",
                    choices=["config2", "llama8b", "attention", "roundtrip", "tp70b", "paged_kv"],
                    help="config2 = the headline line; the others print one JSON line per case")
    args = ap.parse_args()
    if args.workload != "config2" and args.impl == "ours" and not args.ncu:
        return {"llama8b": run_llama8b, "attention": run_attention, "roundtrip": run_roundtrip,
                "tp70b": run_tp70b, "paged_kv": run_paged_kv}[args.workload](args)
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
    if world == 1 and not args.headline_only:
        # the other BASELINE configurations, one JSON line per case, before the headline
        for run in (run_roundtrip, run_llama8b, run_attention):
            run(args)
            torch.cuda.synchronize()
            torch.cuda.empty_cache()
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    W = max(3, args.warmup)
    K = args.steps
    if K_ % world or (K_ // world) % 64:
        raise SystemExit(f"K={K_} does not split into multiples of 64 over {world} ranks")
    Kr = K_ // world   # row-parallel: this rank's K slice of W and X

    # One step = one config-2 GEMM Y = W X^T. With N ranks it runs row-parallel,
    # as a tensor-parallel O / down projection would: rank r holds columns
    # [r K/N, (r+1) K/N) of W (its own compressed shard) and of X, and the
    # partial Ys are summed by an NCCL all-reduce inside the timed graph.
    def make_shards(count, first=0):
        out = []
        for i in range(first, first + count):
            g = torch.Generator(device=dev).manual_seed(1000 * rank + i)
            w = (torch.randn(M_, Kr, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            out.append(zs.compress(w))
            del w
        return out

    comps = make_shards(1)
    cb = comps[0].compressed_bytes()
    n_sets = max(2, -(-int(1.5 * L2_BYTES) // cb))
    comps += make_shards(n_sets - 1, first=1)
    x_full = torch.randn(N_, K_, generator=torch.Generator(device=dev).manual_seed(1), device=dev).to(torch.bfloat16)
    x = x_full[:, rank * Kr:(rank + 1) * Kr].contiguous()
    ys = [torch.empty(N_, M_, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    nbytes = cb + 2 * Kr * N_ + 2 * M_ * N_          # this rank's algorithmic bytes per step
    tb = torch.tensor([float(nbytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tb)
    job_bytes = tb.item()                            # all ranks' algorithmic bytes per step

    if world > 1:
        from zipserv_asplos26_b200.tp import AllReduceBuffers, zipgemm_allreduce
        bufs = AllReduceBuffers(M_, N_, device=dev)

    def step(i, xin, yout):
        if world > 1:   # the all-reduce of Y fused into the ZipGEMM (NVLink peer stores)
            zipgemm_allreduce(comps[i % n_sets], xin, bufs, out=yout)
        else:
            zs.zipgemm(comps[i % n_sets], xin, out=yout)

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for i in range(W):
            step(i, x, ys[i % 2])
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(K):
                step(i, x, ys[i % 2])
        graph.replay()
        stream.synchronize()

        # kernel-only time of the dominant kernel (the ZipGEMM launches alone)
        kgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kgraph, stream=stream):
            for i in range(K):
                zs.zipgemm(comps[i % n_sets], x, out=ys[i % 2])
        kgraph.replay()
        stream.synchronize()
        ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ka.record(stream)
        kgraph.replay()
        kb.record(stream)
        kb.synchronize()
        gemm_ms = ka.elapsed_time(kb) / K

        # context for N > 1: the same steps unfused (ZipGEMM, then an NCCL all-reduce of Y)
        nccl_ms = 0.0
        if world > 1:
            ngraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(ngraph, stream=stream):
                for i in range(K):
                    zs.zipgemm(comps[i % n_sets], x, out=ys[i % 2])
                    dist.all_reduce(ys[i % 2], op=dist.ReduceOp.SUM)
            ngraph.replay()
            stream.synchronize()
            dist.barrier()
            na, nb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            na.record(stream)
            ngraph.replay()
            nb.record(stream)
            nb.synchronize()
            nccl_ms = na.elapsed_time(nb) / K
            del ngraph

        # Load the GPU for about a second while the clock sampler runs. Every rank
        # must replay the graph the same number of times (its collectives pair up
        # across ranks), so the count comes from one timed replay, agreed by MAX.
        t1 = time.perf_counter()
        graph.replay()
        stream.synchronize()
        nsoak = torch.tensor([max(1, int(1.0 / max(time.perf_counter() - t1, 1e-4)))], device=dev)
        if world > 1:
            dist.all_reduce(nsoak, op=dist.ReduceOp.MAX)
        sampler = ClockSampler(local)
        sampler.start()
        for _ in range(int(nsoak.item())):
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

        # e2e through the public API from pinned host memory. Every step copies its
        # X in (H2D), runs the GEMM (and the all-reduce) and copies its Y out (D2H);
        # steps are pipelined as a serving loop would run them: copies in, GEMMs and
        # copies out on three streams with NB device buffers each, so the copies of
        # neighbouring steps overlap the GEMMs. Timed from the first H2D to the last D2H.
        NB = 3
        xh = x.cpu().pin_memory()
        yh = [torch.empty(N_, M_, dtype=torch.bfloat16).pin_memory() for _ in range(NB)]
        xd = [torch.empty_like(x) for _ in range(NB)]
        yd = [torch.empty(N_, M_, dtype=torch.bfloat16, device=dev) for _ in range(NB)]
        s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

        def e2e_steps(n):
            ev_in = [torch.cuda.Event() for _ in range(n)]
            ev_c = [torch.cuda.Event() for _ in range(n)]
            ev_out = [torch.cuda.Event() for _ in range(n)]
            for i in range(n):
                b = i % NB
                with torch.cuda.stream(s_in):
                    if i >= NB:
                        s_in.wait_event(ev_c[i - NB])         # GEMM i-NB has read xd[b]
                    xd[b].copy_(xh, non_blocking=True)
                    ev_in[i].record(s_in)
                with torch.cuda.stream(stream):
                    stream.wait_event(ev_in[i])
                    if i >= NB:
                        stream.wait_event(ev_out[i - NB])     # D2H i-NB has read yd[b]
                    step(i, xd[b], yd[b])
                    ev_c[i].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_c[i])
                    yh[b].copy_(yd[b], non_blocking=True)
                    ev_out[i].record(s_out)

        e2e_steps(W)
        torch.cuda.synchronize()
        # the K pipelined steps are captured once (fork to the copy streams, join
        # back) and replayed, so the host's per-call overhead does not time the copies
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            e2e_steps(K)
            stream.wait_stream(s_in)
            stream.wait_stream(s_out)
        g2.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a, bb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        g2.replay()
        bb.record(stream)
        bb.synchronize()
        e2e_ms = a.elapsed_time(bb)
    t = torch.tensor([ms_total, e2e_ms, gemm_ms, nccl_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, e2e_ms, gemm_ms, nccl_ms = t.tolist()
    ms_step = ms_total / K
    peak, peak_kind = peaks()
    achieved = nbytes / (gemm_ms / 1e3) / 1e9
    traffic = None
    if os.path.exists(PROFILE_TRAFFIC):
        with open(PROFILE_TRAFFIC) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")
    dense_us = dense_bf16_us(torch, dev) if world == 1 else None
    # the config-4 layer at tp = N (printed before the headline, which stays last)
    layer_lines = tp70b_lines(world, rank, dev)
    if rank == 0:
        for line in layer_lines:
            print(json.dumps(line), flush=True)
        par = ("single GPU" if world == 1 else
               f"row-parallel tp{world}: W and X split by K over the ranks (own compressed shard per rank), "
               "the all-reduce (bf16 partials summed in fp32) of Y fused into the ZipGEMM in every step")
        line = {
            "metric": METRIC, "value": job_bytes * K / (ms_total / 1e3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms_step, "us_per_step": ms_step * 1e3,
            "zipgemm_us": gemm_ms * 1e3,
            "tflops": 2.0 * M_ * N_ * K_ / (ms_step / 1e3) / 1e12, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded W ~ N(0,0.02) per rank and set, X ~ N(0,1))",
            "config": dict(CONFIG, parallelism=par, rotating_sets=n_sets, compressed_bytes_per_rank=cb,
                           ratio=round(2 * M_ * Kr / cb, 4)),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic if world == 1 else None,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "algorithmic_bytes_per_launch": nbytes,
                         "kernel": "zs::zipgemm_kernel, CUDA-graph replay of the GEMMs alone, max over ranks"},
            "e2e": {"value": job_bytes * K / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": 2 * N_ * Kr, "d2h_bytes_per_step": 2 * N_ * M_,
                    "ms_per_step": e2e_ms / K,
                    "mode": "per step: H2D of X from pinned host, zipgemm (+ all-reduce), D2H of Y to pinned host; "
                            f"steps pipelined on three streams with {NB} device buffers each, the K steps' API "
                            "calls captured in one CUDA graph and replayed"},
            "dense_bf16_us": dense_us,
            "speedup_vs_dense_bf16": (dense_us / (gemm_ms * 1e3)) if dense_us else None,
            "unfused_nccl_us_per_step": (nccl_ms * 1e3) if world > 1 else None,
            "gpu_launches": K,
            "clocks": clocks,
        }
        if _LINES or layer_lines:
            line["other_configs"] = _summarise(_LINES, layer_lines)
        if world == 1 and not args.no_cpu_baseline:
            v, per, cores, desc = cpu_step_sample()
            line["cpu_baseline"] = {"value": v / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                    "sample": desc, "ms_per_step": per * 1e3}
        print(json.dumps(line), flush=True)
    # Graphs that captured NCCL collectives must be released before the process
    # group goes away (destroying it under live graphs can block forever), and
    # the ranks leave together without tearing the communicator down.
    del graph, kgraph, g2
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        sys.stdout.flush()
        os._exit(0)


if __name__ == "__main__":
    main()
