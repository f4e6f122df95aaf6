"""Benchmark of the NVFP4 x q8_1 hot path on B200 (one JSON line on rank 0).

Workload (the config the GEMV GB/s metric is quoted
on): the dense batched-decode FFN -- gate/up 14336x4096 and down 4096x14336
NVFP4 weights, activations N(0,1) quantized to q8_1 -- at T=1 token.  A step is
one FFN pass: quantize_q8_1(x) -> gate/up matvec with the SwiGLU epilogue ->
quantize_q8_1(GLU) -> down matvec, through fr_ffn_nvfp4.  Steps rotate over
4 weight sets (396 MB > 3x the 126 MB L2), so every step streams its weights
from HBM.  T=8 and T=64 are reported as extra fields of the same line.

`value` = algorithmic bytes (3 weight matrices + x + out) per step / device
time per step, summed over ranks.  `e2e` is the same metric with the pinned
host->device copy of x and the device->host copy of out inside every step.

--impl reference times the CPU restatement of the same op (oracle/, the
reference's ggml CPU backend being unavailable here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flashrt-llama.cpp_b200"))

METRIC = "NVFP4 GEMV GB/s vs HBM peak; MoE decode tok/s at batch 1/64, 1–8 B200"
N_EMBD, N_FF = 4096, 14336
N_SETS = 4
HBM_FALLBACK = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum per launch of the gate/up SwiGLU
# matvec (T=1), from the ncu capture summarised in profiles/; None until taken.
TRAFFIC_GATEUP = None


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return HBM_FALLBACK, "fallback"


def ffn_bytes(T: int) -> int:
    w = 3 * N_FF * (N_EMBD // 64 * 36)
    return w + 2 * T * N_EMBD * 4


def gateup_bytes(T: int) -> int:
    return 2 * N_FF * (N_EMBD // 64 * 36) + T * N_EMBD * 4 + T * N_FF * 4


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.th = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.th = threading.Thread(target=self._read, daemon=True)
            self.th.start()
        except Exception:  # noqa: BLE001
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        self.th.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------- reference arm

def cpu_reference_line(args, T: int = 1, budget_s: float = 12.0):
    """Time the CPU restatement of the FFN matvecs (oracle/, fp32 accumulation
    with int32 sub-block sums, all host threads) on a bounded sample."""
    import numpy as np
    import frb200
    from oracle import oracle as O

    ncores = os.cpu_count() or 1
    # sample: one FFN layer's three matrices, rows subsampled to bound the time
    rows = 2048
    wg = frb200.synth_nvfp4(0x5EED0000 + 1, rows, N_EMBD)
    wd = frb200.synth_nvfp4(0x5EED0000 + 3, rows, N_FF)
    x = frb200.synth_normal(0x5EED0000 + 10, T * N_EMBD).reshape(T, N_EMBD)
    g = frb200.synth_normal(0x5EED0000 + 11, T * N_FF).reshape(T, N_FF)
    qx = O.quantize_q8_1(x)
    qg = O.quantize_q8_1(g)
    O.gemv_q8_1_f32(wg, qx, rows, N_EMBD, nthreads=ncores)          # warm-up
    per_pass = (wg.nbytes + wd.nbytes)
    t0 = time.perf_counter()
    n = 0
    while True:
        O.gemv_q8_1_f32(wg, qx, rows, N_EMBD, nthreads=ncores)
        O.gemv_q8_1_f32(wd, qg, rows, N_FF, nthreads=ncores)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    gbs = n * per_pass / dt / 1e9
    sample = (f"{n} passes over 2048 rows of the gate (K=4096) and down (K=14336) matrices "
              f"({per_pass / 1e6:.1f} MB per pass, T={T}) in {dt:.1f} s")
    return gbs, ncores, sample


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    gbs, cores, sample = cpu_reference_line(args)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8xe2m1 (int32 sub-block sums, fp32 scale)",
        "data": "synthetic (seeded splitmix64 / Box-Muller; BASELINE configs)",
        "config": {"workload": "dense FFN matvecs 14336x4096 / 4096x14336 NVFP4 x q8_1, T=1 (configs[1])",
                   "global_batch": 1, "seq_len": 1, "parallelism": "cpu"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "llama.cpp's ggml CPU backend is not in the image; the oracle's C restatement runs instead",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our arm

def run_ours(args):
    import numpy as np
    import torch
    import frb200

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
    frb200.lib()

    hbm, peak_kind = _peaks()
    rb_e, rb_f = N_EMBD // 64 * 36, N_FF // 64 * 36
    sets = []
    for s in range(N_SETS):
        base = 0x5EED0000 + 100 * s + 1000 * rank
        wg = torch.from_numpy(frb200.synth_nvfp4(base + 1, N_FF, N_EMBD)).to(dev)
        wu = torch.from_numpy(frb200.synth_nvfp4(base + 2, N_FF, N_EMBD)).to(dev)
        wd = torch.from_numpy(frb200.synth_nvfp4(base + 3, N_EMBD, N_FF)).to(dev)
        sets.append((wg, wu, wd))
    stream = torch.cuda.Stream(dev)
    Tmax = 64
    x_all = torch.from_numpy(frb200.synth_normal(0x5EED0000 + 10, Tmax * N_EMBD).reshape(Tmax, N_EMBD)).to(dev)
    outs = [torch.empty((Tmax, N_EMBD), dtype=torch.float32, device=dev) for _ in range(N_SETS)]

    def step(i, T, strm):
        wg, wu, wd = sets[i % N_SETS]
        frb200.ffn(x_all[:T], wg, wu, wd, N_EMBD, N_FF, out=outs[i % N_SETS][:T], stream=strm)

    def graphs_for(T):
        gs = []
        with torch.cuda.stream(stream):
            for i in range(N_SETS):       # eager warm-up sizes the workspaces
                step(i, T, stream)
        stream.synchronize()
        for i in range(N_SETS):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                step(i, T, stream)
            gs.append(g)
        return gs

    def barrier():
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def time_steps(gs, K, W):
        with torch.cuda.stream(stream):
            for i in range(W):
                gs[i % N_SETS].replay()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(K):
                gs[i % N_SETS].replay()
            e1.record(stream)
        e1.synchronize()
        barrier()
        ms = e0.elapsed_time(e1)
        if pg is not None:
            t = torch.tensor([ms], device=dev)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        return ms / K

    launches0 = frb200.lib().fr_kernel_launches()
    g1 = graphs_for(1)
    launches_per_step = (frb200.lib().fr_kernel_launches() - launches0) // (2 * N_SETS)

    # clocks: sample over a load window that contains the timed region
    sampler = ClockSampler(local)
    sampler.start()
    t_end = time.time() + 1.5
    with torch.cuda.stream(stream):
        i = 0
        while time.time() < t_end:
            for _ in range(200):
                g1[i % N_SETS].replay()
                i += 1
            stream.synchronize()
    ms1 = time_steps(g1, args.steps, max(args.warmup, 3))
    clocks = sampler.stop()

    # extra batch sizes on the same path
    extra = {}
    for T in (8, 64):
        gT = graphs_for(T)
        msT = time_steps(gT, max(10, args.steps // 8), max(args.warmup, 3))
        extra[f"ffn_T{T}_gbs"] = round(world * ffn_bytes(T) / (msT * 1e-3) / 1e9, 1)
        extra[f"ffn_T{T}_ms_per_step"] = round(msT, 5)
        del gT

    # dominant kernel: gate/up SwiGLU matvec timed alone (events on its stream)
    q8x = frb200.quantize_q8_1(x_all[:1], stream=stream)
    glu = torch.empty((1, N_FF), dtype=torch.float32, device=dev)
    kgs = []
    for i in range(N_SETS):
        wg, wu, _ = sets[i]
        frb200.gemv_swiglu(wg, wu, q8x, N_FF, N_EMBD, 1, out=glu, stream=stream)
    stream.synchronize()
    for i in range(N_SETS):
        wg, wu, _ = sets[i]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            frb200.gemv_swiglu(wg, wu, q8x, N_FF, N_EMBD, 1, out=glu, stream=stream)
        kgs.append(g)
    k_ms = time_steps(kgs, max(args.steps, 20), 5)
    k_gbs = gateup_bytes(1) / (k_ms * 1e-3) / 1e9

    # e2e through the public C entry point: pinned H2D of x, the FFN, D2H of out
    x_host = torch.from_numpy(frb200.synth_normal(0x5EED0000 + 10, N_EMBD).reshape(1, N_EMBD)).pin_memory()
    o_host = torch.empty((1, N_EMBD), dtype=torch.float32).pin_memory()
    x_dev = torch.empty((1, N_EMBD), dtype=torch.float32, device=dev)
    egs = []
    for i in range(N_SETS):
        with torch.cuda.stream(stream):
            x_dev.copy_(x_host, non_blocking=True)
            wg, wu, wd = sets[i]
            frb200.ffn(x_dev, wg, wu, wd, N_EMBD, N_FF, out=outs[i][:1], stream=stream)
            o_host.copy_(outs[i][:1], non_blocking=True)
    stream.synchronize()
    for i in range(N_SETS):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            x_dev.copy_(x_host, non_blocking=True)
            wg, wu, wd = sets[i]
            frb200.ffn(x_dev, wg, wu, wd, N_EMBD, N_FF, out=outs[i][:1], stream=stream)
            o_host.copy_(outs[i][:1], non_blocking=True)
        egs.append(g)
    e_ms = time_steps(egs, args.steps, max(args.warmup, 3))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, cores, sample = cpu_reference_line(args, budget_s=10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}

    value = world * ffn_bytes(1) / (ms1 * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms1, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8xe2m1 (q8_1 x NVFP4, int32 sub-block sums, fp32 scale)",
        "data": "synthetic (seeded splitmix64 / Box-Muller; BASELINE configs)",
        "config": {"workload": "dense FFN gate/up 14336x4096 + down 4096x14336 NVFP4 x q8_1, T=1 (configs[1])",
                   "global_batch": world, "seq_len": 1,
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                   "l2": f"rotating {N_SETS} weight sets ({N_SETS * ffn_bytes(0) / 1e6:.0f} MB > L2)",
                   "graph": "one CUDA graph per step, PDL edges between kernels"},
        "clocks": clocks,
        "e2e": {"value": round(world * ffn_bytes(1) / (e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": N_EMBD * 4, "d2h_bytes_per_step": N_EMBD * 4,
                "ms_per_step": round(e_ms, 5)},
        "gpu_launches": int(launches_per_step * args.steps),
        "roofline": {"bound": "hbm", "kernel": "k_gemv<32,1,SWIGLU> (gate/up, T=1)", "achieved": round(k_gbs, 1),
                     "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": round(k_gbs / hbm, 4),
                     "traffic": TRAFFIC_GATEUP, "algorithmic_bytes": gateup_bytes(1),
                     "ms_per_launch": round(k_ms, 5)},
        "cpu_baseline": cpu,
    }
    line.update(extra)
    for g in g1 + kgs + egs:
        del g
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
