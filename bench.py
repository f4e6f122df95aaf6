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
# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the gate/up
# SwiGLU FP4 tensor-core matvec on tile-major weights at T=1 (k_fp4t<16,1,1>):
# 66,132,992 + 326,912 bytes, as `ncu --metrics dram__bytes_read.sum,
# dram__bytes_write.sum,gpu__time_duration.sum --clock-control none -k
# regex:k_fp4t -s 8 -c 2 python bench.py --profile-case --layout tiled
# --tokens 1 --steps 8` reports it (step 5 of 8: the four weight sets rotate,
# so its weights come from HBM)
TRAFFIC_GATEUP = 66459904


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

def _host_nvfp4(seed: int, rows: int, K: int):
    """NVFP4 blocks with BASELINE's distribution generated on the host without
    the product library (numpy RNG; scales e4m3(|N(0,1)| * 0.05), RNE through
    torch's float8_e4m3fn): E2M1 codes uniform over all 16 values."""
    import numpy as np
    import torch
    rng = np.random.default_rng(seed)
    nb = rows * (K // 64)
    blk = np.empty((nb, 36), np.uint8)
    blk[:, 4:] = rng.integers(0, 256, size=(nb, 32), dtype=np.uint8)
    sc = np.abs(rng.standard_normal((nb, 4))) * 0.05
    blk[:, :4] = torch.from_numpy(sc.astype(np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    return blk.reshape(rows, K // 64 * 36)


def cpu_reference_line(args, T: int = 1, budget_s: float = 12.0):
    """Time the CPU restatement of the FFN matvecs (oracle/, fp32 accumulation
    with int32 sub-block sums, all host threads) on a bounded sample.  Its
    inputs are generated on the host (numpy), so this leg loads nothing of the
    product."""
    import numpy as np
    from oracle import oracle as O

    ncores = os.cpu_count() or 1
    # sample: one FFN layer's three matrices, rows subsampled to bound the time
    rows = 2048
    rng = np.random.default_rng(0x5EED0000 + 10)
    wg = _host_nvfp4(0x5EED0000 + 1, rows, N_EMBD)
    wd = _host_nvfp4(0x5EED0000 + 3, rows, N_FF)
    x = rng.standard_normal((T, N_EMBD)).astype(np.float32)
    g = rng.standard_normal((T, N_FF)).astype(np.float32)
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

def _moe_sets(frb200, torch, dev, rank, world, n_sets):
    """Config 3 experts (E=128, hidden 2048, FFN 768): this rank's E/world."""
    E, ne, nf = 128, 2048, 768
    Ep = E // world
    sets = []
    for s in range(n_sets):
        base = 0x5EED2000 + 100 * s
        wr = torch.from_numpy(frb200.synth_normal(base, E * ne, 0.0, 0.02).reshape(E, ne)).to(dev)
        # full-model expert tensors are generated per expert id, so each rank
        # holds exactly the rows of its experts
        wg = torch.from_numpy(frb200.synth_nvfp4(base + 1, E * nf, ne)[rank * Ep * nf:(rank + 1) * Ep * nf]).to(dev)
        wu = torch.from_numpy(frb200.synth_nvfp4(base + 2, E * nf, ne)[rank * Ep * nf:(rank + 1) * Ep * nf]).to(dev)
        wd = torch.from_numpy(frb200.synth_nvfp4(base + 3, E * ne, nf)[rank * Ep * ne:(rank + 1) * Ep * ne]).to(dev)
        sets.append((wr, wg, wu, wd))
    return sets


GEMV0_N = GEMV0_K = 4096
GEMV0_COPIES = 32


def gemv0_bytes() -> int:
    return GEMV0_N * (GEMV0_K // 64 * 36) + GEMV0_K * 4 + GEMV0_N * 4


def _gemv_config0(frb200, torch, dev, stream, time_fn, graphs_for, hbm, args):
    """y = W . q8_1(x), W 4096x4096 NVFP4, x 1x4096 f32 -- through
    fr_mul_mat_nvfp4 on ggml's layout, and through fr_gemv_tiled on the
    tile-major copy (same bytes).  Each timed launch reads a different weight
    copy (32 copies, 302 MB > 2x L2), all captured in one CUDA graph."""
    ws = [torch.from_numpy(frb200.synth_nvfp4(0x5EED0100 + c, GEMV0_N, GEMV0_K)).to(dev) for c in range(GEMV0_COPIES)]
    wts = [frb200.tile_nvfp4(w, GEMV0_N, GEMV0_K) for w in ws]
    x = torch.from_numpy(frb200.synth_normal(0x5EED0110, GEMV0_K).reshape(1, GEMV0_K)).to(dev)
    y = torch.empty((1, GEMV0_N), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    res = {}
    for name, call in (("ggml layout, fr_mul_mat_nvfp4",
                        lambda i: frb200.mul_mat(ws[i], x, GEMV0_N, GEMV0_K, out=y, stream=stream)),
                       ("tile-major layout, fr_gemv_tiled",
                        lambda i: frb200.gemv_tiled(wts[i], GEMV0_N, GEMV0_K, x=x, out=y, stream=stream))):
        with torch.cuda.stream(stream):
            for i in range(GEMV0_COPIES):
                call(i)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(GEMV0_COPIES):
                call(i)
        ms = time_fn(lambda i: g.replay(), max(10, args.steps // 4), 3) / GEMV0_COPIES
        del g
        res[name] = ms
    best = min(res, key=res.get)
    us = res[best] * 1e3
    gbs = gemv0_bytes() / (us * 1e-6) / 1e9
    out = {"gemv_4096_us": round(us, 3), "gemv_4096_gbs": round(gbs, 1), "gemv_4096_frac_hbm": round(gbs / hbm, 4),
           "gemv_4096_path": best, "gemv_4096_target_us_at_0.8": round(gemv0_bytes() / (0.8 * hbm * 1e9) * 1e6, 3)}
    for name, ms in res.items():
        out[f"gemv_4096_us[{name}]"] = round(ms * 1e3, 3)
    del ws, wts
    return out


FP4_DENSE_NOMINAL_TFLOPS = 9000.0


def _prefill_config3(frb200, torch, dev, stream, time_fn, graphs_for, hbm, args):
    """a 512-token ubatch (and 4 x 512 = 2048 rows) x the NVFP4
    weights 14336x4096 and 4096x14336 through the reference's W4A4 launch
    interface: fr_quantize_act_f32 (f32 -> NVFP4 + scale atoms) then
    fr_gemm_f32out (tcgen05 kind::mxf4nvf4, f32 out).  Weights repacked once
    (fr_repack_weight), 6 sets rotating (> L2)."""
    out = {}
    n_sets = 6
    for (M, N, K) in ((512, 14336, 4096), (512, 4096, 14336), (2048, 4096, 14336)):
        Bs = []
        for s_ in range(n_sets):
            w = torch.from_numpy(frb200.synth_nvfp4(0x5EED0200 + 7 * s_ + N, N, K)).to(dev)
            Bs.append(frb200.repack_weight(w, N, K))
            del w
        x = torch.from_numpy(frb200.synth_normal(0x5EED0210 + K, M * K).reshape(M, K)).to(dev)
        A = torch.empty((M, K // 2), dtype=torch.uint8, device=dev)
        SFA = torch.zeros(frb200.sf_bytes(M, K), dtype=torch.uint8, device=dev)
        D = torch.empty((M, N), dtype=torch.float32, device=dev)

        def step(i, gemm_only=False):
            if not gemm_only:
                frb200.call("fr_quantize_act_f32", frb200._ptr(x), frb200._ptr(A), frb200._ptr(SFA), M, K,
                            frb200._stream(stream))
            B, SFB = Bs[i % n_sets]
            frb200.gemm_f32out(A, SFA, B, SFB, M, N, K, out=D, stream=stream)

        gs = graphs_for(step)
        ms = time_fn(lambda i: gs[i % 4].replay(), max(10, args.steps // 4), 3)
        gg = graphs_for(lambda i: step(i, True))
        ms_g = time_fn(lambda i: gg[i % 4].replay(), max(10, args.steps // 4), 3)
        del gs, gg
        flop = 2.0 * M * N * K
        tf = flop / (ms_g * 1e-3) / 1e12
        byts = N * K // 2 + frb200.sf_bytes(N, K) + M * K // 2 + frb200.sf_bytes(M, K) + 4 * M * N
        attain = min(FP4_DENSE_NOMINAL_TFLOPS, flop / byts * hbm / 1e3)
        key = f"prefill_{M}x{N}x{K}"
        out[f"{key}_gemm_us"] = round(ms_g * 1e3, 2)
        out[f"{key}_gemm_tflops"] = round(tf, 1)
        out[f"{key}_frac_fp4_nominal"] = round(tf / FP4_DENSE_NOMINAL_TFLOPS, 4)
        out[f"{key}_frac_attainable"] = round(tf / attain, 4)
        out[f"{key}_quant_plus_gemm_us"] = round(ms * 1e3, 2)
        del Bs, x, A, SFA, D
    out["prefill_note"] = ("TFLOP/s of fr_gemm_f32out alone (2MNK); frac_fp4_nominal against the 9 PFLOP/s dense FP4 "
                           "figure (nominal, no measured FP4 peak); frac_attainable against min(FP4 nominal, "
                           "FLOP/byte x measured HBM), bytes = packed A/B + scale atoms + f32 D")
    return out


def _decoder_config4(frb200, torch, dev, stream, args):
    """48 layers, hidden 2048, GQA 32/4 x 128, RoPE 1e6, RMSNorm,
    128 experts top-8 FFN 768, vocab 151936, NVFP4 weights (generated on the
    device), f16 KV cache.  A random 1024-token prompt (token ids uniform) is
    fed by 1024 replays of the captured step, then decode steps are timed
    (CUDA events around graph replays; each replay decodes one token per
    sequence, reading the whole model's weights and the KV cache)."""
    from frb200.decoder import Config, MoeDecoder
    out = {}
    P = 1024
    for T, dense, experts in ((1, "ggml", "ggml"), (64, "ggml", "tiled")):
        cfg = Config(ctx=2048)
        dec = MoeDecoder(cfg, T, dense=dense, experts=experts, device=dev)
        g = torch.Generator(device=dev)
        g.manual_seed(0x5EED7000 + T)
        prompt = torch.randint(0, cfg.vocab, (T, P), generator=g, device=dev, dtype=torch.int32)
        dec.set_prompt(prompt)
        with torch.cuda.stream(stream):
            dec.step(stream=stream)                       # eager warm-up: workspaces
        torch.cuda.synchronize()
        dec.set_prompt(prompt)
        dec.kc.zero_()
        dec.vc.zero_()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            dec.step(stream=stream)
        dec.pos.zero_()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for _ in range(P):                              # the prompt
                graph.replay()
        torch.cuda.synchronize()
        n_dec = max(8, min(args.decode_steps, 2048 - P))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(n_dec):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / n_dec
        assert int(dec.pos) == P + n_dec and frb200.device_status() == 0
        out[f"decode_b{T}_tok_s"] = round(T / (ms * 1e-3), 1)
        out[f"decode_b{T}_ms_per_step"] = round(ms, 4)
        out[f"decode_b{T}_layout"] = f"dense {dense}, experts {experts}"
        del graph, dec
        torch.cuda.empty_cache()
    out["decode_note"] = (f"configs[4] model, {P}-token prompt then {n_dec} timed decode steps (positions "
                          f"{P}..{P + n_dec - 1}), one CUDA graph per step, greedy arg-max feeding the next step")
    return out


def run_ours(args):
    import torch
    import frb200
    from frb200 import parallel as P

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
    stream = torch.cuda.Stream(dev)

    def barrier():
        torch.cuda.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if pg is None:
            return v
        t = torch.tensor([v], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    def time_fn(fn, K, W):
        with torch.cuda.stream(stream):
            for i in range(W):
                fn(i)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(K):
                fn(i)
            e1.record(stream)
        e1.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / K

    # ---------------- dense FFN (config 2): single GPU, or sharded over n_ff.
    # Weights are repacked once (as at model load) into the tile-major layout
    # the FP4 tensor-core matvec streams; ggml's in-place layout is measured
    # beside it (dp4a matvec) on one GPU.
    f0, f1 = P.shard_range(N_FF, rank, world)
    sets, gsets = [], []
    for s in range(N_SETS):
        base = 0x5EED0000 + 100 * s
        wg = torch.from_numpy(frb200.synth_nvfp4(base + 1, N_FF, N_EMBD)[f0:f1].copy()).to(dev)
        wu = torch.from_numpy(frb200.synth_nvfp4(base + 2, N_FF, N_EMBD)[f0:f1].copy()).to(dev)
        wd = torch.from_numpy(P.down_shard(frb200.synth_nvfp4(base + 3, N_EMBD, N_FF), N_EMBD, N_FF, rank,
                                           world)).to(dev)
        F_p = f1 - f0
        sets.append((frb200.tile_nvfp4(wg, F_p, N_EMBD), frb200.tile_nvfp4(wu, F_p, N_EMBD),
                     frb200.tile_nvfp4(wd, N_EMBD, F_p)))
        if world == 1:
            gsets.append((wg, wu, wd))
        else:
            del wg, wu, wd
    torch.cuda.synchronize()
    Tmax = 64
    x_all = torch.from_numpy(frb200.synth_normal(0x5EED0000 + 10, Tmax * N_EMBD).reshape(Tmax, N_EMBD)).to(dev)
    outs = [torch.empty((Tmax, N_EMBD), dtype=torch.float32, device=dev) for _ in range(N_SETS)]
    tp = P.TpFfn(Tmax, N_EMBD, N_FF) if world > 1 else None

    def ffn_step(i, T, x=None, out=None, layout="tiled"):
        xx = x_all[:T] if x is None else x
        oo = outs[i % N_SETS][:T] if out is None else out
        if world > 1:
            tp(xx, *sets[i % N_SETS], out=oo, stream=stream, tiled=True)
        elif layout == "tiled":
            frb200.ffn_tiled(xx, *sets[i % N_SETS], N_EMBD, N_FF, out=oo, stream=stream)
        else:
            frb200.ffn(xx, *gsets[i % N_SETS], N_EMBD, N_FF, out=oo, stream=stream)

    def graphs_for(fn):
        with torch.cuda.stream(stream):
            for i in range(N_SETS):           # eager warm-up sizes workspaces, initialises NCCL
                fn(i)
        barrier()
        gs = []
        for i in range(N_SETS):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                fn(i)
            gs.append(g)
        return gs

    def chain_for(fn):
        """One CUDA graph of N_SETS consecutive steps (the rotating weight
        sets, like consecutive layers of one decode pass: the PDL chain runs
        through them, as it does through a forward pass captured whole)."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(N_SETS):
                fn(i)
        return g

    def time_steps(chain, singles, K, W):
        """Exactly K steps: K // N_SETS replays of the chain, then K % N_SETS
        single-step graphs; W warm-up steps the same way."""
        def run(n):
            for _ in range(n // N_SETS):
                chain.replay()
            for i in range(n % N_SETS):
                singles[i].replay()
        with torch.cuda.stream(stream):
            run(max(W, N_SETS))
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            run(K)
            e1.record(stream)
        e1.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / K

    launches0 = frb200.lib().fr_kernel_launches()
    g1 = graphs_for(lambda i: ffn_step(i, 1))
    launches_per_step = (frb200.lib().fr_kernel_launches() - launches0) // (2 * N_SETS)
    c1 = chain_for(lambda i: ffn_step(i, 1))

    sampler = ClockSampler(local)
    sampler.start()
    # ~1.5 s of steps before timing (clocks settle).  Ranks run the same
    # number of steps: the tensor-parallel step advances in lock step, so the
    # count comes from the slowest rank's first chunk, agreed by all-reduce.
    with torch.cuda.stream(stream):
        t0 = time.time()
        for i in range(50):
            c1.replay()
        stream.synchronize()
        chunks = int(1.5 / max(time.time() - t0, 1e-4))
        chunks = int(max_over_ranks(float(min(chunks, 1000))))
        for c in range(chunks):
            for i in range(50):
                c1.replay()
            stream.synchronize()
    ms1 = time_steps(c1, g1, args.steps, max(args.warmup, 3))
    # the same steps with one graph per step (a graph launch between steps)
    ms1_single = time_fn(lambda i: g1[i % N_SETS].replay(), args.steps, max(args.warmup, 3))
    clocks = sampler.stop()

    extra = {}
    for T in (8, 64):
        # T > 16 runs the tile-major FP4 kernel in windows of 16 tokens (each
        # re-streaming the weights); on one GPU the ggml layout's f16
        # tensor-core kernel reads them once for all 64 and is faster there
        layout = "ggml" if (T > 16 and world == 1) else "tiled"
        gT = graphs_for(lambda i, T=T, layout=layout: ffn_step(i, T, layout=layout))
        msT = time_fn(lambda i: gT[i % N_SETS].replay(), max(10, args.steps // 8), max(args.warmup, 3))
        extra[f"ffn_T{T}_gbs"] = round(ffn_bytes(T) / (msT * 1e-3) / 1e9, 1)
        extra[f"ffn_T{T}_ms_per_step"] = round(msT, 5)
        extra[f"ffn_T{T}_path"] = ("ggml layout, f16 tensor-core matvec" if layout == "ggml"
                                   else "tile-major layout, FP4 tensor-core matvec")
        del gT
    if world == 1:
        # ggml's in-place block_nvfp4 layout (no repack): the dp4a matvec
        gg = graphs_for(lambda i: ffn_step(i, 1, layout="ggml"))
        msg = time_fn(lambda i: gg[i % N_SETS].replay(), max(20, args.steps // 4), max(args.warmup, 3))
        extra["ffn_ggml_layout_T1_gbs"] = round(ffn_bytes(1) / (msg * 1e-3) / 1e9, 1)
        extra["ffn_ggml_layout_T1_ms_per_step"] = round(msg, 5)
        del gg

    # dominant kernel (single GPU): the gate/up SwiGLU matvec with its
    # activation-column kernel, timed alone on its stream
    roof = None
    if world == 1:
        glu = torch.empty((1, N_FF), dtype=torch.float32, device=dev)
        kgs = graphs_for(lambda i: frb200.gemv_tiled_swiglu(sets[i][0], sets[i][1], N_FF, N_EMBD, x=x_all[:1],
                                                             out=glu, stream=stream))
        k_ms = time_fn(lambda i: kgs[i % N_SETS].replay(), max(args.steps, 20), 5)
        k_gbs = gateup_bytes(1) / (k_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "kernel": "k_fp4t<16,SWIGLU,1> + k_act_fp4 (gate/up on tile-major weights, T=1)",
                "achieved": round(k_gbs, 1), "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": round(k_gbs / hbm, 4), "traffic": TRAFFIC_GATEUP, "algorithmic_bytes": gateup_bytes(1),
                "ms_per_launch": round(k_ms, 5)}
        del kgs

    # e2e through the public entry point: pinned H2D of x, the FFN, D2H of out
    x_host = torch.from_numpy(frb200.synth_normal(0x5EED0000 + 10, N_EMBD).reshape(1, N_EMBD)).pin_memory()
    o_host = torch.empty((1, N_EMBD), dtype=torch.float32).pin_memory()
    x_dev = torch.empty((1, N_EMBD), dtype=torch.float32, device=dev)

    def e2e_step(i):
        # pinned x -> device, the FFN, device out -> pinned host: the two
        # transfers by fr_copy_pinned (SM loads/stores across PCIe, inside the
        # PDL chain) instead of copy-engine memcpy nodes
        frb200.copy_pinned(x_dev, x_host, stream=stream)
        ffn_step(i, 1, x=x_dev, out=outs[i % N_SETS][:1])
        frb200.copy_pinned(o_host, outs[i % N_SETS][:1], stream=stream)

    egs = graphs_for(e2e_step)
    ec = chain_for(e2e_step)
    e_ms = time_steps(ec, egs, args.steps, max(args.warmup, 3))

    # ---------------- one 4096x4096 NVFP4 x q8_1 matvec through the
    # ggml_mul_mat op surface (f32 activation quantized to q8_1 in the call),
    # rotating 32 weight copies (302 MB > 2x L2) captured as one graph
    if world == 1:
        extra.update(_gemv_config0(frb200, torch, dev, stream, time_fn, graphs_for, hbm, args))
        extra.update(_prefill_config3(frb200, torch, dev, stream, time_fn, graphs_for, hbm, args))

    # ---------------- the synthetic 48-layer MoE decoder, 1024-token
    # prompt then timed decode steps at 1 and 64 sequences (one GPU)
    if world == 1 and not args.no_decoder:
        extra.update(_decoder_config4(frb200, torch, dev, stream, args))

    # ---------------- MoE layer (config 3): fused on one GPU, expert-parallel over ranks
    msets = _moe_sets(frb200, torch, dev, rank, world, 2)
    ep = P.EpMoe(64, 2048, 768, 128, 8) if world > 1 else None
    # one GPU: the experts also repacked tile-major (same bytes) for the FP4
    # tensor-core expert matvecs; the faster layout is reported per batch
    Ep = 128 // world
    tsets = [(wr, frb200.tile_experts(wg, Ep, 768, 2048), frb200.tile_experts(wu, Ep, 768, 2048),
              frb200.tile_experts(wd, Ep, 2048, 768)) for wr, wg, wu, wd in msets]
    torch.cuda.synchronize()
    for T in (1, 64):
        xm = torch.from_numpy(frb200.synth_normal(0x5EED3000 + rank * 131 + T, T * 2048).reshape(T, 2048)).to(dev)
        om = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        runs = {}
        if world == 1:
            runs["ggml layout, dp4a expert matvecs"] = lambda i, xm=xm, om=om: frb200.moe_ffn(
                xm, *msets[i % 2], 2048, 768, 128, 8, out=om, stream=stream)
            runs["tile-major experts, FP4 tensor-core expert matvecs"] = lambda i, xm=xm, om=om: frb200.moe_ffn_tiled(
                xm, *tsets[i % 2], 2048, 768, 128, 8, out=om, stream=stream)
        else:
            runs["expert parallel, ggml-layout experts"] = lambda i, xm=xm, om=om: ep(xm, *msets[i % 2], out=om,
                                                                                       stream=stream)
            runs["expert parallel, tile-major experts"] = lambda i, xm=xm, om=om: ep(
                xm, *tsets[i % 2], out=om, stream=stream, tiled=True)
        best = None
        for name, fn in runs.items():
            mg = graphs_for(fn)
            mms = time_fn(lambda i: mg[i % N_SETS].replay(), max(20, args.steps // 4), max(args.warmup, 3))
            del mg
            extra[f"moe_T{T}_ms_per_layer[{name}]"] = round(mms, 5)
            if best is None or mms < best[1]:
                best = (name, mms)
        extra[f"moe_T{T}_tok_s"] = round(world * T / (best[1] * 1e-3), 1)
        extra[f"moe_T{T}_ms_per_layer"] = round(best[1], 5)
        extra[f"moe_T{T}_path"] = best[0]
    del tsets

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        gbs, cores, sample = cpu_reference_line(args, budget_s=10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}

    value = ffn_bytes(1) / (ms1 * 1e-3) / 1e9 if world > 1 else ffn_bytes(1) / (ms1 * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms1, 5), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "e2m1 (NVFP4 weights x q8_1 activation held exactly as E2M1 digit columns; tcgen05 kind::mxf4nvf4, "
                 "fp32 accumulation)",
        "data": "synthetic (seeded splitmix64 / Box-Muller; BASELINE configs)",
        "config": {"workload": "dense FFN gate/up 14336x4096 + down 4096x14336 NVFP4 x q8_1, T=1 (configs[1]); "
                               "weights repacked once into the tile-major NVFP4 layout (same bytes)",
                   "global_batch": 1, "seq_len": 1,
                   "parallelism": f"tp{world} (sharded over n_ff; the down matvec's epilogue stores its partial rows "
                                  f"into every rank over NVLink, one bounded wait + rank-order sum)" if world > 1
                   else "single GPU",
                   "l2": f"rotating {N_SETS} weight sets ({N_SETS * ffn_bytes(0) / 1e6:.0f} MB > L2)",
                   "graph": "the 4 rotating-weight steps captured as one CUDA graph (PDL edges through them, as "
                            "through the layers of a captured decode pass; no NCCL call on the tp step); "
                            "ms_per_step_one_graph_per_step beside it",
                   "moe": "config 3 layer (E=128, top-8, hidden 2048, FFN 768): fused on 1 GPU; for N > 1 expert-parallel "
                          "(E/N experts per rank, per-rank tokens, routed rows and outputs exchanged by NVLink peer "
                          "stores, bounded waits, one CUDA graph per layer)"},
        "clocks": clocks,
        "e2e": {"value": round(ffn_bytes(1) / (e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": N_EMBD * 4, "d2h_bytes_per_step": N_EMBD * 4,
                "ms_per_step": round(e_ms, 5), "note": "every step: pinned host x -> device and device out -> pinned host by fr_copy_pinned (SM loads/stores across PCIe inside the graph PDL chain), per rank"},
        "gpu_launches": int(launches_per_step * args.steps),
        "roofline": roof,
        "cpu_baseline": cpu,
    }
    extra["ms_per_step_one_graph_per_step"] = round(ms1_single, 5)
    line.update(extra)
    del g1, egs, c1, ec
    if tp is not None:
        tp.close()
    if ep is not None:
        ep.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def run_profile_case(args):
    """A short, fixed sequence of the hot kernels for profiler captures:
    `--case ffn`: four rotating weight sets (> L2) of config 2, `--steps` dense
    FFN steps at T = --tokens (the q8_1 / activation-column kernel, the gate/up
    SwiGLU matvec, the down matvec); `--case moe`: two config-3 layers
    alternating.  Synchronised after each step.  Prints nothing but a done
    line; never a benchmark number."""
    import torch
    import frb200
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.matvec is not None:
        frb200.set_matvec_path(args.matvec)
    if args.case == "gemm":
        # the prefill GEMM: M = --tokens rows against the
        # 14336x4096 and 4096x14336 weights, alternating
        M = args.tokens
        ops = []
        for (N, K) in ((14336, 4096), (4096, 14336)):
            w = torch.from_numpy(frb200.synth_nvfp4(0x5EED0200 + N, N, K)).to(dev)
            B, SFB = frb200.repack_weight(w, N, K)
            x = torch.from_numpy(frb200.synth_normal(0x5EED0210 + K, M * K).reshape(M, K)).to(dev)
            A, SFA = frb200.quantize_act_f32(x)
            D = torch.empty((M, N), dtype=torch.float32, device=dev)
            ops.append((A, SFA, B, SFB, D, N, K))
        for i in range(args.steps):
            A, SFA, B, SFB, D, N, K = ops[i % 2]
            frb200.gemm_f32out(A, SFA, B, SFB, M, N, K, out=D)
            torch.cuda.synchronize()
        print(f"profile case done: {args.steps} GEMMs, M={M}, status {frb200.device_status()}")
        return
    if args.case == "decoder":
        # a 4-layer configs[4] decoder (--layout for the dense and expert
        # weights; mixed = the batch-64 bench's ggml dense, tiled experts),
        # 8 prompt tokens then --steps decode steps, eager
        from frb200.decoder import Config, MoeDecoder
        T = args.tokens
        cfg = Config(n_layers=4, ctx=2048)
        dense, experts = ("ggml", "tiled") if args.layout == "mixed" else (args.layout, args.layout)
        dec = MoeDecoder(cfg, T, dense=dense, experts=experts, device=dev)
        g = torch.Generator(device=dev)
        g.manual_seed(0x5EED7100 + T)
        dec.set_prompt(torch.randint(0, cfg.vocab, (T, 8), generator=g, device=dev, dtype=torch.int32))
        for i in range(8 + args.steps):
            if i == 8 and args.pos > 8:
                dec.pos.fill_(args.pos)     # decode at --pos (cache rows 8..pos-1 stay zero: finite keys)
            dec.step()
            torch.cuda.synchronize()
        print(f"profile case done: {8 + args.steps} decoder steps, T={T}, 4 layers, status {frb200.device_status()}")
        return
    if args.case == "attn":
        # decode attention (configs[4] shapes): --tokens sequences, keys
        # 0..1023 of a 2048-row f16 cache per layer, 4 layers rotating
        T, nh, nkv, d, ctx = args.tokens, 32, 4, 128, 2048
        g = torch.Generator(device=dev)
        g.manual_seed(1)
        caches = [(torch.randn((T, nkv, ctx, d), generator=g, device=dev).half(),
                   torch.randn((T, nkv, ctx, d), generator=g, device=dev).half()) for _ in range(4)]
        q = torch.randn((T, nh, d), generator=g, device=dev) / d ** 0.5
        out = torch.empty((T, nh * d), dtype=torch.float32, device=dev)
        pos = torch.tensor([1023], dtype=torch.int32, device=dev)
        for i in range(args.steps):
            kc, vc = caches[i % 4]
            frb200.call("fr_attn_decode_f16", frb200._ptr(q), frb200._ptr(kc), frb200._ptr(vc), frb200._ptr(pos),
                        frb200._ptr(out), T, nh, nkv, d, ctx, frb200._stream())
            torch.cuda.synchronize()
        print(f"profile case done: {args.steps} attention launches, T={T}, status {frb200.device_status()}")
        return
    if args.case == "moe":
        msets = _moe_sets(frb200, torch, dev, 0, 1, 2)
        if args.layout == "tiled":
            msets = [(wr, frb200.tile_experts(wg, 128, 768, 2048), frb200.tile_experts(wu, 128, 768, 2048),
                      frb200.tile_experts(wd, 128, 2048, 768)) for wr, wg, wu, wd in msets]
        layer = frb200.moe_ffn_tiled if args.layout == "tiled" else frb200.moe_ffn
        T = args.tokens
        xm = torch.from_numpy(frb200.synth_normal(0x5EED3000 + T, T * 2048).reshape(T, 2048)).to(dev)
        om = torch.empty((T, 2048), dtype=torch.float32, device=dev)
        for i in range(args.steps):
            layer(xm, *msets[i % 2], 2048, 768, 128, 8, out=om)
            torch.cuda.synchronize()
        print(f"profile case done: {args.steps} MoE layers, T={T}, status {frb200.device_status()}")
        return
    sets = []
    for s in range(N_SETS):
        base = 0x5EED0000 + 100 * s
        sets.append(tuple(torch.from_numpy(w).to(dev) for w in (frb200.synth_nvfp4(base + 1, N_FF, N_EMBD),
                                                                 frb200.synth_nvfp4(base + 2, N_FF, N_EMBD),
                                                                 frb200.synth_nvfp4(base + 3, N_EMBD, N_FF))))
    if args.layout == "tiled":
        sets = [(frb200.tile_nvfp4(wg, N_FF, N_EMBD), frb200.tile_nvfp4(wu, N_FF, N_EMBD),
                 frb200.tile_nvfp4(wd, N_EMBD, N_FF)) for wg, wu, wd in sets]
        torch.cuda.synchronize()
    T = args.tokens
    x = torch.from_numpy(frb200.synth_normal(0x5EED0000 + 10, T * N_EMBD).reshape(T, N_EMBD)).to(dev)
    out = torch.empty((T, N_EMBD), dtype=torch.float32, device=dev)
    for i in range(args.steps):
        wg, wu, wd = sets[i % N_SETS]
        if args.layout == "tiled":
            frb200.ffn_tiled(x, wg, wu, wd, N_EMBD, N_FF, out=out)
        else:
            frb200.ffn(x, wg, wu, wd, N_EMBD, N_FF, out=out)
        torch.cuda.synchronize()
    print(f"profile case done: {args.steps} FFN steps, T={T}, status {frb200.device_status()}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-decoder", action="store_true", help="skip the configs[4] decoder lines")
    ap.add_argument("--decode-steps", type=int, default=64, help="timed decode steps of the configs[4] decoder")
    ap.add_argument("--profile-case", action="store_true",
                    help="run a short fixed kernel sequence for profiler captures (no benchmark line)")
    ap.add_argument("--tokens", type=int, default=1, help="tokens per step of --profile-case")
    ap.add_argument("--matvec", type=int, default=None, help="force the matvec kernel (1 dp4a, 2 tc-f16, 3 tc-fp4)")
    ap.add_argument("--layout", choices=["ggml", "tiled", "mixed"], default="ggml",
                    help="weight layout of --profile-case (mixed: decoder dense ggml, experts tiled)")
    ap.add_argument("--pos", type=int, default=0,
                    help="decoder --profile-case: position of the decode steps after the 8-token prompt")
    ap.add_argument("--case", choices=["ffn", "moe", "gemm", "attn", "decoder"], default="ffn",
                    help="workload of --profile-case")
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
