"""Expert-parallel MoE over NVLink peer stores (fr_ep_moe_nvfp4,
frb200.parallel.EpMoe): every rank's output must equal, bit for bit, the
single-GPU fused layer (fr_moe_ffn_nvfp4) on the full expert set for that
rank's tokens -- the same per-slot arithmetic and the same slot-order combine.
Runs one rank per visible GPU, at most 2 (world 1 exercises the dispatch,
bounded waits, empty-slot skipping and return with one peer), including calls
with fewer tokens than the buffer holds and CUDA-graph replays."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "flashrt-llama.cpp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import datetime
    import torch
    import torch.distributed as dist
    import frb200
    from frb200 import parallel as P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    ep = None
    bad = []
    try:
        ne, nf, E, n_used = 256, 512, 32, 4
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        wg = frb200.synth_nvfp4(21, E * nf, ne)
        wu = frb200.synth_nvfp4(22, E * nf, ne)
        wd = frb200.synth_nvfp4(23, E * ne, nf)
        wr = t(frb200.synth_normal(24, E * ne, 0.0, 0.02).reshape(E, ne))
        Ep = E // world
        lg = t(wg[rank * Ep * nf:(rank + 1) * Ep * nf])
        lu = t(wu[rank * Ep * nf:(rank + 1) * Ep * nf])
        ld = t(wd[rank * Ep * ne:(rank + 1) * Ep * ne])
        fg, fu, fd = t(wg), t(wu), t(wd)
        ep = P.EpMoe(16, ne, nf, E, n_used)
        for i, T in enumerate((1, 16, 5, 1, 16)):
            x = t(frb200.synth_normal(30 + 7 * rank + i, T * ne).reshape(T, ne))
            r = t(frb200.synth_normal(40 + 7 * rank + i, T * ne).reshape(T, ne)) if i % 2 else None
            y = ep(x, wr, lg, lu, ld, resid=r)
            ref = frb200.moe_ffn(x, wr, fg, fu, fd, ne, nf, E, n_used, resid=r)
            torch.cuda.synchronize()
            if not torch.equal(y, ref):
                bad.append(f"T={T}: max |d| {float((y - ref).abs().max()):.3e}")
        # captured in a CUDA graph, replayed with new inputs
        xg = torch.empty((8, ne), dtype=torch.float32, device=dev)
        yg = torch.empty((8, ne), dtype=torch.float32, device=dev)
        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            xg.copy_(t(frb200.synth_normal(60, 8 * ne).reshape(8, ne)))
            ep(xg, wr, lg, lu, ld, out=yg, stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ep(xg, wr, lg, lu, ld, out=yg, stream=s)
        for i in range(3):
            xi = t(frb200.synth_normal(70 + 7 * rank + i, 8 * ne).reshape(8, ne))
            xg.copy_(xi)
            g.replay()
            torch.cuda.synchronize()
            ref = frb200.moe_ffn(xi, wr, fg, fu, fd, ne, nf, E, n_used)
            torch.cuda.synchronize()
            if not torch.equal(yg, ref):
                bad.append(f"graph replay {i}: max |d| {float((yg - ref).abs().max()):.3e}")
        del g
        torch.cuda.synchronize()
        # tile-major experts (fr_ep_moe_tiled) against the single-GPU tiled
        # layer: equal to the f32 rounding of the split-K partial sums, whose
        # grouping follows each launch's work split (normwise 1e-5)
        tg, tu, td = (frb200.tile_experts(lg, Ep, nf, ne), frb200.tile_experts(lu, Ep, nf, ne),
                      frb200.tile_experts(ld, Ep, ne, nf))
        Fg, Fu, Fd = (frb200.tile_experts(fg, E, nf, ne), frb200.tile_experts(fu, E, nf, ne),
                      frb200.tile_experts(fd, E, ne, nf))
        for i, T in enumerate((1, 16, 7)):
            x = t(frb200.synth_normal(90 + 7 * rank + i, T * ne).reshape(T, ne))
            y = ep(x, wr, tg, tu, td, tiled=True)
            ref = frb200.moe_ffn_tiled(x, wr, Fg, Fu, Fd, ne, nf, E, n_used)
            torch.cuda.synchronize()
            err = float((y - ref).norm() / ref.norm())
            if not (err <= 1e-5 and bool(torch.isfinite(y).all())):
                bad.append(f"tiled T={T}: normwise {err:.3e}")
        torch.cuda.synchronize()
        q.put((rank, bad, frb200.device_status()))
    except Exception as e:  # noqa: BLE001 - report to the parent instead of hanging it
        q.put((rank, bad + [repr(e)], -1))
        raise
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


def test_ep_moe_matches_single_gpu():
    import torch
    world = min(2, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, bad, status = q.get(timeout=300)
        res[rank] = (bad, status)
    for p in procs:
        p.join(timeout=60)
    for rank in range(world):
        bad, status = res[rank]
        assert not bad, f"rank {rank}: {bad}"
        assert status == 0, f"rank {rank}: device status {status:#x}"
    for p in procs:
        assert p.exitcode == 0
