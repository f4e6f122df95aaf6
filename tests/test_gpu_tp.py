"""Tensor-parallel dense FFN with the all-gathers fused into the matvec
epilogues (fr_tp_ffn_nvfp4, frb200.parallel.TpFfn): every rank's output must
equal, bit for bit, the single-GPU FFN on the unsharded weights (each output
row is the same dot product in the same order; q8_1 blocks never straddle a
shard boundary).  Runs one rank per visible GPU, at most 2 (world 1 on a
one-GPU box exercises the same peer-store and flag code with one peer)."""
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
    tp = None
    try:
        frb200.set_matvec_path(1)
        ne, nf = 1024, 2048
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        wg = t(frb200.synth_nvfp4(41, nf, ne))
        wu = t(frb200.synth_nvfp4(42, nf, ne))
        wd = t(frb200.synth_nvfp4(43, ne, nf))
        f0, f1 = P.shard_range(nf, rank, world)
        e0, e1 = P.shard_range(ne, rank, world)
        shards = (wg[f0:f1].contiguous(), wu[f0:f1].contiguous(), wd[e0:e1].contiguous())
        sc = t(np.array([0.75, 1.25, 0.5], np.float32))
        tp = P.TpFfn(8, ne, nf)
        bad = []
        for i, T in enumerate((1, 3, 8, 1, 2)):
            x = t(frb200.synth_normal(50 + i, T * ne).reshape(T, ne))
            r = t(frb200.synth_normal(60 + i, T * ne).reshape(T, ne)) if i % 2 else None
            kw = dict(sg=sc[0:1], su=sc[1:2], sd=sc[2:3]) if i == 2 else {}
            y = tp(x, *shards, resid=r, **kw)
            ref = frb200.ffn(x, wg, wu, wd, ne, nf, resid=r, **kw)
            torch.cuda.synchronize()
            if not torch.equal(y, ref):
                bad.append(f"T={T}: max |d| {float((y - ref).abs().max()):.3e}")
        # the step captured in a CUDA graph and replayed with new inputs
        xg = torch.empty((2, ne), dtype=torch.float32, device=dev)
        yg = torch.empty((2, ne), dtype=torch.float32, device=dev)
        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            tp(xg.copy_(t(frb200.synth_normal(70, 2 * ne).reshape(2, ne))), *shards, out=yg, stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            tp(xg, *shards, out=yg, stream=s)
        for i in range(4):
            xi = t(frb200.synth_normal(80 + i, 2 * ne).reshape(2, ne))
            xg.copy_(xi)
            g.replay()
            torch.cuda.synchronize()
            ref = frb200.ffn(xi, wg, wu, wd, ne, nf)
            torch.cuda.synchronize()
            if not torch.equal(yg, ref):
                bad.append(f"graph replay {i}: max |d| {float((yg - ref).abs().max()):.3e}")
        del g
        status = frb200.device_status()
        q.put((rank, bad, status))
    except Exception as e:  # noqa: BLE001 - report to the parent instead of hanging it
        q.put((rank, [repr(e)], -1))
        raise
    finally:
        if tp is not None:
            tp.close()
        dist.destroy_process_group()


def test_tp_ffn_fused_epilogue_matches_single_gpu():
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
