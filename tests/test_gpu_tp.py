"""Tensor-parallel dense FFN sharded over n_ff with the reduction fused into
the down matvec's epilogue (fr_tp_ffn_nvfp4, frb200.parallel.TpFfn).  Every
rank must produce the same output, and it must match the single-GPU FFN on
the unsharded weights: the GLU bit for bit (the same dot products; q8_1 blocks
never straddle a shard), the output up to the f32 rounding of summing the
ranks' K-range partials (max |d| <= 1e-5 * max|ref| on the dp4a matvec; on
the tensor-core matvecs, whose split-K order differs too, the matvec
tolerance max |d| / max(|ref|, 1% rms) <= 1e-3).  Consecutive steps run with
no host synchronisation, one rank delayed, to show the double-buffered
partial slots.
Runs one rank per visible GPU, at most 2 (world 1 on a one-GPU box exercises
the same peer-store, flag and reduce code with one peer), including CUDA-graph
replays with new inputs."""
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
    tps = []
    bad, sums = [], []
    try:
        ne, nf = 1024, 2048
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        wg = t(frb200.synth_nvfp4(41, nf, ne))
        wu = t(frb200.synth_nvfp4(42, nf, ne))
        wd = t(frb200.synth_nvfp4(43, ne, nf))
        f0, f1 = P.shard_range(nf, rank, world)
        shards = (wg[f0:f1].contiguous(), wu[f0:f1].contiguous(), P.down_shard(wd, ne, nf, rank, world))
        sc = t(np.array([0.75, 1.25, 0.5], np.float32))

        def check(y, ref, what, tc):
            torch.cuda.synchronize()
            sums.append(float(y.double().sum()))
            if not bool(torch.isfinite(y).all()):
                bad.append(f"{what}: non-finite")
            elif tc:
                # the tensor-core paths sum K in another order, so a GLU value
                # can round to the other side of a q8_1 step: one such flip
                # moves an output by ~3e-4 of its rms -- within the matvec
                # tolerance (max |d| / max(|ref|, 1% rms) <= 1e-3)
                d, r = (y - ref).double().abs(), ref.double()
                floor = 1e-2 * float(r.pow(2).mean().sqrt())
                err = float((d / r.abs().clamp_min(floor)).max())
                if err > 1e-3:
                    bad.append(f"{what}: max rel err {err:.3e}")
            else:
                err = float((y - ref).abs().max() / ref.abs().max())
                if err > 1e-5:
                    bad.append(f"{what}: max err {err:.3e}")

        for path, Ts in ((1, (1, 3, 8, 1, 2, 12)), (2, (3, 16, 64))):
            frb200.set_matvec_path(path)
            tp = P.TpFfn(max(Ts), ne, nf)
            tps.append(tp)
            for i, T in enumerate(Ts):
                x = t(frb200.synth_normal(50 + i, T * ne).reshape(T, ne))
                r = t(frb200.synth_normal(60 + i, T * ne).reshape(T, ne)) if i % 2 else None
                kw = dict(sg=sc[0:1], su=sc[1:2], sd=sc[2:3]) if i == 2 else {}
                y = tp(x, *shards, resid=r, **kw)
                check(y, frb200.ffn(x, wg, wu, wd, ne, nf, resid=r, **kw), f"path {path} T={T}", path == 2)
        # tile-major shards (FP4 tensor-core matvecs)
        frb200.set_matvec_path(0)
        tshards = (frb200.tile_nvfp4(shards[0], nf // world, ne), frb200.tile_nvfp4(shards[1], nf // world, ne),
                   frb200.tile_nvfp4(shards[2], ne, nf // world))
        tpt = P.TpFfn(8, ne, nf)
        tps.append(tpt)
        for i, T in enumerate((1, 2, 8)):
            x = t(frb200.synth_normal(110 + i, T * ne).reshape(T, ne))
            r = t(frb200.synth_normal(115 + i, T * ne).reshape(T, ne))
            y = tpt(x, *tshards, resid=r, tiled=True)
            check(y, frb200.ffn(x, wg, wu, wd, ne, nf, resid=r), f"tiled T={T}", True)
        # the step captured in a CUDA graph and replayed with new inputs
        tp = tps[0]
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
            check(yg, frb200.ffn(xi, wg, wu, wd, ne, nf), f"graph replay {i}", False)
        del g
        torch.cuda.synchronize()
        # consecutive steps on one stream with no host synchronisation between
        # them, the last rank delayed before every other step so that the
        # others run a step ahead: each step's partial rows must land in the
        # other parity half of the shared buffer, never in the half a slower
        # rank is still summing
        # (the kernels are deterministic, so each chained step must equal the
        # same step run with the host synchronised after it, bit for bit)
        xs = [t(frb200.synth_normal(200 + i, 4 * ne).reshape(4, ne)) for i in range(8)]
        for name, fn in (("dp4a", lambda x, o: tps[0](x, *shards, out=o, stream=s)),
                         ("tiled", lambda x, o: tpt(x, *tshards, out=o, stream=s, tiled=True))):
            frb200.set_matvec_path(1 if name == "dp4a" else 0)
            ys = [torch.empty((4, ne), dtype=torch.float32, device=dev) for _ in xs]
            yr = [torch.empty((4, ne), dtype=torch.float32, device=dev) for _ in xs]
            with torch.cuda.stream(s):
                for x, o in zip(xs, yr):
                    fn(x, o)
                    s.synchronize()
            torch.cuda.synchronize()
            dist.barrier()
            with torch.cuda.stream(s):
                for i, (x, o) in enumerate(zip(xs, ys)):
                    if rank == world - 1 and i % 2 == 1:
                        torch.cuda._sleep(2_000_000)
                    fn(x, o)
            s.synchronize()
            for i in range(len(xs)):
                sums.append(float(ys[i].double().sum()))
                if not torch.equal(ys[i], yr[i]):
                    bad.append(f"chained {name} step {i}: differs from the synchronised step by "
                               f"{float((ys[i] - yr[i]).abs().max()):.3e}")
        # the row-sharded form (north-star partitioning): equal to the
        # single-GPU dp4a FFN bit for bit, chained steps included
        frb200.set_matvec_path(1)
        tpr = P.TpFfnRows(8, ne, nf)
        tps.append(tpr)
        rsh = P.row_shards(wg, wu, wd, ne, nf, rank, world)
        yrow = [torch.empty((T, ne), dtype=torch.float32, device=dev) for T in (1, 3, 8, 2, 8, 5)]
        xrow = [t(frb200.synth_normal(300 + i, y.shape[0] * ne).reshape(y.shape[0], ne)) for i, y in enumerate(yrow)]
        rrow = [t(frb200.synth_normal(320 + i, y.shape[0] * ne).reshape(y.shape[0], ne)) for i, y in enumerate(yrow)]
        torch.cuda.synchronize()
        dist.barrier()
        with torch.cuda.stream(s):
            for i, (x, r, y) in enumerate(zip(xrow, rrow, yrow)):
                if rank == world - 1 and i % 2 == 1:
                    torch.cuda._sleep(2_000_000)
                tpr(x, *rsh, resid=r, out=y, stream=s, **(dict(sg=sc[0:1], su=sc[1:2], sd=sc[2:3]) if i == 4 else {}))
        s.synchronize()
        for i, (x, r, y) in enumerate(zip(xrow, rrow, yrow)):
            kw = dict(sg=sc[0:1], su=sc[1:2], sd=sc[2:3]) if i == 4 else {}
            ref = frb200.ffn(x, wg, wu, wd, ne, nf, resid=r, **kw)
            torch.cuda.synchronize()
            sums.append(float(y.double().sum()))
            if not torch.equal(y, ref):
                bad.append(f"rows-sharded step {i}: differs from one GPU by {float((y - ref).abs().max()):.3e}")
        frb200.set_matvec_path(0)
        q.put((rank, bad, frb200.device_status(), sums))
    except Exception as e:  # noqa: BLE001 - report to the parent instead of hanging it
        q.put((rank, bad + [repr(e)], -1, sums))
        raise
    finally:
        for tp in tps:
            tp.close()
        dist.destroy_process_group()


def test_tp_ffn_fused_reduce_matches_single_gpu():
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
        rank, bad, status, sums = q.get(timeout=300)
        res[rank] = (bad, status, sums)
    for p in procs:
        p.join(timeout=60)
    for rank in range(world):
        bad, status, sums = res[rank]
        assert not bad, f"rank {rank}: {bad}"
        assert status == 0, f"rank {rank}: device status {status:#x}"
        assert sums == res[0][2], "ranks disagree"
    for p in procs:
        assert p.exitcode == 0
