"""Multi-rank exchange logic of frb200.parallel on CPU: world_size 2 over gloo,
with the CPU oracle standing in for the kernels.  Expert-parallel MoE must give
exactly the single-rank result (same arithmetic per slot, combine in slot
order); the n_ff-sharded FFN gives the same result on every rank and the
single-rank result up to the f32 rounding of the partial sums."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

WORLD = 2


class OracleKernels:
    """The oracle's arithmetic on CPU tensors (test infrastructure)."""

    def __init__(self, O):
        self.O = O

    def gate_up(self, x, wg, wu, n_rows, K):
        q = self.O.quantize_q8_1(x.numpy())
        g = self.O.gemv_q8_1(wg.numpy(), q, n_rows, K).astype(np.float32)
        u = self.O.gemv_q8_1(wu.numpy(), q, n_rows, K).astype(np.float32)
        return torch.from_numpy(u * self.O.silu_np(g))

    def down(self, glu, wd, n_rows, K):
        q = self.O.quantize_q8_1(glu.numpy())
        return torch.from_numpy(self.O.gemv_q8_1(wd.numpy(), q, n_rows, K).astype(np.float32))

    def route(self, x, w_r, n_used, clamp):
        logits = (x.double() @ w_r.double().T).float().numpy()
        ids, w = self.O.topk_softmax(logits, n_used, clamp)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def experts(self, x, eid, wg, wu, wd, n_embd, n_ff, E):
        out = torch.zeros((x.shape[0], n_embd), dtype=torch.float32)
        for s in range(x.shape[0]):
            e = int(eid[s])
            xs = x[s:s + 1]
            glu = self.gate_up(xs, wg[e * n_ff:(e + 1) * n_ff], wu[e * n_ff:(e + 1) * n_ff], n_ff, n_embd)
            out[s] = self.down(glu, wd[e * n_embd:(e + 1) * n_embd], n_embd, n_ff)[0]
        return out

    def combine(self, part, wts, n_embd, resid=None):
        T, n_used = wts.shape
        p = part.view(T, n_used, n_embd)
        out = p[:, 0] * wts[:, 0:1]
        for k in range(1, n_used):
            out = out + p[:, k] * wts[:, k:k + 1]
        if resid is not None:
            out = out + resid
        return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _data():
    import frb200
    n_embd, n_ff, E, n_used, T = 256, 512, 32, 4, 5
    d = dict(n_embd=n_embd, n_ff=n_ff, E=E, n_used=n_used, T=T)
    d["wg"] = torch.from_numpy(frb200.synth_nvfp4(11, E * n_ff, n_embd))
    d["wu"] = torch.from_numpy(frb200.synth_nvfp4(12, E * n_ff, n_embd))
    d["wd"] = torch.from_numpy(frb200.synth_nvfp4(13, E * n_embd, n_ff))
    d["wr"] = torch.from_numpy(frb200.synth_normal(14, E * n_embd, 0.0, 0.02).reshape(E, n_embd))
    d["x"] = torch.from_numpy(frb200.synth_normal(15, WORLD * T * n_embd).reshape(WORLD * T, n_embd))
    d["r"] = torch.from_numpy(frb200.synth_normal(16, WORLD * T * n_embd).reshape(WORLD * T, n_embd))
    return d


def _worker(rank, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (root, os.path.join(root, "flashrt-llama.cpp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    from oracle import oracle as O
    from frb200 import parallel as P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        d = _data()
        K = OracleKernels(O)
        ne, nf, E = d["n_embd"], d["n_ff"], d["E"]
        # --- tensor parallel: first expert's matrices as a dense FFN
        wg, wu, wd = d["wg"][:nf], d["wu"][:nf], d["wd"][:ne]
        f0, f1 = P.shard_range(nf, rank, WORLD)
        x = d["x"][:2]
        y_tp = P.tp_ffn(x, wg[f0:f1], wu[f0:f1], P.down_shard(wd, ne, nf, rank, WORLD), ne, nf, resid=d["r"][:2],
                        kernels=K)
        # --- expert parallel: this rank's tokens, this rank's experts
        T = d["T"]
        xs = d["x"][rank * T:(rank + 1) * T]
        rs = d["r"][rank * T:(rank + 1) * T]
        Ep = E // WORLD
        sl = slice(rank * Ep * nf, (rank + 1) * Ep * nf)
        sd = slice(rank * Ep * ne, (rank + 1) * Ep * ne)
        y_ep = P.ep_moe(xs, d["wr"], d["wg"][sl], d["wu"][sl], d["wd"][sd], ne, nf, E, d["n_used"], resid=rs,
                        kernels=K)
        q.put((rank, y_tp.numpy(), y_ep.numpy()))
    except Exception as e:  # noqa: BLE001 - report to the parent instead of hanging it
        q.put((rank, repr(e), None))
        raise
    finally:
        dist.destroy_process_group()


def _reference(O):
    d = _data()
    K = OracleKernels(O)
    ne, nf, E, n_used, T = d["n_embd"], d["n_ff"], d["E"], d["n_used"], d["T"]
    x = d["x"][:2]
    glu = K.gate_up(x, d["wg"][:nf], d["wu"][:nf], nf, ne)
    y_tp = K.down(glu, d["wd"][:ne], ne, nf) + d["r"][:2]
    outs = []
    for rank in range(WORLD):
        xs = d["x"][rank * T:(rank + 1) * T]
        rs = d["r"][rank * T:(rank + 1) * T]
        ids, w = K.route(xs, d["wr"], n_used, 6.103515625e-5)
        rows = xs[torch.arange(T).repeat_interleave(n_used)]
        part = K.experts(rows, ids.reshape(-1).int(), d["wg"], d["wu"], d["wd"], ne, nf, E)
        outs.append(K.combine(part, w, ne, resid=rs).numpy())
    return y_tp.numpy(), outs


def test_tp_ffn_and_ep_moe_match_single_rank(O, fr):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(WORLD):
        rank, y_tp, y_ep = q.get(timeout=240)
        assert y_ep is not None, f"rank {rank} failed: {y_tp}"
        res[rank] = (y_tp, y_ep)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref_tp, ref_ep = _reference(O)
    # TP: the ranks agree exactly; the rank-order sum of the K-range partials
    # matches the single-rank product to f32 rounding
    np.testing.assert_array_equal(res[0][0], res[1][0])
    np.testing.assert_allclose(res[0][0], ref_tp, rtol=1e-5, atol=1e-5)
    for rank in range(WORLD):
        np.testing.assert_array_equal(res[rank][1], ref_ep[rank])


def test_shard_range():
    from frb200.parallel import shard_range
    assert shard_range(14336, 3, 8) == (5376, 7168)
    with pytest.raises(ValueError):
        shard_range(100, 0, 8)


def test_down_shard_blocks():
    """The K-shards of a down matrix, put side by side, are the matrix."""
    import frb200
    from frb200.parallel import down_shard
    ne, nf, world = 8, 512, 4
    wd = frb200.synth_nvfp4(3, ne, nf)
    parts = [down_shard(wd, ne, nf, r, world).reshape(ne, -1, 36) for r in range(world)]
    np.testing.assert_array_equal(np.concatenate(parts, axis=1).reshape(ne, -1), wd)
    wt = torch.from_numpy(wd)
    np.testing.assert_array_equal(down_shard(wt, ne, nf, 1, world).numpy(), down_shard(wd, ne, nf, 1, world))
    with pytest.raises(ValueError):
        down_shard(wd, ne, nf, 0, 3)
