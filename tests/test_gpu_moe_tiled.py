"""Parity of the MoE path on tile-major expert weights (fr_mul_mat_id_tiled,
fr_moe_ffn_tiled: per-expert matvecs on the FP4 tensor cores) through the
C-ABI on a B200, against the fp64 oracle with the dense tolerances (max rel
err 1e-3 against max(|ref|, 1% rms), normwise 1e-5, zero values outside the
reference's gate, all finite).  The routing, grouping and combine are the
ones test_gpu_moe.py pins; here the stages are checked on the device's own
intermediates (GLU, per-slot down outputs), including experts that receive
more than one 16-token window and CUDA-graph replays."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3
NTOL = 1e-5
CLAMP = 6.103515625e-5


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _check(mine, ref, O, what=""):
    mine = np.asarray(mine, np.float64)
    assert np.all(np.isfinite(mine)), what
    err = O.rel_err(mine, ref)
    assert err <= RTOL, f"{what}: max rel err {err:.3e}"
    assert O.norm_err(mine, ref) <= NTOL, what
    assert O.ref_gate_bad(mine, ref) == 0, what


def _expert_dot(O, w_all, e, N, K, q8row):
    return O.gemv_q8_1(w_all[e * N:(e + 1) * N], q8row, N, K)[0]


@pytest.mark.parametrize("T,n_used,bcast,E,N,K", [
    (1, 8, True, 32, 256, 2048),
    (4, 8, False, 32, 256, 768),
    (16, 6, True, 16, 384, 512),
    (3, 2, False, 8, 128, 256),
    (40, 2, True, 4, 128, 512),      # ~20 tokens per expert: two windows
])
def test_mul_mat_id_tiled(fr, O, dev, T, n_used, bcast, E, N, K):
    import torch
    w = fr.synth_nvfp4(900 + T, E * N, K)
    rng = np.random.default_rng(T * 10 + n_used)
    ids = np.stack([rng.choice(E, n_used, replace=False) for _ in range(T)]).astype(np.int32)
    if bcast:
        x = fr.synth_normal(901, T * K).reshape(T, K)
    else:
        x = fr.synth_normal(902, T * n_used * K).reshape(T, n_used, K)
    wt = fr.tile_experts(_t(w, dev), E, N, K)
    out = fr.mul_mat_id_tiled(wt, E, N, K, _t(x, dev), _t(ids, dev), bcast)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for t in range(T):
        for k in range(n_used):
            xr = x[t] if bcast else x[t, k]
            ref = _expert_dot(O, w, ids[t, k], N, K, O.quantize_q8_1(xr.reshape(1, K)))
            _check(got[t, k], ref, O, f"t={t} k={k}")
    assert fr.device_status() == 0


def test_mul_mat_id_tiled_one_hot_expert(fr, O, dev):
    """Every token on expert 5 (and one slot per token elsewhere): 37 tokens
    on one expert is three windows of the same weights, each slot its row."""
    import torch
    E, N, K, T, n_used = 8, 128, 512, 37, 2
    w = fr.synth_nvfp4(910, E * N, K)
    ids = np.zeros((T, n_used), np.int32)
    ids[:, 0] = 5
    ids[:, 1] = np.where(np.arange(T) % E == 5, 6, np.arange(T) % E)
    x = fr.synth_normal(911, T * K).reshape(T, K)
    wt = fr.tile_experts(_t(w, dev), E, N, K)
    out = fr.mul_mat_id_tiled(wt, E, N, K, _t(x, dev), _t(ids, dev), True)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for t in range(T):
        q = O.quantize_q8_1(x[t].reshape(1, K))
        for k in range(n_used):
            _check(got[t, k], _expert_dot(O, w, ids[t, k], N, K, q), O, f"t={t} k={k}")
    assert fr.device_status() == 0


def _moe_weights(fr, dev, E, n_embd, n_ff, seed):
    wg = fr.synth_nvfp4(seed + 1, E * n_ff, n_embd)
    wu = fr.synth_nvfp4(seed + 2, E * n_ff, n_embd)
    wd = fr.synth_nvfp4(seed + 3, E * n_embd, n_ff)
    wr = fr.synth_normal(seed + 4, E * n_embd, 0.0, 0.02).reshape(E, n_embd)
    tiled = (fr.tile_experts(_t(wg, dev), E, n_ff, n_embd), fr.tile_experts(_t(wu, dev), E, n_ff, n_embd),
             fr.tile_experts(_t(wd, dev), E, n_embd, n_ff))
    return wg, wu, wd, wr, tiled


@pytest.mark.parametrize("T,E", [(1, 128), (8, 128), (64, 128), (64, 32)])
def test_moe_ffn_tiled_stagewise(fr, O, dev, T, E):
    """Config 3 shapes (hidden 2048, FFN 768, top-8); E=32 at T=64 puts ~16
    tokens on each expert, so several experts take two windows."""
    import torch
    n_embd, n_ff, n_used = 2048, 768, 8
    wg, wu, wd, wr, (wg_t, wu_t, wd_t) = _moe_weights(fr, dev, E, n_embd, n_ff, 950)
    sg = np.abs(fr.synth_normal(955, E)).astype(np.float32) + 0.5
    x = fr.synth_normal(960 + T, T * n_embd).reshape(T, n_embd)
    r = fr.synth_normal(961, T * n_embd).reshape(T, n_embd)
    xd = _t(x, dev)
    out, chk = fr.moe_ffn_tiled(xd, _t(wr, dev), wg_t, wu_t, wd_t, n_embd, n_ff, E, n_used, sg=_t(sg, dev),
                                resid=_t(r, dev), check=True)
    _, ids_r, wts_r, _, _, _ = fr.moe_route(xd, _t(wr, dev), n_used, CLAMP)
    torch.cuda.synchronize()
    ids = chk["ids"].cpu().numpy()
    wts = chk["wts"].cpu().numpy()
    np.testing.assert_array_equal(ids, ids_r.cpu().numpy())
    np.testing.assert_array_equal(wts, wts_r.cpu().numpy())
    glu = chk["glu"].cpu().numpy()
    part = chk["part"].cpu().numpy()
    o = out.cpu().numpy()
    for t in sorted({0, T // 2, T - 1}):
        qx = O.quantize_q8_1(x[t].reshape(1, n_embd))
        for k in range(n_used):
            e = ids[t, k]
            g = sg[e] * _expert_dot(O, wg, e, n_ff, n_embd, qx)
            u = _expert_dot(O, wu, e, n_ff, n_embd, qx)
            _check(glu[t, k], u * (g / (1.0 + np.exp(-g))), O, f"glu t={t} k={k}")
            qg = O.quantize_q8_1(glu[t, k].reshape(1, n_ff))
            _check(part[t, k], _expert_dot(O, wd, e, n_embd, n_ff, qg), O, f"part t={t} k={k}")
        ref = (part[t].astype(np.float64) * wts[t].astype(np.float64)[:, None]).sum(0) + r[t]
        np.testing.assert_allclose(o[t], ref, rtol=1e-5, atol=1e-5)
    assert fr.device_status() == 0


def test_moe_ffn_tiled_matches_ggml_layout(fr, O, dev):
    """The tiled layer and the ggml-layout layer agree (same routing; expert
    outputs within the matvec tolerance of each other)."""
    import torch
    n_embd, n_ff, E, n_used, T = 2048, 768, 128, 8, 16
    wg, wu, wd, wr, (wg_t, wu_t, wd_t) = _moe_weights(fr, dev, E, n_embd, n_ff, 970)
    x = _t(fr.synth_normal(975, T * n_embd).reshape(T, n_embd), dev)
    wrd = _t(wr, dev)
    a, ca = fr.moe_ffn_tiled(x, wrd, wg_t, wu_t, wd_t, n_embd, n_ff, E, n_used, check=True)
    b, cb = fr.moe_ffn(x, wrd, _t(wg, dev), _t(wu, dev), _t(wd, dev), n_embd, n_ff, E, n_used, check=True)
    torch.cuda.synchronize()
    assert torch.equal(ca["ids"], cb["ids"])
    _check(ca["glu"].cpu().numpy(), cb["glu"].cpu().numpy().astype(np.float64), O, "glu")
    assert O.norm_err(a.cpu().numpy(), b.cpu().numpy().astype(np.float64)) <= 2e-3


def test_moe_ffn_tiled_graph_replay(fr, dev):
    """Captured once, replayed on new inputs (the window count comes from the
    device routing), equal to eager calls on the same inputs."""
    import torch
    n_embd, n_ff, E, n_used, T = 2048, 768, 128, 8, 64
    _, _, _, wr, (wg_t, wu_t, wd_t) = _moe_weights(fr, dev, E, n_embd, n_ff, 980)
    wrd = _t(wr, dev)
    xs = [_t(fr.synth_normal(985 + i, T * n_embd).reshape(T, n_embd), dev) for i in range(3)]
    eager = [fr.moe_ffn_tiled(x, wrd, wg_t, wu_t, wd_t, n_embd, n_ff, E, n_used) for x in xs]
    xin = xs[0].clone()
    out = torch.empty((T, n_embd), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fr.moe_ffn_tiled(xin, wrd, wg_t, wu_t, wd_t, n_embd, n_ff, E, n_used, out=out, stream=s)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            fr.moe_ffn_tiled(xin, wrd, wg_t, wu_t, wd_t, n_embd, n_ff, E, n_used, out=out, stream=s)
    torch.cuda.synchronize()
    for i in (2, 0, 1, 1):
        xin.copy_(xs[i])
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager[i]), f"replay {i}"
    del g
    assert fr.device_status() == 0


def test_moe_tiled_rejects_bad_shapes(fr, dev):
    import torch
    L = fr.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    p = fr._ptr(buf)
    s = fr._stream()
    # N % 128, K % 256, per-slot rows not evenly spaced
    assert L.fr_mul_mat_id_tiled(p, 4, 100, 256, p, 0, 256, p, 2, p, 100, 200, 2, 2, s) == -1
    assert L.fr_mul_mat_id_tiled(p, 4, 128, 320, p, 0, 320, p, 2, p, 128, 256, 2, 2, s) == -1
    assert L.fr_mul_mat_id_tiled(p, 4, 128, 256, p, 256, 1024, p, 2, p, 128, 256, 2, 2, s) == -1
    assert L.fr_moe_ffn_tiled(p, p, p, p, p, None, None, None, None, p, 1, 2048, 700, 128, 8, CLAMP,
                              None, None, None, None, s) == -1
    assert fr.device_status() == 0
