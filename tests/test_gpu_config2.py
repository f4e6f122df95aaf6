"""Parity at the benchmark's full sizes: configs[1] (gate/up 14336x4096, down
4096x14336) at T = 64 and 128 tokens, and configs[3] (a 512-token ubatch)
through the ggml_mul_mat op surface -- on every dense matvec kernel (dp4a,
f16 tensor cores on ggml's layout, FP4 tensor cores on ggml's layout and on
tile-major weights).

The device computes every output; the fp64 oracle checks a sample of rows
(the first and last 128 and 256 spread between them, all tokens) with the
dense tolerances: max rel err <= 1e-3 against max(|ref|, 1% rms(ref)),
normwise <= 1e-5, zero values outside the reference's gate (abs > 1e-4 and
rel > 2e-3), all finite.  FFN stages hand on the device's own intermediates
(as the reference's FRT_B_HREF check mode does), and the q8_1 of the device
GLU is checked bit for bit on every token.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3
NTOL = 1e-5
NE, NF = 4096, 14336


@pytest.fixture(params=[1, 2, 3], ids=["dp4a", "tc-f16", "tc-fp4"])
def ggml_path(request, fr):
    prev = fr.set_matvec_path(request.param)
    yield request.param
    fr.set_matvec_path(prev)


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _rows(N, seed):
    rng = np.random.default_rng(seed)
    mid = rng.choice(np.arange(128, N - 128), 256, replace=False)
    return np.unique(np.concatenate([np.arange(128), np.sort(mid), np.arange(N - 128, N)]))


def _check(mine, ref, O, what):
    mine = np.asarray(mine, np.float64)
    assert np.all(np.isfinite(mine)), what
    err = O.rel_err(mine, ref)
    assert err <= RTOL, f"{what}: max rel err {err:.3e}"
    nerr = O.norm_err(mine, ref)
    assert nerr <= NTOL, f"{what}: norm err {nerr:.3e}"
    assert O.ref_gate_bad(mine, ref) == 0, what


@pytest.fixture(scope="module")
def weights(fr):
    return (fr.synth_nvfp4(0x5EED0001, NF, NE), fr.synth_nvfp4(0x5EED0002, NF, NE),
            fr.synth_nvfp4(0x5EED0003, NE, NF))


@pytest.mark.parametrize("T", [64, 128])
@pytest.mark.parametrize("which", ["gate", "down"])
def test_config2_gemv_ggml_layout(fr, O, dev, weights, ggml_path, which, T):
    import torch
    w = weights[0] if which == "gate" else weights[2]
    N, K = (NF, NE) if which == "gate" else (NE, NF)
    x = fr.synth_normal(0x5EED0010 + T, T * K).reshape(T, K)
    q = O.quantize_q8_1(x)
    y = fr.gemv_q8_1(_t(w, dev), _t(q, dev), N, K, T)
    torch.cuda.synchronize()
    rows = _rows(N, T)
    ref = O.gemv_q8_1(w[rows], q, len(rows), K, nthreads=8)
    _check(y.cpu().numpy()[:, rows], ref, O, f"{which} T={T} path {ggml_path}")
    assert fr.device_status() == 0


@pytest.mark.parametrize("T", [64, 128])
def test_config2_ffn_ggml_layout_stagewise(fr, O, dev, weights, ggml_path, T):
    """The dense FFN at configs[1] sizes through fr_ffn_nvfp4 (the path the
    benchmark's T=64 line runs on ggml's layout)."""
    import torch
    wg, wu, wd = weights
    x = fr.synth_normal(0x5EED0020 + T, T * NE).reshape(T, NE)
    glu = torch.empty((T, NF), dtype=torch.float32, device=dev)
    gq8 = torch.empty((T, NF // 32 * 36), dtype=torch.uint8, device=dev)
    out = fr.ffn(_t(x, dev), _t(wg, dev), _t(wu, dev), _t(wd, dev), NE, NF, chk_glu=glu, chk_glu_q8=gq8)
    torch.cuda.synchronize()
    q = O.quantize_q8_1(x)
    cols = _rows(NF, 2 * T)
    g = O.gemv_q8_1(wg[cols], q, len(cols), NE, nthreads=8)
    u = O.gemv_q8_1(wu[cols], q, len(cols), NE, nthreads=8)
    dglu = glu.cpu().numpy()
    _check(dglu[:, cols], u * (g / (1.0 + np.exp(-g))), O, f"ffn glu T={T}")
    dq = gq8.cpu().numpy()
    np.testing.assert_array_equal(dq, O.quantize_q8_1(dglu))
    rows = _rows(NE, 3 * T)
    _check(out.cpu().numpy()[:, rows], O.gemv_q8_1(wd[rows], dq, len(rows), NF, nthreads=8), O,
           f"ffn out T={T}")
    assert fr.device_status() == 0


@pytest.mark.parametrize("T", [64, 128])
def test_config2_tiled(fr, O, dev, weights, T):
    """Tile-major weights (FP4 tensor cores): the gate/up SwiGLU pair and the
    down matvec at configs[1] sizes."""
    import torch
    wg, wu, wd = weights
    wgt, wut = fr.tile_nvfp4(_t(wg, dev), NF, NE), fr.tile_nvfp4(_t(wu, dev), NF, NE)
    wdt = fr.tile_nvfp4(_t(wd, dev), NE, NF)
    x = fr.synth_normal(0x5EED0030 + T, T * NE).reshape(T, NE)
    q = O.quantize_q8_1(x)
    glu = fr.gemv_tiled_swiglu(wgt, wut, NF, NE, q8=_t(q, dev))
    torch.cuda.synchronize()
    dglu = glu.cpu().numpy()
    cols = _rows(NF, 4 * T)
    g = O.gemv_q8_1(wg[cols], q, len(cols), NE, nthreads=8)
    u = O.gemv_q8_1(wu[cols], q, len(cols), NE, nthreads=8)
    _check(dglu[:, cols], u * (g / (1.0 + np.exp(-g))), O, f"tiled swiglu T={T}")
    dq = O.quantize_q8_1(dglu)
    y = fr.gemv_tiled(wdt, NE, NF, q8=_t(dq, dev))
    torch.cuda.synchronize()
    rows = _rows(NE, 5 * T)
    _check(y.cpu().numpy()[:, rows], O.gemv_q8_1(wd[rows], dq, len(rows), NF, nthreads=8), O, f"tiled down T={T}")
    assert fr.device_status() == 0


@pytest.mark.parametrize("N,K", [(NF, NE), (NE, NF)])
def test_config4_mul_mat_512(fr, O, dev, weights, ggml_path, N, K):
    """ggml_mul_mat with a 512-token ubatch (configs[3]'s shapes) with q8_1
    activation semantics, on sampled rows."""
    import torch
    w = weights[0] if N == NF else weights[2]
    T = 512
    x = fr.synth_normal(0x5EED0040 + K, T * K).reshape(T, K)
    y = fr.mul_mat(_t(w, dev), _t(x, dev), N, K)
    torch.cuda.synchronize()
    rows = _rows(N, K)[::4]
    ref = O.gemv_q8_1(w[rows], O.quantize_q8_1(x), len(rows), K, nthreads=8)
    _check(y.cpu().numpy()[:, rows], ref, O, f"mul_mat T=512 N={N} K={K} path {ggml_path}")
    assert fr.device_status() == 0
