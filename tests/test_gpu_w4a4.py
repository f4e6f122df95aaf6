"""Parity of the W4A4 (Thor) launch interface on B200: quantize_act_f32 and
repack_weight bit-exact against the oracle, gemm_f32out (tcgen05
kind::mxf4nvf4, TMEM accumulator) within max rel err 1e-3 of the fp64 product
of the dequantized operands (the reference's W4A4 GEMM semantics,
src/fr_gemm_f32out.cu:122-187)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3      # max |d| / max(|ref|, 1% rms(ref))
NTOL = 1e-5      # ||d|| / ||ref||
E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _e4m3_table(O):
    L = O.lib()
    return np.array([L.or_e4m3_to_f32(c) for c in range(256)], np.float64)


def _sf_offsets(rows, K):
    r = np.arange(rows)[:, None]
    k = np.arange(0, K, 16)[None, :]
    kb = (K + 63) >> 6
    rr = r & 127
    return (r >> 7) * kb * 512 + (k >> 6) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + ((k & 63) >> 4)


def dequant(packed, sf, rows, K, O):
    codes = np.empty((rows, K), np.uint8)
    codes[:, 0::2] = packed & 0xF
    codes[:, 1::2] = packed >> 4
    vals = E2M1[codes]
    scale = _e4m3_table(O)[sf[_sf_offsets(rows, K)]]
    return vals * np.repeat(scale, 16, axis=1)


def _check(mine, ref, O, what):
    mine = np.asarray(mine, np.float64)
    assert np.all(np.isfinite(mine)), what
    err = O.rel_err(mine, ref)
    assert err <= RTOL, f"{what}: max rel err {err:.3e}"
    assert O.norm_err(mine, ref) <= NTOL, what


@pytest.mark.parametrize("M,K", [(1, 64), (3, 48), (130, 4096), (512, 14336), (7, 960)])
def test_quantize_act_bit_exact(fr, O, dev, M, K):
    import torch
    x = fr.synth_normal(700 + M + K, M * K).reshape(M, K)
    x[0, :16] = 0.0
    if K >= 64:
        x[0, 16:32] *= 1e-8
        x[0, 32:48] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2, np.float32)   # boundaries
    packed, sf = fr.quantize_act_f32(_t(x, dev))
    torch.cuda.synchronize()
    rp, rsf = O.quantize_act_f32(x)
    np.testing.assert_array_equal(packed.cpu().numpy(), rp)
    got_sf = sf.cpu().numpy()
    offs = _sf_offsets(M, K)
    np.testing.assert_array_equal(got_sf[offs], rsf[offs])


@pytest.mark.parametrize("N,K", [(16, 64), (300, 4096), (14336, 4096), (128, 768)])
def test_repack_bit_exact(fr, O, dev, N, K):
    import torch
    w = fr.synth_nvfp4(800 + N, N, K)
    packed, sf = fr.repack_weight(_t(w, dev), N, K)
    torch.cuda.synchronize()
    rp, rsf = O.repack_weight(w, N, K)
    np.testing.assert_array_equal(packed.cpu().numpy(), rp)
    np.testing.assert_array_equal(sf.cpu().numpy(), rsf)


def _gemm_case(fr, O, dev, M, N, K, alpha=1.0, row_sample=None):
    import torch
    x = fr.synth_normal(900 + M, M * K).reshape(M, K)
    w = fr.synth_nvfp4(901 + N, N, K)
    A, SFA = fr.quantize_act_f32(_t(x, dev))
    B, SFB = fr.repack_weight(_t(w, dev), N, K)
    D = fr.gemm_f32out(A, SFA, B, SFB, M, N, K, alpha=alpha)
    torch.cuda.synchronize()
    a = dequant(A.cpu().numpy(), SFA.cpu().numpy(), M, K, O)
    b = dequant(B.cpu().numpy(), SFB.cpu().numpy(), N, K, O)
    rows = np.arange(M) if row_sample is None else np.sort(
        np.random.default_rng(0).choice(M, row_sample, replace=False))
    ref = alpha * (a[rows] @ b.T)
    _check(D.cpu().numpy()[rows], ref, O, f"gemm M={M} N={N} K={K}")
    return D


@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (1, 16, 64), (200, 144, 320), (256, 256, 1024),
                                   (512, 1024, 4096), (64, 4096, 14336)])
def test_gemm_f32out(fr, O, dev, M, N, K):
    _gemm_case(fr, O, dev, M, N, K)
    assert fr.device_status() == 0


def test_gemm_alpha(fr, O, dev):
    _gemm_case(fr, O, dev, 130, 48, 512, alpha=0.37)


def test_gemm_config4_prefill(fr, O, dev):
    """Config 4: 512-token ubatch x 14336x4096, and 4x512 = 2048 rows x 4096x14336."""
    _gemm_case(fr, O, dev, 512, 14336, 4096, row_sample=96)
    _gemm_case(fr, O, dev, 2048, 4096, 14336, row_sample=64)


def test_gemm_matches_oracle_semantics(fr, O, dev):
    """Same numbers through the oracle's own W4A4 chain on a small case."""
    import torch
    M, N, K = 5, 32, 256
    x = fr.synth_normal(990, M * K).reshape(M, K)
    w = fr.synth_nvfp4(991, N, K)
    A, SFA = fr.quantize_act_f32(_t(x, dev))
    B, SFB = fr.repack_weight(_t(w, dev), N, K)
    D = fr.gemm_f32out(A, SFA, B, SFB, M, N, K)
    torch.cuda.synchronize()
    ra, rsa = O.quantize_act_f32(x)
    rb, rsb = O.repack_weight(w, N, K)
    ref = O.gemm_f32out(ra, rsa, rb, rsb, M, N, K)
    _check(D.cpu().numpy(), ref, O, "oracle chain")


def test_gemm_rejects_bad_shapes(fr, dev):
    import torch
    L = fr.lib()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    p = fr._ptr(buf)
    assert L.fr_gemm_f32out(p, p, p, p, p, 128, 100, 256, 1.0, False, fr._stream()) == -1   # N % 16
    assert L.fr_gemm_f32out(p, p, p, p, p, 128, 128, 96, 1.0, False, fr._stream()) == -1    # K % 64


@pytest.mark.parametrize("M,N,K", [(300, 16400, 512), (1000, 16384, 256), (256, 16384, 4096), (512, 4096, 14336),
                                   (300, 4096, 1024)])
def test_gemm_pair_tiles(fr, O, dev, M, N, K):
    """Shapes that take the SM-pair kernel (256 x 256 tiles on clusters of
    two CTAs, tcgen05 cta_group::2): rows and columns past the last full tile
    (M = 300, N = 16400), several tiles per cluster (M = 1000), one row of
    tiles (M = 256), and two K halves per tile handed over between clusters
    (N = 4096: 32 tiles on 74 SM pairs); sampled rows against the fp64
    products."""
    _gemm_case(fr, O, dev, M, N, K, row_sample=96)
    assert fr.device_status() == 0


def test_gemm_pair_tiles_deterministic_and_graph_replay(fr, dev):
    """The SM-pair kernel gives the same bits eager and replayed from a CUDA
    graph (static tile order, no cross-CTA reduction)."""
    import torch
    M, N, K = 512, 14336, 4096
    A, SFA = fr.quantize_act_f32(_t(fr.synth_normal(0x5EED4A00, M * K).reshape(M, K), dev))
    B, SFB = fr.repack_weight(_t(fr.synth_nvfp4(0x5EED4A01, N, K), dev), N, K)
    d0 = fr.gemm_f32out(A, SFA, B, SFB, M, N, K)
    s = torch.cuda.Stream(dev)
    out = torch.empty_like(d0)
    with torch.cuda.stream(s):
        fr.gemm_f32out(A, SFA, B, SFB, M, N, K, out=out, stream=s)
    s.synchronize()
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=s):
        fr.gemm_f32out(A, SFA, B, SFB, M, N, K, out=out, stream=s)
    for _ in range(3):
        out.zero_()
        gph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, d0)
    assert fr.device_status() == 0


@pytest.mark.parametrize("M,n_ff,K", [(512, 14336, 4096), (100, 768, 2048), (7, 208, 320)])
def test_gemm_swiglu_fused_epilogue(fr, O, dev, M, n_ff, K):
    """The prefill FFN's gate/up GEMM with the SwiGLU in its epilogue
    (fr_gemm_swiglu_f32out on fr_repack_weight_pair_interleaved weights):
    silu(g) * u against the fp64 products of the dequantized operands, and
    against two plain GEMMs, within the GEMM tolerance (max rel err 1e-3
    against max(|ref|, 1% rms), normwise 1e-5)."""
    import torch
    x = fr.synth_normal(0x5EED4800 + M, M * K).reshape(M, K)
    wg = fr.synth_nvfp4(0x5EED4810 + n_ff, n_ff, K)
    wu = fr.synth_nvfp4(0x5EED4820 + n_ff, n_ff, K)
    A, SFA = fr.quantize_act_f32(_t(x, dev))
    Bp, SFBp = fr.repack_weight_pair_interleaved(_t(wg, dev), _t(wu, dev), n_ff, K)
    out = fr.gemm_swiglu_f32out(A, SFA, Bp, SFBp, M, n_ff, K, alpha=0.75)
    Bg, SFBg = fr.repack_weight(_t(wg, dev), n_ff, K)
    Bu, SFBu = fr.repack_weight(_t(wu, dev), n_ff, K)
    g = fr.gemm_f32out(A, SFA, Bg, SFBg, M, n_ff, K, alpha=0.75)
    u = fr.gemm_f32out(A, SFA, Bu, SFBu, M, n_ff, K, alpha=0.75)
    torch.cuda.synchronize()
    two = (u * (g / (1.0 + torch.exp(-g)))).cpu().numpy()
    _check(out.cpu().numpy(), two, O, "fused vs two GEMMs")
    rows = np.arange(M) if M <= 128 else np.sort(np.random.default_rng(1).choice(M, 64, replace=False))
    a = dequant(A.cpu().numpy(), SFA.cpu().numpy(), M, K, O)[rows]
    gd = 0.75 * (a @ dequant(Bg.cpu().numpy(), SFBg.cpu().numpy(), n_ff, K, O).T)
    ud = 0.75 * (a @ dequant(Bu.cpu().numpy(), SFBu.cpu().numpy(), n_ff, K, O).T)
    _check(out.cpu().numpy()[rows], ud * (gd / (1.0 + np.exp(-gd))), O, "fused vs fp64")
    assert fr.device_status() == 0


def test_gemm_deterministic_and_graph_replay(fr, dev):
    """Stream-K partial tiles are added in CTA order: the same inputs give the
    same bits on every launch, eager or replayed from a CUDA graph."""
    import torch
    M, N, K = 300, 4096, 14336
    A, SFA = fr.quantize_act_f32(_t(fr.synth_normal(0x5EED4900, M * K).reshape(M, K), dev))
    B, SFB = fr.repack_weight(_t(fr.synth_nvfp4(0x5EED4901, N, K), dev), N, K)
    d0 = fr.gemm_f32out(A, SFA, B, SFB, M, N, K)
    d1 = fr.gemm_f32out(A, SFA, B, SFB, M, N, K)
    s = torch.cuda.Stream(dev)
    out = torch.empty_like(d0)
    with torch.cuda.stream(s):
        fr.gemm_f32out(A, SFA, B, SFB, M, N, K, out=out, stream=s)
    s.synchronize()
    gph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gph, stream=s):
        fr.gemm_f32out(A, SFA, B, SFB, M, N, K, out=out, stream=s)
    for _ in range(3):
        out.zero_()
        gph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, d0)
    assert torch.equal(d0, d1)
    assert fr.device_status() == 0
