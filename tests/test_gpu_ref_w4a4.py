"""Pins of the W4A4 (Thor) path against the reference's own kernels.

oracle/_ref/libfrref.so is the reference's src/fr_quant_act.cu,
src/fr_repack.cu and src/fr_gemm_f32out.cu compiled unmodified for sm_100a
against the image's CUTLASS 4.5 headers (oracle/ref.mk).  On the same seeded
inputs:
  * fr_quantize_act_f32 and the CPU oracle's restatement must equal the
    reference's quantize_act_f32 byte for byte (packed E2M1 and every
    scale-factor byte the GEMM reads -- which pins the scale-factor atom
    layout, not only a bijection);
  * fr_repack_weight and the oracle must equal repack_weight byte for byte
    (packed codes and the whole scale buffer);
  * fr_gemm_f32out must agree with the reference's CUTLASS tcgen05 GEMM to
    max rel err 1e-3 (against max(|ref|, 1% rms), normwise 1e-5) at the
    prefill shapes of configs[3] (512 x 14336 x 4096 and 4 x 512 = 2048 rows
    x 4096 x 14336) and at small and ragged shapes.
Skipped when the reference build is absent (it needs the reference sources).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3
NTOL = 1e-5


@pytest.fixture(scope="module")
def R(O):
    L = O.ref_lib()
    if L is None:
        pytest.skip("oracle/_ref/libfrref.so not built (make -f oracle/ref.mk needs the reference sources)")
    return L


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _sf_valid(rows, K):
    """Offsets of the scale bytes of rows < `rows`, K columns, in the atom
    layout (the bytes a GEMM of those rows reads)."""
    r = np.arange(rows)[:, None]
    k = np.arange(0, K, 16)[None, :]
    kb = (K + 63) >> 6
    rr = r & 127
    return ((r >> 7) * kb * 512 + (k >> 6) * 512 + (rr & 31) * 16 + (rr >> 5) * 4 + ((k & 63) >> 4)).reshape(-1)


def _ref_quant(R, fr, x):
    import torch
    M, K = x.shape
    packed = torch.zeros((M, K // 2), dtype=torch.uint8, device=x.device)
    sf = torch.zeros(fr.sf_bytes(M, K), dtype=torch.uint8, device=x.device)
    assert R.frref_quantize_act_f32(fr._ptr(x), fr._ptr(packed), fr._ptr(sf), M, K, fr._stream()) == 0
    return packed, sf


def _ref_repack(R, fr, w, N, K):
    import torch
    packed = torch.zeros((N, K // 2), dtype=torch.uint8, device=w.device)
    sf = torch.zeros(fr.sf_bytes(N, K), dtype=torch.uint8, device=w.device)
    assert R.frref_repack_weight(fr._ptr(w), fr._ptr(packed), fr._ptr(sf), N, K, fr._stream()) == 0
    return packed, sf


def test_sf_bytes_agree(R, fr):
    for rows, K in ((1, 64), (130, 4096), (512, 14336), (14336, 4096), (7, 960)):
        assert R.frref_sf_bytes(rows, K) == fr.sf_bytes(rows, K)


@pytest.mark.parametrize("M,K", [(1, 64), (3, 48), (130, 4096), (512, 4096), (512, 14336), (7, 960)])
def test_quantize_act_equals_reference(R, fr, O, dev, M, K):
    import torch
    x = fr.synth_normal(0x5EED4000 + M + K, M * K).reshape(M, K)
    x[0, :16] = 0.0
    if K >= 64:
        x[0, 16:32] *= 1e-8
        x[0, 32:48] = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0] * 2, np.float32)
    xd = _t(x, dev)
    rp, rsf = _ref_quant(R, fr, xd)
    mp, msf = fr.quantize_act_f32(xd)
    torch.cuda.synchronize()
    rp, rsf, mp, msf = rp.cpu().numpy(), rsf.cpu().numpy(), mp.cpu().numpy(), msf.cpu().numpy()
    offs = _sf_valid(M, K)
    np.testing.assert_array_equal(mp, rp)
    np.testing.assert_array_equal(msf[offs], rsf[offs])
    op, osf = O.quantize_act_f32(x)
    np.testing.assert_array_equal(op, rp)
    np.testing.assert_array_equal(osf[offs], rsf[offs])


@pytest.mark.parametrize("N,K", [(16, 64), (300, 4096), (14336, 4096), (4096, 14336), (128, 768)])
def test_repack_equals_reference(R, fr, O, dev, N, K):
    import torch
    w = fr.synth_nvfp4(0x5EED4100 + N, N, K)
    w.reshape(N, K // 64, 36)[: min(N, 9), 0, 1] = 0xFF       # scale bytes ggml reads specially
    w.reshape(N, K // 64, 36)[: min(N, 5), 0, 2] |= 0x80
    wd = _t(w, dev)
    rp, rsf = _ref_repack(R, fr, wd, N, K)
    mp, msf = fr.repack_weight(wd, N, K)
    torch.cuda.synchronize()
    rp, rsf = rp.cpu().numpy(), rsf.cpu().numpy()
    np.testing.assert_array_equal(mp.cpu().numpy(), rp)
    np.testing.assert_array_equal(msf.cpu().numpy(), rsf)
    op, osf = O.repack_weight(w, N, K)
    np.testing.assert_array_equal(op, rp)
    np.testing.assert_array_equal(osf, rsf)


@pytest.mark.parametrize("M,N,K", [(512, 14336, 4096), (2048, 4096, 14336), (128, 128, 256), (100, 4096, 4096),
                                   (1, 16, 64), (200, 144, 320), (300, 1024, 2048)])
def test_gemm_matches_reference_cutlass(R, fr, O, dev, M, N, K):
    import torch
    x = fr.synth_normal(0x5EED4200 + M, M * K).reshape(M, K)
    w = fr.synth_nvfp4(0x5EED4300 + N, N, K)
    A, SFA = fr.quantize_act_f32(_t(x, dev))
    B, SFB = fr.repack_weight(_t(w, dev), N, K)
    D = fr.gemm_f32out(A, SFA, B, SFB, M, N, K, alpha=0.5)
    Dr = torch.empty((M, N), dtype=torch.float32, device=dev)
    assert R.frref_gemm_f32out(fr._ptr(A), fr._ptr(SFA), fr._ptr(B), fr._ptr(SFB), fr._ptr(Dr), M, N, K, 0.5, 0,
                               fr._stream()) == 0
    torch.cuda.synchronize()
    mine, ref = D.cpu().numpy().astype(np.float64), Dr.cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(mine)) and np.all(np.isfinite(ref))
    err = O.rel_err(mine, ref)
    assert err <= RTOL, f"M={M} N={N} K={K}: max rel err {err:.3e} against the reference GEMM"
    assert O.norm_err(mine, ref) <= NTOL
    assert fr.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(512, 14336, 4096), (512, 4096, 14336), (2048, 4096, 14336)])
def test_gemm_time_beside_reference(R, fr, dev, M, N, K, capsys):
    """Device time of fr_gemm_f32out and of the reference's CUTLASS GEMM on the
    same operands (CUDA events, 20 launches after 5 warm-up ones, weights
    rotating over 4 copies).  Reported, not asserted: the figures go into the
    performance notes."""
    import torch
    x = fr.synth_normal(0x5EED4400 + M, M * K).reshape(M, K)
    A, SFA = fr.quantize_act_f32(_t(x, dev))
    Bs = [fr.repack_weight(_t(fr.synth_nvfp4(0x5EED4500 + c + N, N, K), dev), N, K) for c in range(4)]
    D = torch.empty((M, N), dtype=torch.float32, device=dev)
    s = torch.cuda.current_stream()

    def ours(i):
        B, SFB = Bs[i % 4]
        fr.gemm_f32out(A, SFA, B, SFB, M, N, K, out=D)

    def ref(i):
        B, SFB = Bs[i % 4]
        assert R.frref_gemm_f32out(fr._ptr(A), fr._ptr(SFA), fr._ptr(B), fr._ptr(SFB), fr._ptr(D), M, N, K, 1.0, 0,
                                   fr._stream()) == 0

    res = {}
    for name, fn in (("ours", ours), ("reference", ref)):
        for i in range(5):
            fn(i)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(s)
        for i in range(20):
            fn(i)
        e1.record(s)
        e1.synchronize()
        res[name] = e0.elapsed_time(e1) / 20 * 1e3
    tf = {k: 2.0 * M * N * K / (v * 1e-6) / 1e12 for k, v in res.items()}
    with capsys.disabled():
        print(f"\n[gemm timing] M={M} N={N} K={K}: ours {res['ours']:.1f} us ({tf['ours']:.0f} TFLOP/s), "
              f"reference CUTLASS {res['reference']:.1f} us ({tf['reference']:.0f} TFLOP/s)")
    assert fr.device_status() == 0


@pytest.mark.parametrize("n_ff,K", [(14336, 4096), (200, 512), (64, 64)])
def test_pair_interleaved_repack_equals_reference(R, fr, dev, n_ff, K):
    """fr_repack_weight_pair_interleaved against the reference's
    repack_weight_pair_interleaved, byte for byte (packed and scales)."""
    import ctypes as C
    import torch
    if not hasattr(R, "frref_repack_weight_pair_interleaved"):
        pytest.skip("reference shim without the pair repack")
    R.frref_repack_weight_pair_interleaved.restype = C.c_int
    R.frref_repack_weight_pair_interleaved.argtypes = [C.c_void_p] * 4 + [C.c_int, C.c_int, C.c_void_p]
    g = _t(fr.synth_nvfp4(0x5EED4600 + n_ff, n_ff, K), dev)
    u = _t(fr.synth_nvfp4(0x5EED4700 + n_ff, n_ff, K), dev)
    rp = torch.zeros((2 * n_ff, K // 2), dtype=torch.uint8, device=dev)
    rsf = torch.zeros(fr.sf_bytes(2 * n_ff, K), dtype=torch.uint8, device=dev)
    assert R.frref_repack_weight_pair_interleaved(fr._ptr(g), fr._ptr(u), fr._ptr(rp), fr._ptr(rsf), n_ff, K,
                                                  fr._stream()) == 0
    mp, msf = fr.repack_weight_pair_interleaved(g, u, n_ff, K)
    torch.cuda.synchronize()
    assert torch.equal(mp, rp)
    assert torch.equal(msf, rsf)
