"""Parity of the FP4 tensor-core matvec on tile-major weights (fr_nvfp4_tile,
fr_gemv_tiled, fr_gemv_tiled_swiglu, fr_ffn_tiled) through the C-ABI on a
B200: the repack bit-exact against the CPU restatement, the matvecs against
the fp64 oracle with the dense tolerances (max rel err 1e-3 against
max(|ref|, 1% rms), normwise 1e-5, zero values outside the reference's gate,
all finite)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3
NTOL = 1e-5


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


@pytest.mark.parametrize("N,K", [(130, 512), (64, 320), (14336, 4096), (300, 768)])
def test_tile_bit_exact(fr, O, dev, N, K):
    import torch
    w = fr.synth_nvfp4(300 + N, N, K)
    w.reshape(N, K // 64, 36)[: min(N, 9), 1 % (K // 64), 2] = 0xFF
    wt = fr.tile_nvfp4(_t(w, dev), N, K)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(wt.cpu().numpy(), O.tile_nvfp4(w, N, K))


CASES = [
    (4096, 4096, 1), (14336, 4096, 1), (4096, 14336, 1), (300, 256, 1), (130, 768, 2), (1000, 2048, 3),
    (4096, 4096, 8), (517, 4096, 13), (256, 1024, 21), (200, 512, 22), (128, 4096, 64),
]


@pytest.mark.parametrize("N,K,T", CASES)
def test_gemv_tiled_matches_oracle(fr, O, dev, N, K, T):
    import torch
    w = fr.synth_nvfp4(1000 + N, N, K)
    x = fr.synth_normal(2000 + K + T, T * K).reshape(T, K)
    q = O.quantize_q8_1(x)
    wt = fr.tile_nvfp4(_t(w, dev), N, K)
    y = fr.gemv_tiled(wt, N, K, q8=_t(q, dev))
    yx = fr.gemv_tiled(wt, N, K, x=_t(x, dev))
    torch.cuda.synchronize()
    ref = O.gemv_q8_1(w, q, N, K, nthreads=8)
    _check(y.cpu().numpy(), ref, O, f"tiled gemv N={N} K={K} T={T}")
    assert torch.equal(y, yx), "f32 input quantizes exactly like q8_1 input"
    assert fr.device_status() == 0


def test_gemv_tiled_scale_residual_special_blocks(fr, O, dev):
    import torch
    N, K, T = 300, 1024, 3
    w = fr.synth_nvfp4(91, N, K)
    blocks = w.reshape(N, K // 64, 36)
    blocks[0:7, 0, 0] = 0x7F
    blocks[7:15, 1, 2] = 0xFF
    blocks[15:40, 2, 1] |= 0x80
    x = fr.synth_normal(92, T * K).reshape(T, K)
    x[0, 0:32] = 0.0
    x[1, 64:96] *= 1e-6
    x[2, 128:160] *= 1e3
    r = fr.synth_normal(93, T * N).reshape(T, N)
    q = O.quantize_q8_1(x)
    s = torch.tensor([0.37], dtype=torch.float32, device=dev)
    wt = fr.tile_nvfp4(_t(w, dev), N, K)
    y = fr.gemv_tiled(wt, N, K, x=_t(x, dev), scale=s, resid=_t(r, dev))
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), O.gemv_q8_1(w, q, N, K, scale=0.37) + r, O, "scale/resid/special")


@pytest.mark.parametrize("N,K,T", [(14336, 4096, 1), (768, 2048, 2), (1000, 512, 8)])
def test_swiglu_tiled(fr, O, dev, N, K, T):
    import torch
    wg = fr.synth_nvfp4(61, N, K)
    wu = fr.synth_nvfp4(62, N, K)
    x = fr.synth_normal(63, T * K).reshape(T, K)
    q = O.quantize_q8_1(x)
    y = fr.gemv_tiled_swiglu(fr.tile_nvfp4(_t(wg, dev), N, K), fr.tile_nvfp4(_t(wu, dev), N, K), N, K,
                             q8=_t(q, dev))
    torch.cuda.synchronize()
    g = O.gemv_q8_1(wg, q, N, K, nthreads=8)
    u = O.gemv_q8_1(wu, q, N, K, nthreads=8)
    _check(y.cpu().numpy(), u * (g / (1.0 + np.exp(-g))), O, "tiled swiglu")


@pytest.mark.parametrize("T", [1, 8])
def test_ffn_tiled_stagewise(fr, O, dev, T):
    import torch
    n_embd, n_ff = 1024, 2816
    wg = fr.synth_nvfp4(81, n_ff, n_embd)
    wu = fr.synth_nvfp4(82, n_ff, n_embd)
    wd = fr.synth_nvfp4(83, n_embd, n_ff)
    x = fr.synth_normal(84, T * n_embd).reshape(T, n_embd)
    r = fr.synth_normal(85, T * n_embd).reshape(T, n_embd)
    glu = torch.empty((T, n_ff), dtype=torch.float32, device=dev)
    tl = lambda w, N, K: fr.tile_nvfp4(_t(w, dev), N, K)  # noqa: E731
    out = fr.ffn_tiled(_t(x, dev), tl(wg, n_ff, n_embd), tl(wu, n_ff, n_embd), tl(wd, n_embd, n_ff), n_embd, n_ff,
                       resid=_t(r, dev), chk_glu=glu)
    torch.cuda.synchronize()
    q = O.quantize_q8_1(x)
    g = O.gemv_q8_1(wg, q, n_ff, n_embd, nthreads=8)
    u = O.gemv_q8_1(wu, q, n_ff, n_embd, nthreads=8)
    _check(glu.cpu().numpy(), u * (g / (1.0 + np.exp(-g))), O, "tiled ffn glu")
    ref = O.gemv_q8_1(wd, O.quantize_q8_1(glu.cpu().numpy()), n_embd, n_ff, nthreads=8) + r
    _check(out.cpu().numpy(), ref, O, "tiled ffn out")


def test_tiled_rejects_bad_shapes(fr, dev):
    import torch
    L = fr.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    p = fr._ptr(buf)
    s = fr._stream()
    assert L.fr_gemv_tiled(p, 128, 320, p, 320, None, 0, None, None, 0, p, 128, 1, s) == -1   # K % 256
    assert L.fr_gemv_tiled(p, 128, 256, p, 256, p, 8, None, None, 0, p, 128, 1, s) == -1      # both inputs
    assert L.fr_nvfp4_tile(p, 36, 4, 100, p, s) == -1                                        # K % 64
