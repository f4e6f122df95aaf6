"""Parity of the dense hot path (quantize_q8_1, NVFP4 x q8_1 matvec, SwiGLU
pair, mul_mat, FFN) against the CPU oracle, through the C-ABI on a B200.

Tolerances (written here, as the reference's check mode states them):
  * q8_1 blocks: bit-exact (int8 values, f16 d and f16 sum);
  * matvec outputs: max rel err <= 1e-3 against the fp64 oracle, the
    relative error taken against max(|ref|, 1e-2 * rms(ref)) (values below 1%
    of the rms measure cancellation, not the kernel), normwise error <= 1e-5,
    and zero "bad" values under the reference's gate (abs > 1e-4 and rel >
    2e-3, src/fr_win_flint_batched.cuh:478-489);
  * no non-finite values.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3      # max |d| / max(|ref|, 1% rms(ref))
NTOL = 1e-5      # ||d|| / ||ref||


@pytest.fixture(params=[1, 2, 3], ids=["dp4a", "tc-f16", "tc-fp4"], autouse=True)
def matvec_path(request, fr):
    """Run every dense parity test on all three matvec kernels: dp4a, the
    tensor-core kernel on decoded f16 weights, the FP4 tensor-core kernel on
    the stored codes."""
    prev = fr.set_matvec_path(request.param)
    yield request.param
    fr.set_matvec_path(prev)


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


@pytest.mark.parametrize("T,K", [(1, 32), (1, 4096), (3, 2048), (64, 4096), (2, 14336), (5, 768)])
def test_quantize_q8_1_bit_exact(fr, O, dev, T, K):
    import torch
    x = fr.synth_normal(100 + T + K, T * K).reshape(T, K)
    x[0, :32] = 0.0                       # all-zero chunk: d = 0, q = 0
    if K >= 96:
        x[0, 32:64] *= 1e-20              # tiny chunk
        x[0, 64:96] = np.linspace(-127, 127, 32)   # exact integer ratios
    q = fr.quantize_q8_1(_t(x, dev))
    torch.cuda.synchronize()
    ref = O.quantize_q8_1(x)
    np.testing.assert_array_equal(q.cpu().numpy(), ref)


def test_quantize_q8_1_strided_rows(fr, O, dev):
    import torch
    T, K, ldx = 4, 1024, 1100
    x = fr.synth_normal(7, T * ldx).reshape(T, ldx)
    xd = _t(x, dev)
    out = torch.zeros((T, K // 32 * 36 + 72), dtype=torch.uint8, device=dev)
    fr.call("fr_quantize_q8_1", fr._ptr(xd), ldx, fr._ptr(out), out.stride(0) // 36, T, K, fr._stream())
    torch.cuda.synchronize()
    ref = O.quantize_q8_1(np.ascontiguousarray(x[:, :K]))
    np.testing.assert_array_equal(out.cpu().numpy()[:, :K // 32 * 36], ref)
    assert np.all(out.cpu().numpy()[:, K // 32 * 36:] == 0)


GEMV_CASES = [
    (4096, 4096, 1),      # config 1
    (14336, 4096, 1),     # config 2 gate/up
    (4096, 14336, 1),     # config 2 down
    (768, 2048, 1),       # MoE expert gate/up
    (2048, 768, 1),       # MoE expert down (K = 12 blocks)
    (130, 64, 1),         # one block per row, ragged N
    (333, 256, 2),
    (1000, 2048, 3),
    (517, 4096, 4),
    (129, 4096, 8),
    (77, 1024, 13),       # several token windows
    (5120, 2048, 64),     # configs[4] QKV at batch 64 (the f16 kernel unsplit along K)
    (2048, 4096, 64),     # configs[4] attention output at batch 64
]


@pytest.mark.parametrize("N,K,T", GEMV_CASES)
def test_gemv_q8_1_matches_oracle(fr, O, dev, N, K, T):
    import torch
    w = fr.synth_nvfp4(1000 + N, N, K)
    x = fr.synth_normal(2000 + K + T, T * K).reshape(T, K)
    q = O.quantize_q8_1(x)
    y = fr.gemv_q8_1(_t(w, dev), _t(q, dev), N, K, T)
    torch.cuda.synchronize()
    ref = O.gemv_q8_1(w, q, N, K, nthreads=8)
    _check(y.cpu().numpy(), ref, O, f"gemv N={N} K={K} T={T}")
    assert fr.device_status() == 0


@pytest.mark.parametrize("N,K,T", [(4096, 4096, 1), (300, 2048, 3), (64, 768, 8)])
def test_gemv_fused_quantize_is_identical(fr, dev, N, K, T):
    """Quantizing inside the matvec gives the same bits as the separate kernel."""
    import torch
    w = _t(fr.synth_nvfp4(31, N, K), dev)
    x = _t(fr.synth_normal(32, T * K).reshape(T, K), dev)
    y1 = fr.gemv_f32(w, x, N, K)
    q = fr.quantize_q8_1(x)
    y2 = fr.gemv_q8_1(w, q, N, K, T)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_gemv_scale_and_residual(fr, O, dev):
    import torch
    N, K, T = 500, 1024, 2
    w = fr.synth_nvfp4(41, N, K)
    x = fr.synth_normal(42, T * K).reshape(T, K)
    r = fr.synth_normal(43, T * N).reshape(T, N)
    q = O.quantize_q8_1(x)
    s = torch.tensor([0.37], dtype=torch.float32, device=dev)
    y = fr.gemv_q8_1(_t(w, dev), _t(q, dev), N, K, T, scale=s, resid=_t(r, dev))
    torch.cuda.synchronize()
    ref = O.gemv_q8_1(w, q, N, K, scale=0.37) + r
    _check(y.cpu().numpy(), ref, O, "scale+resid")


def test_gemv_strided_weight_rows(fr, O, dev):
    """w_ld larger than the packed row (a view into a wider tensor)."""
    import torch
    N, K, T = 200, 512, 1
    rb = K // 64 * 36
    w = fr.synth_nvfp4(51, N, K)
    wpad = np.zeros((N, rb + 16 * 3), np.uint8)
    wpad[:, :rb] = w
    x = fr.synth_normal(52, K).reshape(1, K)
    q = O.quantize_q8_1(x)
    wd = _t(wpad, dev)
    y = torch.empty((1, N), dtype=torch.float32, device=dev)
    qd = _t(q, dev)
    fr.call("fr_gemv_nvfp4_q8_1", fr._ptr(wd), wpad.shape[1], fr._ptr(qd), K // 32, None, None, 0, fr._ptr(y), N,
            N, K, T, fr._stream())
    torch.cuda.synchronize()
    _check(y.cpu().numpy(), O.gemv_q8_1(w, q, N, K), O, "strided")


@pytest.mark.parametrize("N,K,T", [(14336, 4096, 1), (768, 2048, 2), (1000, 512, 8)])
def test_swiglu_pair(fr, O, dev, N, K, T):
    import torch
    wg = fr.synth_nvfp4(61, N, K)
    wu = fr.synth_nvfp4(62, N, K)
    x = fr.synth_normal(63, T * K).reshape(T, K)
    q = O.quantize_q8_1(x)
    y = fr.gemv_swiglu(_t(wg, dev), _t(wu, dev), _t(q, dev), N, K, T)
    torch.cuda.synchronize()
    g = O.gemv_q8_1(wg, q, N, K, nthreads=8)
    u = O.gemv_q8_1(wu, q, N, K, nthreads=8)
    ref = u * (g / (1.0 + np.exp(-g)))
    _check(y.cpu().numpy(), ref, O, "swiglu")


@pytest.mark.parametrize("T", [1, 2, 5, 17])
def test_mul_mat_drop_in(fr, O, dev, T):
    import torch
    N, K = 1024, 4096
    w = fr.synth_nvfp4(71, N, K)
    x = fr.synth_normal(72 + T, T * K).reshape(T, K)
    y = fr.mul_mat(_t(w, dev), _t(x, dev), N, K)
    torch.cuda.synchronize()
    ref = O.gemv_q8_1(w, O.quantize_q8_1(x), N, K, nthreads=8)
    _check(y.cpu().numpy(), ref, O, f"mul_mat T={T}")


@pytest.mark.parametrize("T", [1, 8])
def test_ffn_stagewise(fr, O, dev, T):
    """Dense FFN checked stage by stage like the reference's FRT_B_HREF mode:
    GLU vs fp64, q8_1 of the device GLU bit-exact, down output vs fp64 on the
    device's q8 GLU (+ residual)."""
    import torch
    n_embd, n_ff = 1024, 2816
    wg = fr.synth_nvfp4(81, n_ff, n_embd)
    wu = fr.synth_nvfp4(82, n_ff, n_embd)
    wd = fr.synth_nvfp4(83, n_embd, n_ff)
    x = fr.synth_normal(84, T * n_embd).reshape(T, n_embd)
    r = fr.synth_normal(85, T * n_embd).reshape(T, n_embd)
    glu = torch.empty((T, n_ff), dtype=torch.float32, device=dev)
    gq8 = torch.empty((T, n_ff // 32 * 36), dtype=torch.uint8, device=dev)
    out = fr.ffn(_t(x, dev), _t(wg, dev), _t(wu, dev), _t(wd, dev), n_embd, n_ff, resid=_t(r, dev),
                 chk_glu=glu, chk_glu_q8=gq8)
    torch.cuda.synchronize()
    q = O.quantize_q8_1(x)
    g = O.gemv_q8_1(wg, q, n_ff, n_embd, nthreads=8)
    u = O.gemv_q8_1(wu, q, n_ff, n_embd, nthreads=8)
    _check(glu.cpu().numpy(), u * (g / (1.0 + np.exp(-g))), O, "ffn glu")
    dglu = glu.cpu().numpy()
    np.testing.assert_array_equal(gq8.cpu().numpy(), O.quantize_q8_1(dglu))
    ref = O.gemv_q8_1(wd, gq8.cpu().numpy(), n_embd, n_ff, nthreads=8) + r
    _check(out.cpu().numpy(), ref, O, "ffn out")


def test_gemv_special_scales_and_blocks(fr, O, dev):
    """Scale bytes ggml treats specially (sign bit set: ignored; 0x7F / 0xFF:
    zero) and activation blocks of very different size (zero, 1e-6, 1e3)."""
    import torch
    N, K, T = 300, 1024, 3
    w = fr.synth_nvfp4(91, N, K)
    blocks = w.reshape(N, K // 64, 36)
    blocks[0:7, 0, 0] = 0x7F
    blocks[7:15, 1, 2] = 0xFF
    blocks[15:40, 2, 1] |= 0x80
    blocks[40:60, 3, :4] = 0x7F
    x = fr.synth_normal(92, T * K).reshape(T, K)
    x[0, 0:32] = 0.0
    x[1, 64:96] *= 1e-6
    x[2, 128:160] *= 1e3
    x[2, 512:1024] = 0.0
    q = O.quantize_q8_1(x)
    y = fr.gemv_q8_1(_t(w, dev), _t(q, dev), N, K, T)
    y2 = fr.gemv_f32(_t(w, dev), _t(x, dev), N, K)
    torch.cuda.synchronize()
    ref = O.gemv_q8_1(w, q, N, K)
    _check(y.cpu().numpy(), ref, O, "special scales / blocks (q8 input)")
    _check(y2.cpu().numpy(), ref, O, "special scales / blocks (f32 input)")
    assert fr.device_status() == 0


def test_invalid_arguments_return_minus_one(fr, dev):
    import torch
    x = torch.zeros((1, 64), dtype=torch.float32, device=dev)
    w = torch.zeros((4, 36), dtype=torch.uint8, device=dev)
    y = torch.zeros((1, 4), dtype=torch.float32, device=dev)
    L = fr.lib()
    # K not a multiple of 64
    assert L.fr_gemv_nvfp4_f32(fr._ptr(w), 36, fr._ptr(x), 64, None, None, 0, fr._ptr(y), 4, 4, 48, 1,
                               fr._stream()) == -1
    # w_ld smaller than a row
    assert L.fr_gemv_nvfp4_f32(fr._ptr(w), 32, fr._ptr(x), 64, None, None, 0, fr._ptr(y), 4, 4, 64, 1,
                               fr._stream()) == -1
    assert fr.device_status() == 0
