"""The allocation-free dense FFN entry point (fr_ffn_nvfp4_noalloc).

It exists for callers that cannot call cudaMalloc -- code inside a CUDA-graph
capture, hosts (such as ggml) whose allocator plans all device buffers up
front, processes with a fixed device-memory budget -- and keeps its
intermediates in a static device array instead of a grown workspace.  This
test calls it through the C-ABI twice in a row, with different inputs, and
checks each result against the regular entry point fr_ffn_nvfp4 and against
the CPU oracle's restatement of the same FFN (q8_1 of x, SwiGLU of the
gate/up dot products, q8_1 of the GLU, down dot products, residual), within
the tolerance the parity tests use (max rel err 1e-3).  The allocation-free
entry always runs the dp4a matvec, whatever the matvec-path setting, so it
can differ from fr_ffn_nvfp4 within that tolerance.  It also checks the size
limit.  The file is named so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-3


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _rel(mine, ref):
    mine = np.asarray(mine, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref * ref)))
    return float(np.max(np.abs(mine - ref) / np.maximum(np.abs(ref), 1e-3 * rms)))


def _noalloc(fr, x, wg, wu, wd, n_embd, n_ff, out, resid=None):
    return fr.lib().fr_ffn_nvfp4_noalloc(fr._ptr(x), fr._ptr(wg), fr._ptr(wu), fr._ptr(wd), None, None, None,
                                         fr._ptr(resid), fr._ptr(out), x.shape[0], n_embd, n_ff, fr._stream())


def _oracle_ffn(O, x, wg, wu, wd, n_embd, n_ff, r):
    qx = O.quantize_q8_1(x)
    g = O.gemv_q8_1(wg, qx, n_ff, n_embd)
    u = O.gemv_q8_1(wu, qx, n_ff, n_embd)
    glu = (u * (g / (1.0 + np.exp(-g)))).astype(np.float32)
    return O.gemv_q8_1(wd, O.quantize_q8_1(glu), n_embd, n_ff) + r.astype(np.float64)


def test_noalloc_ffn_matches_regular_entry_twice(fr, dev, O):
    import torch
    n_embd, n_ff, T = 1024, 2816, 4
    hw = [fr.synth_nvfp4(901, n_ff, n_embd), fr.synth_nvfp4(902, n_ff, n_embd), fr.synth_nvfp4(903, n_embd, n_ff)]
    wg, wu, wd = (_t(w, dev) for w in hw)
    for call, seed in enumerate((904, 905)):
        hx = fr.synth_normal(seed, T * n_embd).reshape(T, n_embd)
        hr = fr.synth_normal(seed + 10, T * n_embd).reshape(T, n_embd)
        x, r = _t(hx, dev), _t(hr, dev)
        out = torch.full((T, n_embd), float("nan"), dtype=torch.float32, device=dev)
        rc = _noalloc(fr, x, wg, wu, wd, n_embd, n_ff, out, resid=r)
        assert rc == 0, f"call {call}: rc={rc}"
        ref = fr.ffn(x, wg, wu, wd, n_embd, n_ff, resid=r)
        torch.cuda.synchronize()
        mine = out.cpu().numpy()
        assert np.all(np.isfinite(mine)), f"call {call}"
        assert _rel(mine, ref.cpu().numpy()) <= RTOL, f"call {call}"
        assert O.rel_err(mine, _oracle_ffn(O, hx, *hw, n_embd, n_ff, hr)) <= RTOL, f"call {call} vs oracle"
    assert fr.device_status() == 0


def test_noalloc_ffn_rejects_oversize(fr, dev):
    import torch
    n_embd, n_ff = 4096, 14336
    per_tok = n_embd // 32 * 36 + n_ff * 4 + n_ff // 32 * 36
    T = (8 << 20) // per_tok + 1                      # one token past the limit
    x = torch.zeros((T, n_embd), dtype=torch.float32, device=dev)
    w = torch.zeros((n_ff, n_embd // 64 * 36), dtype=torch.uint8, device=dev)
    wd = torch.zeros((n_embd, n_ff // 64 * 36), dtype=torch.uint8, device=dev)
    out = torch.zeros((T, n_embd), dtype=torch.float32, device=dev)
    before = fr.lib().fr_kernel_launches()
    rc = _noalloc(fr, x, w, w, wd, n_embd, n_ff, out)
    assert rc == -904
    assert fr.lib().fr_kernel_launches() == before     # nothing launched
    # the largest T that fits is accepted
    T2 = (8 << 20) // (per_tok + 768) 
    rc = _noalloc(fr, x[:T2], w, w, wd, n_embd, n_ff, out[:T2])
    assert rc == 0
    torch.cuda.synchronize()
