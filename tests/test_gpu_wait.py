"""A bounded device-side wait that runs out.

Every spin-wait in the library's kernels gives up after a limit (2 s by
default, settable with fr_set_wait_ns), records bit 0 and its site in the
device status word and lets its kernel return, so the context stays usable.
This test shortens the limit, launches the tensor-parallel completion wait
(fr_tp_wait) on a one-rank buffer whose flag nothing raises, and checks that
the launch returns within the limit's order, that the status word reads
timeout at site 30 (the tensor-parallel flag wait), and that the library
works normally afterwards.  No GPU fault is involved: the flag simply never
arrives.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SITE_TP_WAIT = 30


def test_wait_limit_bounds(fr):
    L = fr.lib()
    assert L.fr_set_wait_ns(10) == -1                 # below 1 us
    assert L.fr_set_wait_ns(3_000_000_000) == -1      # above the 2 s maximum


def test_flag_wait_times_out_and_reports(fr, dev):
    import torch
    L = fr.lib()
    ne = 256
    nbytes = int(L.fr_tp_buffer_bytes(1, ne, ne, 1))
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    s = torch.cuda.Stream(dev)
    fr.device_status(clear=True)
    prev = L.fr_set_wait_ns(50_000_000)               # 50 ms
    try:
        assert prev == 2_000_000_000
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        # one publication expected from rank 0; none ever comes
        rc = L.fr_tp_wait(fr._ptr(buf), nbytes, ne, 1, 1, fr._stream(s))
        assert rc == 0
        s.synchronize()
        dt = time.perf_counter() - t0
        status = fr.device_status(clear=True)
        assert status == 0x1 | (SITE_TP_WAIT << 8), f"status {status:#x}"
        assert 0.04 <= dt < 1.5, f"wait took {dt:.3f} s"
        # the late publication arrives: the next wait (nothing more expected)
        # sees it and returns at once without a timeout
        buf[0:4].view(torch.int32).fill_(1)
        torch.cuda.synchronize()
        assert L.fr_tp_wait(fr._ptr(buf), nbytes, ne, 1, 0, fr._stream(s)) == 0
        s.synchronize()
        assert fr.device_status(clear=True) == 0
    finally:
        assert L.fr_set_wait_ns(prev) == 50_000_000
    # the library still computes: a small matvec against the CPU oracle
    from oracle import oracle as O
    w = fr.synth_nvfp4(31, 128, 512)
    x = fr.synth_normal(32, 512).reshape(1, 512)
    y = fr.gemv_f32(torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev), 128, 512)
    ref = O.gemv_q8_1(w, O.quantize_q8_1(x), 128, 512)
    assert O.rel_err(y.cpu().numpy().astype(np.float64), ref) <= 1e-3
    assert fr.device_status() == 0
