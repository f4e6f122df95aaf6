"""fr_copy_pinned: the SM-driven transfer between device memory and pinned
host memory that the decode loop's per-step inputs and results use."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fr():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    import frb200
    return frb200


def test_copy_round_trip(fr):
    import torch
    dev = torch.device("cuda", 0)
    for n in (4, 4096, 1 << 20):
        h = torch.from_numpy(np.random.default_rng(n).standard_normal(n).astype(np.float32)).pin_memory()
        d = torch.empty(n, dtype=torch.float32, device=dev)
        back = torch.empty(n, dtype=torch.float32).pin_memory()
        fr.copy_pinned(d, h)
        fr.copy_pinned(back, d)
        torch.cuda.synchronize()
        assert torch.equal(d.cpu(), h)
        assert torch.equal(back, h)
    assert fr.device_status() == 0


def test_copy_in_graph_reads_host_every_replay(fr):
    """Inside a captured graph each replay moves the host buffer's current
    bytes (nothing is cached at capture time)."""
    import torch
    dev = torch.device("cuda", 0)
    h = torch.zeros(1024, dtype=torch.float32).pin_memory()
    d = torch.empty(1024, dtype=torch.float32, device=dev)
    out = torch.zeros(1024, dtype=torch.float32).pin_memory()
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        fr.copy_pinned(d, h, stream=s)
        d.mul_(2.0)
        fr.copy_pinned(out, d, stream=s)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fr.copy_pinned(d, h, stream=s)
        d.mul_(2.0)
        fr.copy_pinned(out, d, stream=s)
    for k in range(3):
        h.copy_(torch.arange(1024, dtype=torch.float32) + k)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, 2.0 * (torch.arange(1024, dtype=torch.float32) + k))


def test_copy_rejects_pageable_and_misaligned(fr):
    import torch
    dev = torch.device("cuda", 0)
    d = torch.empty(64, dtype=torch.float32, device=dev)
    pageable = torch.zeros(64, dtype=torch.float32)
    L = fr.lib()
    assert L.fr_copy_pinned(fr._ptr(d), fr._ptr(pageable), 256, fr._stream()) == -1
    h = torch.zeros(64, dtype=torch.float32).pin_memory()
    assert L.fr_copy_pinned(fr._ptr(d), fr._ptr(h), 20, fr._stream()) == -1
