"""Bounded device waits: a tensor-core conv whose waits run out gives up,
reports GCDR_ERR_TIMEOUT, and leaves the context usable.

No GPU fault is made.  The layer entry's test hook `timeout_probe` makes the
kernel issue no copies and no MMAs, so its barriers are never completed and
every role's first wait runs out after `wait_cycles` (a few hundred
microseconds here instead of the default ~2 s).  The kernel then raises its
abort flag, sets the timeout bit of the device error word, drains (nothing
was issued) and frees its TMEM.  The host reads the status with
gcdr_k_status; the next, normal call on the same device must be correct.
The reference's analogue is tests/Sdcb.SimdGcdrNet.Tests/VulkanDeviceLossTests.cs:14-33.
"""
import ctypes
import time

import numpy as np
import pytest

from gpu_util import ConvDesc, pack_weights, torch_conv

pytestmark = pytest.mark.gpu

GCDR_OK, GCDR_ERR_TIMEOUT = 0, 5


def _layer(lib, kind, H, W, C, N, seed):
    import torch
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((H, W, C)).astype(np.float32)
    k = 1 if kind == 2 else 3
    w = (rng.standard_normal((N, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    dev = torch.device("cuda:0")
    xt = torch.from_numpy(x).to(dev, torch.float16)
    if kind == 2:
        inp = xt
    else:
        n = lib.gcdr_k_to_layout(None, H, W, C, 1, None, None)
        inp = torch.empty(n, dtype=torch.float16, device=dev)
        assert lib.gcdr_k_to_layout(xt.data_ptr(), H, W, C, 1, inp.data_ptr(), None) == n
    wt = torch.from_numpy(pack_weights(w)).to(dev, torch.float16)
    bt = torch.from_numpy(b).to(dev)
    return x, w, b, inp, wt, bt


# (kind, H, W, C, N): a 1x1 token Gemm (flat implicit-GEMM kernel) and a 3x3 reflect conv
# (row-window kernel, resident weights: the weight load is held back too)
CASES = [(2, 18, 25, 128, 128), (0, 24, 40, 32, 64)]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "k%d_%dx%d_c%d_n%d" % c)
def test_wait_runs_out_and_reports_timeout(case):
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    kind, H, W, C, N = case
    x, w, b, inp, wt, bt = _layer(L, kind, H, W, C, N, 21)
    assert L.gcdr_k_status(None) == GCDR_OK          # clears anything earlier tests left
    out = torch.full((H, W, N), float("nan"), dtype=torch.float16, device="cuda:0")
    d = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), 0, out.data_ptr(), None, 1, 1)
    d.bias_host = b.ctypes.data
    d.wait_cycles = 400_000                              # ~0.2 ms at 1.9 GHz
    d.timeout_probe = 1
    t0 = time.perf_counter()
    assert L.gcdr_k_conv(ctypes.byref(d), 0, None) == GCDR_OK   # enqueued
    assert L.gcdr_k_status(None) == GCDR_ERR_TIMEOUT
    assert time.perf_counter() - t0 < 5.0
    assert torch.isnan(out).all().item(), "the probe wrote outputs"
    assert L.gcdr_k_status(None) == GCDR_OK          # read and cleared
    # the context is intact: the same layer, default wait bound, is correct
    d.timeout_probe = 0
    d.wait_cycles = 0
    assert L.gcdr_k_conv(ctypes.byref(d), 0, None) == GCDR_OK
    assert L.gcdr_k_status(None) == GCDR_OK
    got = out.float().cpu().numpy()
    want = torch_conv(0 if kind == 0 else 2, x, w, b, 0)
    assert np.abs(got - want).max() / (np.abs(want).max() + 1e-6) < 4e-3


def test_host_bias_copy_makes_the_call_asynchronous():
    """With bias_host the layer call only enqueues work: a call issued behind a long
    queue returns before the queue drains, and the result is the same as with the
    device bias read back."""
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    kind, H, W, C, N = 2, 64, 96, 128, 128
    x, w, b, inp, wt, bt = _layer(L, kind, H, W, C, N, 22)
    s = torch.cuda.Stream()
    outs = []
    for host in (False, True):
        out = torch.full((H, W, N), float("nan"), dtype=torch.float16, device="cuda:0")
        d = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), 0, out.data_ptr(), None, 1, 1)
        if host:
            d.bias_host = b.ctypes.data
        with torch.cuda.stream(s):
            torch.cuda._sleep(200_000_000)               # ~0.1 s of device time queued ahead
            t0 = time.perf_counter()
            assert L.gcdr_k_conv(ctypes.byref(d), 0, ctypes.c_void_p(s.cuda_stream)) == GCDR_OK
            dt = time.perf_counter() - t0
        assert L.gcdr_k_status(ctypes.c_void_p(s.cuda_stream)) == GCDR_OK
        outs.append((out.float().cpu().numpy(), dt))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert outs[1][1] < 0.05, f"host-bias call blocked for {outs[1][1]:.3f} s"
