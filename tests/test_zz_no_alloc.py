"""gcdr_k_conv_static: the k-split convolution layer whose fp32 partial sums
live in a static device workspace (no allocation by the library).

Its output is checked against the allocating layer entry gcdr_k_conv on the
same inputs, on two calls in a row (different layers and inputs, so the
second call cannot pass on what the first one left in the workspace).  The
file is named to be collected last: it must pass both alone (the first call
then does the workspace set-up) and after every other test.
"""
import ctypes

import numpy as np
import pytest

from gpu_util import ConvDesc, pack_weights

pytestmark = pytest.mark.gpu

GCDR_ERR_RANGE = 2
STATIC_WS_FLOATS = 16 * 1024 * 1024 // 4


def _layer(lib, kind, H, W, C, N, seed):
    """Device tensors of one seeded layer: (input in the kind's layout, packed weights, bias)."""
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
        lay = {0: 1, 1: 2, 3: 3}[kind]
        n = lib.gcdr_k_to_layout(None, H, W, C, lay, None, None)
        inp = torch.empty(n, dtype=torch.float16, device=dev)
        assert lib.gcdr_k_to_layout(xt.data_ptr(), H, W, C, lay, inp.data_ptr(), None) == n
    wt = torch.from_numpy(pack_weights(w)).to(dev, torch.float16)
    bt = torch.from_numpy(b).to(dev)
    return inp, wt, bt


def _out_dims(kind, H, W):
    return (H // 2, W // 2) if kind == 1 else (H, W)


# (kind, H, W, C, N, epilogue, nsplit, ksplit, seed): GC pe3 at /8 of a small page
# (stride 2, 18 k-blocks in 3 splits), a DR fc2-like 1x1 token Gemm with relu, and the
# two padded-pitch layouts (reflect border, zero border) at widths that are not a
# multiple of 128: their grid rows carry two pitch columns per image row that the
# partial-sum epilogue drops, packing the partials by pixel index.
CALLS = [
    (1, 16, 20, 128, 160, 0, 1, 3, 11),
    (2, 18, 25, 256, 256, 2, 2, 4, 12),
    (0, 20, 150, 64, 64, 0, 1, 3, 13),
    (3, 16, 200, 32, 128, 2, 2, 9, 14),
]


def test_static_workspace_conv_matches_allocating_entry():
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    for kind, H, W, C, N, ep, ns, ks, seed in CALLS:
        Ho, Wo = _out_dims(kind, H, W)
        assert ks * Ho * Wo * N <= STATIC_WS_FLOATS
        inp, wt, bt = _layer(L, kind, H, W, C, N, seed)
        Ho, Wo = _out_dims(kind, H, W)
        want = torch.full((Ho, Wo, N), float("nan"), dtype=torch.float16, device="cuda:0")
        got = torch.full((Ho, Wo, N), float("nan"), dtype=torch.float16, device="cuda:0")
        d = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), ep, want.data_ptr(), None, 1, 1)
        assert L.gcdr_k_conv(ctypes.byref(d), 0, None) == 0
        torch.cuda.synchronize()
        s = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), ep, got.data_ptr(), None, ns, ks)
        assert L.gcdr_k_conv_static(ctypes.byref(s), None) == 0
        torch.cuda.synchronize()
        a = got.float().cpu().numpy()
        r = want.float().cpu().numpy()
        assert not np.isnan(a).any(), "static-workspace conv left outputs unwritten"
        # both sides round fp32 sums to fp16; they differ in accumulation order only
        scale = np.abs(r).max() + 1e-6
        assert np.abs(a - r).max() / scale < 2e-3
        assert np.linalg.norm(a - r) / (np.linalg.norm(r) + 1e-12) < 1e-3


def test_static_workspace_rejects_oversize_layer():
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    H, W, C, N, ks = 64, 128, 512, 512, 8
    assert ks * H * W * N > STATIC_WS_FLOATS
    buf = torch.zeros(64, dtype=torch.float16, device="cuda:0")
    bias = torch.zeros(N, dtype=torch.float32, device="cuda:0")
    p = buf.data_ptr()
    d = ConvDesc(2, H, W, C, N, p, p, bias.data_ptr(), 0, p, None, 1, ks)
    assert L.gcdr_k_conv_static(ctypes.byref(d), None) == GCDR_ERR_RANGE
