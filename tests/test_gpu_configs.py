"""Parity on the benchmark configurations themselves, at their full sizes.

  c0  one 1600x1152 Bgr24 document (seed 0 of the document generator) against
      the CPU oracle at the gate: u8 within +-2 LSB on >= 99.9 % of the values
      and never more than 8 off; the shading map I_sm with relative L2 <= 1e-2;
      the net input bit-exact; the fused division correction (GC head epilogue
      -> DR stem input, stored as an fp16 hi/lo pair) equal to the oracle's
      div6 of the same shading map.
  c1  the conv microbenchmark shapes (3x3 stride-1 zero-pad conv + bias + relu,
      and the 1x1 256 -> 3 head) against an fp32 conv of the UNROUNDED fp32
      activations and weights: relative L2 <= 1e-3, i.e. the fp16 operand
      quantisation is inside the bar.
  c2  a 1600x1152 Bgra32 document with row stride width*4 + 64, enhanced in
      place: alpha bit-exact, u8 at the gate, row padding untouched.
  c4  a large odd Rgba32 shape near the top of the stress range
      (4011 x 3001, seed 7): replicate padding to a multiple of 32, crop back,
      u8 at the gate, alpha bit-exact.

Mirrors tests/Sdcb.SimdGcdrNet.Tests/GoldenTests.cs:52-73 (pipeline u8 against
the CPU path) and the GPU tolerance ladder of VulkanTests.cs:15-80, 138-185.
"""
import ctypes

import numpy as np
import pytest

import golden_data as G
from gpu_util import ConvDesc, pack_weights
from oracle import gcdr_oracle as O

pytestmark = pytest.mark.gpu

U8_TOL, U8_MAX, FRAC = 2, 8, 0.999


def u8_check(got, want, what):
    d = np.abs(got.astype(np.int32) - want.astype(np.int32))
    frac = (d <= U8_TOL).mean()
    assert d.max() <= U8_MAX and frac >= FRAC, f"{what}: max {d.max()}, within {U8_TOL}: {frac:.6f}"


def test_c0_headline_image_matches_oracle(oracle):
    from sdcb.gcdrnet_b200 import CudaWorker, synth
    w, h = 1600, 1152
    src = synth.document(w, h, seed=0)
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        wk.set_debug(True)
        dst = np.zeros_like(src)
        wk.enhance(src, w, h, w * 3, dst, w * 3, 0)
        x, ism, x6 = wk.debug_intermediates(h, w)
    ox, oshadow, ox6, oy = oracle.stages(src, w, h, w * 3, 0)
    assert np.array_equal(x, ox), "net input"
    rl2 = np.linalg.norm(ism - oshadow) / np.linalg.norm(oshadow)
    assert rl2 <= 1e-2, f"I_sm rel L2 {rl2}"
    # the fused div6: DR input = [x, clamp(x / max(I_sm, 1e-6), 0, 1)] on the backend's own I_sm
    assert np.array_equal(x6[..., :3], ox6[..., :3])
    want_r = O.div6(x, ism)[..., 3:]
    assert np.abs(x6[..., 3:] - want_r).max() <= 2e-6, "fused div6 vs div6 of the same I_sm"
    rl2_6 = np.linalg.norm(x6 - ox6) / np.linalg.norm(ox6)
    assert rl2_6 <= 1e-2, f"DR input rel L2 vs oracle {rl2_6}"
    want = np.zeros_like(src)
    O.post(oy, w, h, want, w * 3, 0)
    u8_check(dst, want, "c0 1600x1152 Bgr24 vs oracle")


def test_c2_bgra32_strided_in_place(oracle):
    from sdcb.gcdrnet_b200 import GcdrEnhancer, synth
    w, h = 1600, 1152
    stride = w * 4 + 64
    px = synth.document(w, h, seed=0, fmt=2)
    buf = np.full((h, stride), 0x5A, np.uint8)
    buf[:, :w * 4] = px.reshape(h, w * 4)
    src = buf.copy().reshape(-1)
    want = src.copy()
    oracle.enhance(src, w, h, stride, want, stride, 2)
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        io = buf.reshape(-1)
        enh.enhance(io, w, h, stride, io, stride, 2)       # in place
    got = buf
    assert np.all(got[:, w * 4:] == 0x5A), "row padding written"
    g = got[:, :w * 4].reshape(h, w, 4)
    s = src.reshape(h, stride)[:, :w * 4].reshape(h, w, 4)
    assert np.array_equal(g[:, :, 3], s[:, :, 3]), "alpha not copied through"
    u8_check(g[:, :, :3], want.reshape(h, stride)[:, :w * 4].reshape(h, w, 4)[:, :, :3], "c2 Bgra32 in place")


def test_c4_large_odd_rgba32(oracle):
    from sdcb.gcdrnet_b200 import GcdrEnhancer, synth
    w, h = 4011, 3001
    src = synth.document(w, h, seed=7, fmt=3)
    want = np.zeros_like(src)
    oracle.enhance(src, w, h, w * 4, want, w * 4, 3)
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        got = enh.enhance_image(src.ravel(), w, h, 3).reshape(h, w, 4)
    assert np.array_equal(got[:, :, 3], src[:, :, 3]), "alpha not copied through"
    u8_check(got[:, :, :3], want[:, :, :3], "c4 4011x3001 Rgba32 vs oracle")


# c1: (Cin, Cout, H, W, k); kind 3 = zero pad 1 + relu, kind 2 = the 1x1 head (no relu)
C1_SHAPES = [(6, 32, 1152, 1600, 3), (32, 64, 576, 800, 3), (64, 128, 288, 400, 3),
             (128, 256, 144, 200, 3), (256, 256, 72, 100, 3), (256, 3, 1152, 1600, 1)]


@pytest.mark.parametrize("shape", C1_SHAPES, ids=lambda s: "%d_%d_%dx%d_k%d" % s)
def test_c1_microbench_conv_vs_unrounded_fp32(shape):
    """The kernel takes fp16 operands (the activations and weights are rounded on
    upload) and accumulates in fp32; the bar is relative L2 <= 1e-3 against the
    fp32 conv of the original fp32 tensors.  Channel counts the kernel does not
    take directly are zero-padded (Cin 6 -> 16, Cout 3 -> 16), which leaves the
    sums unchanged; only the real output channels are compared."""
    import torch
    import torch.nn.functional as F
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    cin, cout, H, W, k = shape
    rng = np.random.default_rng(1)
    x = rng.standard_normal((H, W, cin), dtype=np.float32)                      # N(0, 1) activations
    w = (rng.standard_normal((cout, cin, k, k), dtype=np.float32) * np.sqrt(2.0 / (cin * k * k))).astype(np.float32)
    b = (rng.standard_normal(cout, dtype=np.float32) * 0.1).astype(np.float32)   # Kaiming-normal weights
    C = max(16, cin)
    N = max(16, cout)
    dev = torch.device("cuda:0")
    xt = torch.zeros((H, W, C), dtype=torch.float16, device=dev)
    xt[:, :, :cin] = torch.from_numpy(x).to(dev)
    wp = np.zeros((N, C, k, k), np.float32)
    wp[:cout, :cin] = w
    bp = np.zeros(N, np.float32)
    bp[:cout] = b
    kind, ep = (3, 2) if k == 3 else (2, 0)
    if kind == 3:
        n = L.gcdr_k_to_layout(None, H, W, C, 3, None, None)
        inp = torch.empty(n, dtype=torch.float16, device=dev)
        assert L.gcdr_k_to_layout(xt.data_ptr(), H, W, C, 3, inp.data_ptr(), None) == n
    else:
        inp = xt
    wt = torch.from_numpy(pack_weights(wp)).to(dev, torch.float16)
    bt = torch.from_numpy(bp).to(dev)
    out = torch.full((H, W, N), float("nan"), dtype=torch.float16, device=dev)
    d = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), ep, out.data_ptr(), None, 1, 1)
    d.bias_host = bp.ctypes.data
    assert L.gcdr_k_conv(ctypes.byref(d), 0, None) == 0
    assert L.gcdr_k_status(None) == 0
    got = out[:, :, :cout].float().cpu().numpy()
    del inp, xt, out
    # fp32 reference of the unrounded tensors (torch CPU conv; the 1x1 as one matrix product)
    if k == 1:
        want = (x.reshape(-1, cin) @ w.reshape(cout, cin).T + b).reshape(H, W, cout)
    else:
        xc = torch.from_numpy(x).permute(2, 0, 1)[None]
        want = F.relu(F.conv2d(xc, torch.from_numpy(w), torch.from_numpy(b), padding=1))[0].permute(1, 2, 0).numpy()
    assert not np.isnan(got).any()
    rl2 = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rl2 <= 1e-3, f"rel L2 vs unrounded fp32 {rl2:.2e}"
