"""Kernel-level parity of the token-stage kernels against the CPU oracle's
operators, through the C ABI (gcdr_k_dw_gelu_shift, gcdr_k_up_add,
gcdr_k_ln_finalize).

The pipeline fuses these operators of the shifted-MLP blocks and decoder
joins (gc#38-130, gc#234-250): each test feeds the kernel fp16 activations and
the real GC-Net / DR-Net parameters of one block, and compares its fp16
output with the oracle's fp32 composition of the same operators
(oracle/gcdr_oracle.py: dwconv3x3, gelu, shift, resize2x, relu, add,
layernorm).  Mirrors the reference's GPU-kernel-vs-CPU-kernel tests
(tests/Sdcb.SimdGcdrNet.Tests/VkKernelTests.cs:15-65).

Tolerance: the kernels store fp16 (2^-11 relative rounding), so the largest
difference is bounded at 2e-3 of the output's scale and the relative L2
error at 1e-3; the oracle's shift is exact and must move the same channels
(a wrong group or offset shows as an O(1) error).
"""
import ctypes

import numpy as np
import pytest

import golden_data as G
from gpu_util import Act, Shift, from_device_layout, to_device_layout
from oracle import gcdr_oracle as O

pytestmark = pytest.mark.gpu

MAX_REL, L2_REL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def nets():
    return {"gc": O.GcdrNet.load(G.GC_PATH), "dr": O.GcdrNet.load(G.DR_PATH)}


def _dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda:0", dtype) if dtype is not None else t.to("cuda:0")


def _close(got, want, what):
    scale = np.abs(want).max() + 1e-6
    d = np.abs(got - want).max() / scale
    l2 = np.linalg.norm(got - want) / (np.linalg.norm(want) + 1e-12)
    assert d < MAX_REL and l2 < L2_REL, f"{what}: max rel {d:.2e}, rel L2 {l2:.2e}"


def _f16(x):
    return x.astype(np.float16).astype(np.float32)


def _blocks(nets):
    return [(n, b, getattr(nets[n], b)) for n in ("gc", "dr") for b in ("block1", "block2", "dblock1", "dblock2")]


# (net, block, H, W): the block's channels at small grids, odd widths, one row and one column
DW_CASES = [("gc", "block1", 9, 13), ("gc", "block2", 4, 7), ("gc", "dblock2", 16, 21),
            ("dr", "block1", 6, 11), ("dr", "block2", 3, 5), ("dr", "dblock2", 1, 9), ("gc", "dblock1", 7, 1)]


@pytest.mark.parametrize("case", DW_CASES, ids=lambda c: "%s_%s_%dx%d" % c)
def test_dw_gelu_shift_matches_oracle(nets, case):
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    net, name, H, W = case
    blk = getattr(nets[net], name)
    w, b = blk.dw
    C = w.shape[0]
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    x = _f16(rng.standard_normal((H, W, C)).astype(np.float32) * 2)
    axis, ends, offs = blk.shift_w
    assert axis == 3
    want = O.shift(O.gelu(O.dwconv3x3(x, w, b)), axis, ends, offs)
    wt = np.ascontiguousarray(w.reshape(C, 9).T)          # tap-major [9][C]
    dx = _dev(x, torch.float16)
    out = torch.full((H, W, C), float("nan"), dtype=torch.float16, device="cuda:0")
    sh = Shift.of(ends, offs)
    dwt, db = _dev(wt), _dev(b.astype(np.float32))
    rc = L.gcdr_k_dw_gelu_shift(dx.data_ptr(), H, W, C, dwt.data_ptr(), db.data_ptr(), ctypes.byref(sh),
                                out.data_ptr(), None)
    assert rc == 0
    got = out.float().cpu().numpy()
    assert not np.isnan(got).any(), "unwritten outputs"
    _close(got, want, f"dw_gelu_shift {case}")


# (C, H, W, ends, offs): W-shift groups whose boundaries fall inside 8-channel chunks,
# with offsets far apart (the gather reads each part of a chunk at its own offset);
# 24 channels take the direct kernel, 64 and 96 the tiled one (slabs of 8 and 4
# chunks, several column and row tiles), offsets 80 apart the direct one again
STRADDLE_SHIFTS = [(24, 5, 13, [5, 19, 24], [3, -2, 1]), (24, 5, 13, [12, 20, 24], [-4, 0, 6]),
                   (24, 5, 13, [8, 16, 24], [9, -9, 0]), (64, 9, 70, [13, 26, 39, 52, 64], [2, 1, 0, -1, -2]),
                   (96, 7, 300, [20, 45, 70, 96], [5, -3, 0, 1]), (64, 6, 100, [30, 64], [40, -40])]


@pytest.mark.parametrize("shift", STRADDLE_SHIFTS, ids=lambda s: "C%d_%dx%d_ends%s" % (s[0], s[1], s[2], "_".join(map(str, s[3]))))
def test_dw_shift_straddling_groups(shift):
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    C, H, W, ends, offs = shift
    rng = np.random.default_rng(sum(ends) + 7 * sum(offs))
    x = _f16(rng.standard_normal((H, W, C)).astype(np.float32))
    w = (rng.standard_normal((C, 1, 3, 3)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(C) * 0.1).astype(np.float32)
    want = O.shift(O.gelu(O.dwconv3x3(x, w, b)), 3, ends, offs)
    wt = np.ascontiguousarray(w.reshape(C, 9).T)
    out = torch.full((H, W, C), float("nan"), dtype=torch.float16, device="cuda:0")
    dx, dwt, db = _dev(x, torch.float16), _dev(wt), _dev(b)
    sh = Shift.of(ends, offs)
    assert L.gcdr_k_dw_gelu_shift(dx.data_ptr(), H, W, C, dwt.data_ptr(), db.data_ptr(), ctypes.byref(sh),
                                  out.data_ptr(), None) == 0
    got = out.float().cpu().numpy()
    assert not np.isnan(got).any(), "unwritten outputs"
    _close(got, want, f"dw_gelu_shift {shift}")


def test_dw_shift_rejects_three_groups_in_a_chunk():
    """The depthwise gather gives a chunk of 8 channels two shift groups at most."""
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    H, W, C = 2, 4, 16
    x = torch.zeros((H, W, C), dtype=torch.float16, device="cuda:0")
    wt = torch.zeros((9, C), dtype=torch.float32, device="cuda:0")
    b = torch.zeros(C, dtype=torch.float32, device="cuda:0")
    sh = Shift.of([3, 6, 16], [1, 0, -1])
    assert L.gcdr_k_dw_gelu_shift(x.data_ptr(), H, W, C, wt.data_ptr(), b.data_ptr(), ctypes.byref(sh),
                                  x.data_ptr(), None) == 1


# (ends, offs) of H-shift groups for the token join's LayerNorm scatter: boundaries
# inside chunks (a chunk's two parts stored apart), and groups narrower than a chunk
JOIN_SHIFTS = [([5, 19, 27, 40], [2, -1, 0, -2]), ([3, 6, 11, 30, 40], [2, 1, 0, -1, -2]),
               ([13, 26, 40], [-3, 4, 1])]


@pytest.mark.parametrize("shift", JOIN_SHIFTS, ids=lambda s: "ends%s" % "_".join(map(str, s[0])))
def test_join_ln_shift_groups(shift):
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    ends, offs = shift
    H, W, C = 8, 6, 40
    rng = np.random.default_rng(sum(ends))
    d = _f16(rng.standard_normal((H // 2, W // 2, C)).astype(np.float32))
    skip = _f16(rng.standard_normal((H, W, C)).astype(np.float32))
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    bb = (0.1 * rng.standard_normal(C)).astype(np.float32)
    want = O.add(O.relu(O.resize2x(d)), skip)
    want_h = O.shift(O.layernorm(_f16(want), g, bb), 2, ends, offs)
    dd, dskip = _dev(d, torch.float16), _dev(skip, torch.float16)
    sk = Act(dskip.data_ptr(), H, W, C, 0)
    out = torch.full((H * W * C,), float("nan"), dtype=torch.float16, device="cuda:0")
    h = torch.full((H * W * C,), float("nan"), dtype=torch.float16, device="cuda:0")
    oa = Act(out.data_ptr(), H, W, C, 0)
    sh = Shift.of(ends, offs)
    dg, db = _dev(g), _dev(bb)
    assert L.gcdr_k_up_add(dd.data_ptr(), ctypes.byref(sk), ctypes.byref(oa), dg.data_ptr(), db.data_ptr(),
                           ctypes.c_float(1e-5), ctypes.byref(sh), h.data_ptr(), None) == 0
    got_h = h.float().cpu().numpy().reshape(H, W, C)
    assert not np.isnan(got_h).any(), "unwritten outputs"
    _close(got_h, want_h, f"join LN2 + H shift {shift}")


# (net, block, H, W, skip layout, kind of join): the decoder joins at small grids
JOIN_CASES = [("gc", "dblock1", 6, 10, 2, "tok"), ("dr", "dblock1", 4, 6, 2, "tok"),
              ("gc", "dblock2", 8, 14, 2, "tok"), ("dr", "dblock2", 10, 4, 2, "tok"),
              ("gc", None, 16, 22, 1, "pad"), ("dr", None, 12, 18, 1, "pad"), ("dr", None, 2, 2, 1, "pad")]


@pytest.mark.parametrize("case", JOIN_CASES, ids=lambda c: "%s_%s_%dx%d_skip%d_%s" % c)
def test_up_add_matches_oracle(nets, case):
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    net, name, H, W, skind, form = case
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    if form == "tok":
        blk = getattr(nets[net], name)
        C = blk.norm2[0].shape[0]
    else:
        C = nets[net].enc[0][0].shape[0] if H > 8 else nets[net].enc[1][0].shape[0]
    d = _f16(rng.standard_normal((H // 2, W // 2, C)).astype(np.float32))
    skip = _f16(np.maximum(rng.standard_normal((H, W, C)).astype(np.float32), 0))
    want = O.add(O.relu(O.resize2x(d)), skip)
    dd = _dev(d, torch.float16)
    dskip = to_device_layout(L, _dev(skip, torch.float16), skind)
    sk = Act(dskip.data_ptr(), H, W, C, skind)
    if form == "tok":
        out = torch.full((H * W * C,), float("nan"), dtype=torch.float16, device="cuda:0")
        h = torch.full((H * W * C,), float("nan"), dtype=torch.float16, device="cuda:0")
        g, b = blk.norm2
        axis, ends, offs = blk.shift_h
        assert axis == 2
        sh = Shift.of(ends, offs)
        dg, db = _dev(g.astype(np.float32)), _dev(b.astype(np.float32))
        oa = Act(out.data_ptr(), H, W, C, 0)
        rc = L.gcdr_k_up_add(dd.data_ptr(), ctypes.byref(sk), ctypes.byref(oa), dg.data_ptr(), db.data_ptr(),
                             ctypes.c_float(1e-5), ctypes.byref(sh), h.data_ptr(), None)
        assert rc == 0
        got = out.float().cpu().numpy().reshape(H, W, C)
        _close(got, want, f"join {case}")
        want_h = O.shift(O.layernorm(_f16(want), g, b), axis, ends, offs)
        got_h = h.float().cpu().numpy().reshape(H, W, C)
        assert not np.isnan(got_h).any()
        _close(got_h, want_h, f"join LN2 + H shift {case}")
    else:
        n = L.gcdr_k_to_layout(None, H, W, C, 1, None, None)
        out = torch.full((n,), float("nan"), dtype=torch.float16, device="cuda:0")
        oa = Act(out.data_ptr(), H, W, C, 1)
        rc = L.gcdr_k_up_add(dd.data_ptr(), ctypes.byref(sk), ctypes.byref(oa), None, None, ctypes.c_float(0),
                             None, None, None)
        assert rc == 0
        padded = out.float().cpu().numpy().reshape(H + 2, W + 2, C)
        got = padded[1:H + 1, 1:W + 1]
        _close(got, want, f"join {case}")
        # the producer writes the reflect border its consumer (a reflect-pad conv) reads
        ry = [1 if H > 1 else 0] + list(range(H)) + [H - 2 if H > 1 else 0]
        rx = [1 if W > 1 else 0] + list(range(W)) + [W - 2 if W > 1 else 0]
        assert np.array_equal(padded, got[np.ix_(ry, rx)]), "reflect border"


# (net, norm, H, W, ksplit, out layout, residual, with LN2 + shift)
FIN_CASES = [("gc", "pe3", 6, 10, 3, 0, False, True), ("dr", "pe4", 3, 5, 9, 0, False, True),
             ("gc", "pe4", 2, 3, 5, 0, False, True),          # H shift by +-2 on a 2-row grid: zero groups
             ("gc", "block1", 6, 10, 2, 2, True, False), ("dr", "block2", 4, 4, 4, 1, True, False),
             ("dr", "dblock2", 8, 6, 1, 1, True, False), ("gc", "dblock1", 5, 9, 5, 0, True, False)]


@pytest.mark.parametrize("case", FIN_CASES, ids=lambda c: "%s_%s_%dx%d_ks%d_out%d_res%d_ln2%d" % c)
def test_ln_finalize_matches_oracle(nets, case):
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    net, name, H, W, ks, okind, use_res, ln2 = case
    n_ = nets[net]
    if name in ("pe3", "pe4"):
        g1, b1 = n_.pe3_norm if name == "pe3" else n_.pe4_norm
        nxt = n_.block1 if name == "pe3" else n_.block2
    else:
        g1, b1 = getattr(n_, name).norm_out
        nxt = None
    N = g1.shape[0]
    T = H * W
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    part = rng.standard_normal((ks, T, N)).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float32)
    res = _f16(rng.standard_normal((T, N)).astype(np.float32)) if use_res else None
    v = part[0].copy()
    for k in range(1, ks):
        v += part[k]
    v = v + bias
    if use_res:
        v = v + res
    want = O.layernorm(v.reshape(H, W, N), g1, b1)
    dpart, dbias = _dev(part), _dev(bias)
    dres = _dev(res, torch.float16) if use_res else None
    dg1, db1 = _dev(g1.astype(np.float32)), _dev(b1.astype(np.float32))
    nrows = T if okind == 0 else L.gcdr_k_to_layout(None, H, W, N, okind, None, None) // N
    out = torch.full((nrows * N,), float("nan"), dtype=torch.float16, device="cuda:0")
    oa = Act(out.data_ptr(), H, W, N, okind)
    if ln2:
        g2, b2 = nxt.norm2
        axis, ends, offs = nxt.shift_h
        sh = Shift.of(ends, offs)
        dg2, db2 = _dev(g2.astype(np.float32)), _dev(b2.astype(np.float32))
        out2 = torch.full((T * N,), float("nan"), dtype=torch.float16, device="cuda:0")
        rc = L.gcdr_k_ln_finalize(dpart.data_ptr(), ks, H, W, N, dbias.data_ptr(), None, dg1.data_ptr(),
                                  db1.data_ptr(), ctypes.c_float(1e-5), dg2.data_ptr(), db2.data_ptr(),
                                  ctypes.c_float(1e-5), ctypes.byref(sh), ctypes.byref(oa), out2.data_ptr(), None)
    else:
        rc = L.gcdr_k_ln_finalize(dpart.data_ptr(), ks, H, W, N, dbias.data_ptr(),
                                  dres.data_ptr() if use_res else None, dg1.data_ptr(), db1.data_ptr(),
                                  ctypes.c_float(1e-5), None, None, ctypes.c_float(0), None, ctypes.byref(oa), None,
                                  None)
    assert rc == 0
    got = from_device_layout(out, H, W, N, okind)
    assert not np.isnan(got).any(), "unwritten outputs"
    _close(got, want, f"ln_finalize {case}")
    if ln2:
        want2 = O.shift(O.layernorm(_f16(want), g2, b2), axis, ends, offs)
        got2 = out2.float().cpu().numpy().reshape(H, W, N)
        assert not np.isnan(got2).any()
        _close(got2, want2, f"ln_finalize LN2 + H shift {case}")


@pytest.mark.parametrize("off", [5, -7, 9])
def test_shift_offset_beyond_width_zeros(off):
    """A group shifted by |off| >= W is all zeros (EngineTests.cs:171-180 for the CPU
    kernel): here through the depthwise kernel's W-shift scatter on a 5-wide grid."""
    import torch
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    H, W, C = 4, 5, 16
    x = torch.ones((H, W, C), dtype=torch.float16, device="cuda:0")
    wt = torch.zeros((9, C), dtype=torch.float32, device="cuda:0")
    wt[4] = 1.0                                       # centre tap: dw(x) = x
    b = torch.zeros(C, dtype=torch.float32, device="cuda:0")
    out = torch.full((H, W, C), -1.0, dtype=torch.float16, device="cuda:0")
    sh = Shift.of([8, 16], [off, 0])                 # group 0 shifted, group 1 in place
    assert L.gcdr_k_dw_gelu_shift(x.data_ptr(), H, W, C, wt.data_ptr(), b.data_ptr(), ctypes.byref(sh),
                                  out.data_ptr(), None) == 0
    got = out.float().cpu().numpy()
    assert (got[:, :, :8] == 0).all(), "shifted-out group must be zeros"
    assert np.allclose(got[:, :, 8:], 0.8413447, atol=2e-3), "unshifted group: gelu(1) = 0.8413"


def test_token_entries_reject_bad_arguments():
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    sh = Shift.of([32, 64, 96, 128, 200], [2, 1, 0, -1, -2])   # an end past C = 160
    x = ctypes.c_void_p(16)
    assert L.gcdr_k_dw_gelu_shift(x, 4, 4, 160, x, x, ctypes.byref(sh), x, None) == 1
    bad = Act(None, 4, 4, 32, 0)
    assert L.gcdr_k_up_add(x, ctypes.byref(bad), ctypes.byref(bad), None, None, ctypes.c_float(0), None, None,
                           None) == 1
