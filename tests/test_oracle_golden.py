"""Pins the CPU oracle against the reference's onnxruntime goldens.

Mirrors tests/Sdcb.SimdGcdrNet.Tests/GoldenTests.cs:13-73 and
EngineTests.cs:143-180 of the reference: per-net float outputs within
max abs 1e-4, the division/concat glue within 1e-3, and the u8 pipeline
within 2 LSB of the truncated golden.
"""
import numpy as np
import pytest

import golden_data as G
from oracle import gcdr_oracle as O


@pytest.mark.parametrize("tag", G.TAGS)
def test_gcnet_matches_onnxruntime(oracle, tag):
    s = O.net_forward(oracle.gc, G.input_nhwc(tag))
    d = np.abs(s - G.f32_nhwc(tag, "shadow")).max()
    assert d < 1e-4, f"gcnet[{tag}] max diff {d}"


@pytest.mark.parametrize("tag", G.TAGS)
def test_drnet_matches_onnxruntime(oracle, tag):
    o = O.net_forward(oracle.dr, G.dr_in_nhwc(tag))
    d = np.abs(o - G.f32_nhwc(tag, "output")).max()
    assert d < 1e-4, f"drnet[{tag}] max diff {d}"


@pytest.mark.parametrize("tag", G.TAGS)
def test_pre_matches_golden_input(tag):
    h, w, ph, pw, oh, ow = G.dims(tag)
    x = O.pre(G.bgr(tag), ow, oh, ow * 3, 0)
    assert x.shape == (h, w, 3)
    assert np.array_equal(x, G.input_nhwc(tag))


@pytest.mark.parametrize("tag", G.TAGS)
def test_divconcat_matches_golden_float(oracle, tag):
    x = G.input_nhwc(tag)
    s = O.net_forward(oracle.gc, x)
    d = np.abs(O.div6(x, s) - G.dr_in_nhwc(tag)).max()
    assert d < 1e-3, f"dr_in[{tag}] max diff {d}"


@pytest.mark.parametrize("tag", ["small", "pad"])
def test_pipeline_matches_golden_u8(oracle, tag):
    h, w, ph, pw, oh, ow = G.dims(tag)
    src = G.bgr(tag)
    dst = np.zeros_like(src)
    oracle.enhance(src, ow, oh, ow * 3, dst, ow * 3, 0)
    d = np.abs(dst.astype(int) - G.final_u8(tag).astype(int)).max()
    assert d <= 2, f"pipeline[{tag}] max u8 diff {d}"


def test_shift_offset_beyond_width_zeros():
    # EngineTests.ChannelShift_OffsetBeyondWidth_Zeros: |off| >= w zeroes the group
    x = np.ones((4, 5, 2), np.float32)
    y = O.shift(x, 3, [2], [5])
    assert np.all(y == 0)


def test_shift_groups_and_zero_fill():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((6, 7, 10)).astype(np.float32)
    ends, offs = [2, 4, 6, 8, 10], [2, 1, 0, -1, -2]
    for axis in (2, 3):
        y = O.shift(x, axis, ends, offs)
        g0 = 0
        for g1, off in zip(ends, offs):
            for yy in range(6):
                for xx in range(7):
                    sy, sx = (yy + off, xx) if axis == 2 else (yy, xx + off)
                    want = x[sy, sx, g0:g1] if 0 <= sy < 6 and 0 <= sx < 7 else 0
                    assert np.array_equal(y[yy, xx, g0:g1], np.broadcast_to(want, (g1 - g0,)))
            g0 = g1


def test_post_rounds_crops_and_copies_alpha():
    rng = np.random.default_rng(1)
    y = rng.uniform(-0.1, 1.1, (64, 64, 3)).astype(np.float32)
    h, w = 60, 57
    for fmt in range(4):
        bpp = O.BPP[fmt]
        stride = w * bpp + 7
        src = rng.integers(0, 256, (h * stride,), dtype=np.uint8)
        dst = np.full(h * stride, 0xA5, np.uint8)
        O.post(y, w, h, dst, stride, fmt, src, stride)
        q = np.clip(np.floor(y[4:, 7:] * np.float32(255) + np.float32(0.5)), 0, 255).astype(np.uint8)
        rows = dst.reshape(h, stride)
        px = rows[:, : w * bpp].reshape(h, w, bpp)
        order = [2, 1, 0] if fmt in (1, 3) else [0, 1, 2]
        assert np.array_equal(px[:, :, order], q)
        if bpp == 4:
            assert np.array_equal(px[:, :, 3], src.reshape(h, stride)[:, : w * 4].reshape(h, w, 4)[:, :, 3])
        assert np.all(rows[:, w * bpp:] == 0xA5)


def test_oracle_builds_agree_bit_for_bit():
    """The AVX2 and AVX-512 builds of the oracle give identical results (the CPU
    baseline uses the widest one the host runs)."""
    import ctypes
    import numpy as np
    from oracle import gcdr_oracle as O
    O.build()
    if not O.isa().startswith("avx512"):
        pytest.skip("host without AVX-512")
    rng = np.random.default_rng(3)
    x = rng.standard_normal((20, 30, 32)).astype(np.float32)
    w = rng.standard_normal((48, 32, 3, 3)).astype(np.float32)
    b = rng.standard_normal(48).astype(np.float32)
    outs = []
    for path in (O.LIB_PATH, O.LIB512_PATH):
        L = ctypes.CDLL(path)
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.orc_conv2d.argtypes = [vp, i, i, i, vp, vp, i, i, i, i, i, vp]
        out = np.empty((20, 30, 48), np.float32)
        L.orc_conv2d(x.ctypes.data, 20, 30, 32, w.ctypes.data, b.ctypes.data, 48, 3, 1, 1, 1, out.ctypes.data)
        outs.append(out)
    assert np.array_equal(outs[0], outs[1])
