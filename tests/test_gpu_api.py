"""The public GcdrEnhancer boundary on the CUDA backend.

Mirrors the reference's pixel-format and engine tests
(tests/Sdcb.SimdGcdrNet.Tests/PixelFormatTests.cs:26-87,
EngineTests.cs:183-281, VulkanTests.cs:84-131,
VulkanDeviceLossTests.cs:15-37): every format gives the Bgr24 result of the
same backend with channels permuted, alpha is copied through, strides are
honoured and row padding stays untouched; in-place enhancement; one worker
serves every size with results identical to a fresh enhancer; concurrent
callers; recovery after a device loss (injected on the host); the 32x32
minimum; odd, unpadded shapes against the oracle.
"""
import threading

import numpy as np
import pytest

import golden_data as G
from oracle import gcdr_oracle as O

pytestmark = pytest.mark.gpu

BGR24, RGB24, BGRA32, RGBA32 = 0, 1, 2, 3
U8_TOL, U8_MAX, FRAC = 2, 8, 0.999


def u8_check(got, want, what):
    d = np.abs(got.astype(np.int32) - want.astype(np.int32))
    frac = (d <= U8_TOL).mean()
    assert d.max() <= U8_MAX and frac >= FRAC, f"{what}: max {d.max()}, within {U8_TOL}: {frac:.6f}"


@pytest.fixture(scope="module")
def enh():
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    e = GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH)
    yield e
    e.dispose()


def _bpp(fmt):
    return 4 if fmt in (BGRA32, RGBA32) else 3


def pack(bgr, w, h, fmt, stride):
    """Tight BGR24 -> `fmt` rows of `stride` bytes; alpha (x*7 + y*13) & 255, padding 0x5A
    (PixelFormatTests.cs:93-110)."""
    bpp = _bpp(fmt)
    out = np.full((h, stride), 0x5A, np.uint8)
    px = out[:, :w * bpp].reshape(h, w, bpp)
    swap = fmt in (RGB24, RGBA32)
    px[:, :, 0] = bgr[:, :, 2] if swap else bgr[:, :, 0]
    px[:, :, 1] = bgr[:, :, 1]
    px[:, :, 2] = bgr[:, :, 0] if swap else bgr[:, :, 2]
    if bpp == 4:
        ys, xs = np.mgrid[0:h, 0:w]
        px[:, :, 3] = ((xs * 7 + ys * 13) & 255).astype(np.uint8)
    return out.reshape(-1)


@pytest.mark.parametrize("fmt", [BGR24, RGB24, BGRA32, RGBA32])
def test_format_matches_bgr24(enh, fmt):
    h, w, ph, pw, oh, ow = G.dims("pad")
    bgr = G.bgr("pad")
    expect = enh.enhance_image(bgr, ow, oh).reshape(oh, ow, 3)
    bpp = _bpp(fmt)
    ss, ds = ow * bpp + 11, ow * bpp + 7
    src = pack(bgr, ow, oh, fmt, ss)
    dst = np.full(ds * oh, 0xA5, np.uint8)
    enh.enhance(src, ow, oh, ss, dst, ds, fmt)
    rows = dst.reshape(oh, ds)
    px = rows[:, :ow * bpp].reshape(oh, ow, bpp)
    swap = fmt in (RGB24, RGBA32)
    got = np.stack([px[:, :, 2] if swap else px[:, :, 0], px[:, :, 1], px[:, :, 0] if swap else px[:, :, 2]], -1)
    assert np.array_equal(got, expect), f"format {fmt}: channels differ from Bgr24"
    if bpp == 4:
        assert np.array_equal(px[:, :, 3], src.reshape(oh, ss)[:, :ow * 4].reshape(oh, ow, 4)[:, :, 3])
    assert (rows[:, ow * bpp:] == 0xA5).all(), "row padding of dst was written"


def test_in_place_rgba32(enh):
    h, w, ph, pw, oh, ow = G.dims("small")
    src = pack(G.bgr("small"), ow, oh, RGBA32, ow * 4)
    expect = enh.enhance_image(src, ow, oh, RGBA32)
    enh.enhance(src, ow, oh, ow * 4, src, ow * 4, RGBA32)
    assert np.array_equal(expect, src)


@pytest.mark.parametrize("tag,src_pad,dst_pad", [("small", 13, 17), ("pad", 8, 5)])
def test_strided_matches_golden(enh, tag, src_pad, dst_pad):
    h, w, ph, pw, oh, ow = G.dims(tag)
    tight = G.bgr(tag)
    ss, ds = ow * 3 + src_pad, ow * 3 + dst_pad
    src = np.zeros((oh, ss), np.uint8)
    src[:, :ow * 3] = tight.reshape(oh, ow * 3)
    dst = np.zeros((oh, ds), np.uint8)
    enh.enhance(src, ow, oh, ss, dst, ds, BGR24)
    u8_check(dst[:, :ow * 3].reshape(oh, ow, 3), G.final_u8(tag), f"strided[{tag}] vs golden")


def test_size_switching_matches_fresh():
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    tags = ["mid", "small", "pad", "mid", "small"]
    fresh = {}
    for tag in dict.fromkeys(tags):
        *_, oh, ow = G.dims(tag)
        with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as e:
            fresh[tag] = e.enhance_image(G.bgr(tag), ow, oh)
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as e:
        for tag in tags:
            *_, oh, ow = G.dims(tag)
            assert np.array_equal(e.enhance_image(G.bgr(tag), ow, oh), fresh[tag]), f"size switch [{tag}]"
        assert e.pool_stats[1] == 1, "one worker should serve every size"


def test_concurrent_same_size(enh):
    *_, oh, ow = G.dims("small")
    src = G.bgr("small")
    expect = enh.enhance_image(src, ow, oh)
    results, errors = [None] * 8, []

    def run(t):
        try:
            results[t] = enh.enhance_image(src, ow, oh)
        except Exception as ex:  # surfaced below
            errors.append(ex)

    threads = [threading.Thread(target=run, args=(t,)) for t in range(8)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors
    for t, r in enumerate(results):
        assert np.array_equal(r, expect), f"concurrent caller {t} differs"
    u8_check(expect.reshape(oh, ow, 3), G.final_u8("small"), "concurrent vs golden")


def test_recovers_from_device_loss():
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    *_, oh, ow = G.dims("small")
    src = G.bgr("small")
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as e:
        first = e.enhance_image(src, ow, oh)
        evicted0 = e.pool_stats[2]
        e.inject_device_loss(1)
        second = e.enhance_image(src, ow, oh)
        assert np.array_equal(first, second)
        assert e.pool_stats[2] > evicted0, "the failed pool should have been dropped"


def test_min_size_32x32(enh, oracle):
    rng = np.random.default_rng(3)
    src = rng.integers(0, 256, 32 * 32 * 3, dtype=np.uint8)
    dst = enh.enhance_image(src, 32, 32)
    assert dst.shape == (32 * 32 * 3,)
    want = np.zeros_like(src)
    oracle.enhance(src, 32, 32, 32 * 3, want, 32 * 3, BGR24)
    u8_check(dst, want, "32x32 vs oracle")


@pytest.mark.parametrize("w,h,fmt,seed", [(45, 37, BGRA32, 5), (2011, 1503, RGBA32, 7)])
def test_odd_shapes_match_oracle(enh, oracle, w, h, fmt, seed):
    """Unpadded shapes (top/left replicate padding to a multiple of 32 and crop back)."""
    from sdcb.gcdrnet_b200.synth import document
    src = document(w, h, seed=seed, fmt=fmt, strokes=max(8, w * h // 16000))
    stride = w * 4
    dst = np.zeros_like(src)
    enh.enhance(src, w, h, stride, dst, stride, fmt)
    want = np.zeros_like(src)
    oracle.enhance(src, w, h, stride, want, stride, fmt)
    got = dst.reshape(h, w, 4)
    ref = want.reshape(h, w, 4)
    assert np.array_equal(got[:, :, 3], src.reshape(h, w, 4)[:, :, 3]), "alpha must be copied bit-exact"
    u8_check(got[:, :, :3], ref[:, :, :3], f"{w}x{h} vs oracle")


def test_from_bytes_and_streams_match_from_files():
    """FromBytes / FromStreams give the bytes FromFiles gives (ModelsPackageTests.cs:24-35)."""
    import io
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    *_, oh, ow = G.dims("small")
    src = G.bgr("small")
    gc, dr = open(G.GC_PATH, "rb").read(), open(G.DR_PATH, "rb").read()
    outs = []
    for make in (lambda: GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH),
                 lambda: GcdrEnhancer.from_bytes(gc, dr),
                 lambda: GcdrEnhancer.from_streams(io.BytesIO(gc), io.BytesIO(dr))):
        with make() as e:
            outs.append(e.enhance_image(src, ow, oh))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
