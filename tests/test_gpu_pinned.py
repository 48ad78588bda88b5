"""Page-locked caller buffers: the enhancer copies them by DMA directly (no
staging), with the same bytes as the staged path, for tight and strided rows,
in place, and for either side alone page-locked (register_host /
gcdr_host_register, or memory allocated pinned)."""
import numpy as np
import pytest

import golden_data as G

pytestmark = pytest.mark.gpu


def _aligned(nbytes):
    raw = np.empty(nbytes + 8192, np.uint8)
    off = (-raw.ctypes.data) % 4096
    return raw[off:off + nbytes]


def _doc(w, h, fmt, stride):
    from sdcb.gcdrnet_b200 import synth
    bpp = 4 if fmt >= 2 else 3
    px = synth.document(w, h, seed=5, fmt=fmt, strokes=30)
    buf = _aligned(h * stride)
    buf[:] = 0x5A
    buf.reshape(h, stride)[:, :w * bpp] = px.reshape(h, w * bpp)
    return buf


@pytest.mark.parametrize("fmt,pad", [(0, 0), (2, 64), (3, 7)])
def test_pinned_buffers_match_staged(fmt, pad):
    from sdcb.gcdrnet_b200 import GcdrEnhancer, register_host, unregister_host
    w, h = 301, 203
    bpp = 4 if fmt >= 2 else 3
    stride = w * bpp + pad
    src = _doc(w, h, fmt, stride)
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        want = np.full_like(src, 0x5A)
        enh.enhance(src, w, h, stride, want, stride, fmt)                 # pageable: staged
        for pin_src, pin_dst in ((True, True), (True, False), (False, True)):
            s = _aligned(src.size)
            s[:] = src
            d = _aligned(src.size)
            d[:] = 0x5A
            if pin_src:
                register_host(s)
            if pin_dst:
                register_host(d)
            try:
                enh.enhance(s, w, h, stride, d, stride, fmt)
            finally:
                if pin_src:
                    unregister_host(s)
                if pin_dst:
                    unregister_host(d)
            assert np.array_equal(d, want), f"pinned src {pin_src} dst {pin_dst}"
            assert np.array_equal(s, src), "source modified"
        # in place on a page-locked buffer (the destination is written after the device flag)
        io = _aligned(src.size)
        io[:] = src
        register_host(io)
        try:
            enh.enhance(io, w, h, stride, io, stride, fmt)
        finally:
            unregister_host(io)
        assert np.array_equal(io, want), "pinned in place"


def test_allocated_pinned_memory_is_used_directly():
    import torch
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    w, h = 256, 160
    src = _doc(w, h, 0, w * 3)
    ps = torch.empty(src.size, dtype=torch.uint8, pin_memory=True).numpy()
    pd = torch.empty(src.size, dtype=torch.uint8, pin_memory=True).numpy()
    ps[:] = src
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        want = np.empty_like(src)
        enh.enhance(src, w, h, w * 3, want, w * 3, 0)
        enh.enhance(ps, w, h, w * 3, pd, w * 3, 0)
    assert np.array_equal(pd, want)
