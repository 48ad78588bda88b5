"""Host-side checks of the C ABI (no GPU): the library loads, exports every
entry point include/gcdr_cuda.h declares, and its ONNX reader recognises the
GCDRNet topology (the part of the reference's GraphCompiler + GCDR fusion
passes this backend needs) and rejects what it cannot run."""
import ctypes
import os
import re

import pytest

import golden_data as G

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gcdr_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"GCDR_API\s+[\w\s\*]+?\b(gcdr_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    syms = declared_symbols()
    assert len(syms) >= 25
    missing = [s for s in syms if not hasattr(L, s)]
    assert not missing, f"not exported: {missing}"


def test_model_topology_recognised():
    from sdcb.gcdrnet_b200 import describe_models
    d = describe_models(open(G.GC_PATH, "rb").read(), open(G.DR_PATH, "rb").read())
    assert d["gc"]["cin"] == 3 and d["gc"]["channels"] == [16, 32, 128, 160, 256]
    assert d["dr"]["cin"] == 6 and d["dr"]["channels"] == [32, 64, 128, 256, 512]
    for net, ends in (("gc", [[32, 64, 96, 128, 160], [32, 64, 96, 128, 160], [52, 104, 156, 208, 256]]),
                      ("dr", [[52, 104, 156, 208, 256], [52, 104, 156, 208, 256], [103, 206, 309, 412, 512]])):
        blocks = d[net]["blocks"]
        assert len(blocks) == 4
        for b in blocks:
            a, w = b["shifts"]
            assert a["axis"] == 2 and w["axis"] == 3            # shift along H, then W (gc#48, gc#99)
            assert a["offs"] == [2, 1, 0, -1, -2] == w["offs"]  # ChannelShiftOp.cs:158-161
        assert blocks[0]["shifts"][0]["ends"] == ends[0]
        assert blocks[1]["shifts"][0]["ends"] == ends[2]


def test_model_oracle_agrees_on_shift_groups(oracle):
    from sdcb.gcdrnet_b200 import describe_models
    d = describe_models(open(G.GC_PATH, "rb").read(), open(G.DR_PATH, "rb").read())
    for net, on in (("gc", oracle.gc), ("dr", oracle.dr)):
        for b, ob in zip(d[net]["blocks"], (on.block1, on.block2, on.dblock1, on.dblock2)):
            assert b["shifts"][0]["ends"] == ob.shift_h[1] and b["shifts"][0]["offs"] == ob.shift_h[2]
            assert b["shifts"][1]["ends"] == ob.shift_w[1] and b["shifts"][1]["offs"] == ob.shift_w[2]


def test_model_rejects_bad_inputs():
    from sdcb.gcdrnet_b200 import ModelError, NotSupportedError, describe_models
    gc, dr = open(G.GC_PATH, "rb").read(), open(G.DR_PATH, "rb").read()
    with pytest.raises(ModelError):
        describe_models(gc[:4096], dr)
    with pytest.raises(NotSupportedError):
        describe_models(dr, gc)            # nets swapped: 6-channel GC
    with pytest.raises((ModelError, NotSupportedError)):
        describe_models(b"\x08\x07" * 64, dr)


def test_enhancer_argument_validation_without_gpu():
    # argument checks run before any device work (GcdrEnhancer.cs:184-192)
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    err = ctypes.create_string_buffer(256)
    buf = (ctypes.c_uint8 * (32 * 32 * 4))()
    # a null enhancer handle is an argument error, never a crash
    assert L.gcdr_enhancer_enhance(None, buf, len(buf), 32, 32, 96, buf, len(buf), 128, 2, err, 256) == 1


def test_enhancer_batching_controls_without_gpu():
    """gcdr_enhancer_set_batching validates its limits and gcdr_enhancer_batch_stats counts
    nothing before the first call; creating an enhancer only parses the models (no device
    work), so this runs on CPU."""
    from sdcb.gcdrnet_b200 import lib
    L = lib()
    gc, dr = open(G.GC_PATH, "rb").read(), open(G.DR_PATH, "rb").read()
    h = ctypes.c_void_p()
    err = ctypes.create_string_buffer(256)
    assert L.gcdr_enhancer_create(0, gc, len(gc), dr, len(dr), 0, ctypes.byref(h), err, 256) == 0, err.value
    try:
        for bad in ((0, 1), (17, 1), (8, 0), (8, 65)):
            assert L.gcdr_enhancer_set_batching(h, *bad) == 1, bad
        assert L.gcdr_enhancer_set_batching(h, 1, 1) == 0          # batching off
        assert L.gcdr_enhancer_set_batching(h, 16, 64) == 0
        calls, launches = ctypes.c_int64(-1), ctypes.c_int64(-1)
        L.gcdr_enhancer_batch_stats(h, ctypes.byref(calls), ctypes.byref(launches))
        assert (calls.value, launches.value) == (0, 0)
        assert L.gcdr_enhancer_set_batching(None, 8, 3) == 1
    finally:
        L.gcdr_enhancer_destroy(h)
