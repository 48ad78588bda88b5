"""The per-shape plan cache of a worker: up to 8 image shapes keep their arena,
op sequence and CUDA graph, least recently used evicted first.

Mirrors the reference's per-size cache (GcdrEnhancer.cs:45-46, 128-136: at
most 8 sizes, evicted beyond that) and its size-switch test
(tests/Sdcb.SimdGcdrNet.Tests/EngineTests.cs:183-243): alternating sizes give
the same bytes as a fresh enhancer, and here also capture one graph per shape
and worker, not one per switch.
"""
import time

import numpy as np
import pytest

import golden_data as G

pytestmark = pytest.mark.gpu


def _doc(w, h, fmt, seed):
    from sdcb.gcdrnet_b200 import synth
    return synth.document(w, h, seed=seed, fmt=fmt, strokes=20)


def _run(wk, img, w, h, fmt):
    bpp = 4 if fmt >= 2 else 3
    dst = np.zeros_like(img)
    wk.enhance(img, w, h, w * bpp, dst, w * bpp, fmt)
    return dst


SHAPES = [(217, 150, 0), (300, 200, 2), (96, 128, 3)]


def test_alternating_shapes_capture_once_each():
    from sdcb.gcdrnet_b200 import CudaWorker
    imgs = {s: _doc(s[0], s[1], s[2], seed=i) for i, s in enumerate(SHAPES)}
    fresh = {}
    for s in SHAPES:
        with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
            fresh[s] = _run(wk, imgs[s], *s)
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        for rnd in range(3):
            for s in SHAPES:
                assert np.array_equal(_run(wk, imgs[s], *s), fresh[s]), f"shape {s} round {rnd}"
        assert wk.plan_stats == (3, 3), wk.plan_stats
        # debug mode is part of the key: one more plan, and back without a capture
        wk.set_debug(True)
        _run(wk, imgs[SHAPES[0]], *SHAPES[0])
        wk.set_debug(False)
        assert np.array_equal(_run(wk, imgs[SHAPES[0]], *SHAPES[0]), fresh[SHAPES[0]])
        assert wk.plan_stats == (4, 4), wk.plan_stats


def test_least_recently_used_shape_is_evicted_beyond_eight():
    from sdcb.gcdrnet_b200 import CudaWorker
    shapes = [(64 + 32 * k, 64, 0) for k in range(9)]
    imgs = [_doc(w, h, f, seed=k) for k, (w, h, f) in enumerate(shapes)]
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        first = [_run(wk, im, *s) for im, s in zip(imgs, shapes)]
        assert wk.plan_stats == (9, 8)              # shape 0 was evicted
        _run(wk, imgs[8], *shapes[8])               # cached: no capture
        assert wk.plan_stats == (9, 8)
        again = _run(wk, imgs[0], *shapes[0])       # evicted: planned and captured again
        assert wk.plan_stats == (10, 8)
        assert np.array_equal(again, first[0])
        _run(wk, imgs[2], *shapes[2])               # still cached (shape 1 was the LRU one)
        assert wk.plan_stats == (10, 8)


def test_enhancer_second_pass_runs_from_cached_plans():
    """Odd large shapes (c4-like): the first pass plans and captures each shape, the second
    pass re-uses the one worker's cached plans and is faster."""
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    rng = np.random.default_rng(7)
    shapes = [(int(rng.integers(2000, 4097)), int(rng.integers(1500, 3073))) for _ in range(3)]
    imgs = [_doc(w, h, 3, seed=100 + k) for k, (w, h) in enumerate(shapes)]
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        times, outs = [], []
        for rep in range(2):
            t0 = time.perf_counter()
            outs.append([enh.enhance_image(im.ravel(), w, h, 3) for im, (w, h) in zip(imgs, shapes)])
            times.append(time.perf_counter() - t0)
        assert enh.pool_stats[1] == 1, "one worker serves every shape"
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    assert times[1] < 0.8 * times[0], f"second pass {times[1]:.3f} s vs first {times[0]:.3f} s"


def test_concurrent_callers_mixed_shapes_match_serial():
    """Four threads (the pool's idle capacity) share one enhancer and draw among three
    shapes: the pool rents workers holding the requested shape's plan or plans it, and every
    result equals the serial one (the kernels are deterministic).  The reference's concurrency test is
    EngineTests.cs:245-263 (one size)."""
    import threading
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    imgs = {s: _doc(s[0], s[1], s[2], seed=30 + i) for i, s in enumerate(SHAPES)}
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        want = {s: enh.enhance_image(imgs[s].ravel(), s[0], s[1], s[2]) for s in SHAPES}
        rng = np.random.default_rng(5)
        plan = [[SHAPES[j] for j in rng.integers(0, len(SHAPES), 12)] for _ in range(4)]
        errors = []

        def run(k):
            try:
                for s in plan[k]:
                    got = enh.enhance_image(imgs[s].ravel(), s[0], s[1], s[2])
                    if not np.array_equal(got, want[s]):
                        errors.append(f"thread {k} shape {s} differs")
            except Exception as ex:   # surfaced below
                errors.append(repr(ex))

        th = [threading.Thread(target=run, args=(k,)) for k in range(4)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert not errors, errors[:3]
        pools, workers, evicted = enh.pool_stats
        assert pools == 1 and evicted == 0 and 1 <= workers <= 4
