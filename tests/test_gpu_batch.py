"""Batched images per launch: n same-shape images in one CUDA-graph launch
(gcdr_cuda_enhance_batch / _batch_device), each kernel of the graph covering all
n images, give the same bytes as n single enhancements, in every pixel format,
strided and in place.  The reference does not batch (README.md:182); the
per-image results are the contract it defines (GcdrEnhancer.cs:181-271)."""
import numpy as np
import pytest

import golden_data as G

pytestmark = pytest.mark.gpu


def _docs(n, w, h, fmt, stride, seed0=40):
    from sdcb.gcdrnet_b200 import synth
    bpp = 4 if fmt >= 2 else 3
    out = []
    for k in range(n):
        px = synth.document(w, h, seed=seed0 + k, fmt=fmt, strokes=25)
        buf = np.full((h, stride), 0x5A, np.uint8)
        buf[:, :w * bpp] = px.reshape(h, w * bpp)
        out.append(buf.reshape(-1))
    return out


@pytest.mark.parametrize("n,w,h,fmt,pad", [(3, 217, 150, 0, 0), (4, 160, 96, 2, 64), (2, 301, 203, 3, 5),
                                           (5, 45, 37, 1, 3), (16, 64, 64, 0, 0)])
def test_batch_matches_single_images(n, w, h, fmt, pad):
    from sdcb.gcdrnet_b200 import CudaWorker
    bpp = 4 if fmt >= 2 else 3
    stride = w * bpp + pad
    srcs = _docs(n, w, h, fmt, stride)
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        want = []
        for s in srcs:
            d = np.full_like(s, 0x5A)
            wk.enhance(s, w, h, stride, d, stride, fmt)
            want.append(d)
        dsts = [np.full_like(s, 0x5A) for s in srcs]
        wk.enhance_batch(srcs, w, h, stride, dsts, stride, fmt)
        for k in range(n):
            assert np.array_equal(dsts[k], want[k]), f"image {k} of the batch"
        caps = wk.plan_stats[0]
        # one launch per layer for the whole batch: as many kernels as one image's graph
        batch_launches = wk.launch_count
        wk.enhance(srcs[0], w, h, stride, np.empty_like(srcs[0]), stride, fmt)
        single_launches = wk.launch_count
        assert batch_launches == single_launches, (batch_launches, single_launches)
        # in place, a second time: the batch plan is cached (no capture)
        io = [s.copy() for s in srcs]
        wk.enhance_batch(io, w, h, stride, io, stride, fmt)
        for k in range(n):
            assert np.array_equal(io[k], want[k]), f"in place, image {k}"
        assert wk.plan_stats[0] == caps


def test_batch_device_matches_single():
    import torch
    from sdcb.gcdrnet_b200 import CudaWorker
    n, w, h = 4, 640, 480
    srcs = _docs(n, w, h, 0, w * 3, seed0=70)
    dev = torch.device("cuda:0")
    d_src = [torch.from_numpy(s).to(dev) for s in srcs]
    d_one = [torch.empty_like(t) for t in d_src]
    d_bat = [torch.empty_like(t) for t in d_src]
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        for k in range(n):
            wk.enhance_device(d_src[k].data_ptr(), w, h, d_one[k].data_ptr(), 0)
        torch.cuda.synchronize()
        wk.enhance_batch_device([t.data_ptr() for t in d_src], w, h, [t.data_ptr() for t in d_bat], 0)
        torch.cuda.synchronize()
        assert wk.plan_stats == (2, 2), "a single-image plan and a batch plan"
    for k in range(n):
        assert torch.equal(d_one[k], d_bat[k]), f"image {k}"


def test_batch_full_size_matches_single():
    """Two 1600x1152 documents in one batched graph (the shapes of the throughput workload)."""
    from sdcb.gcdrnet_b200 import CudaWorker
    n, w, h = 2, 1600, 1152
    srcs = _docs(n, w, h, 0, w * 3, seed0=90)
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        want = []
        for s in srcs:
            d = np.empty_like(s)
            wk.enhance(s, w, h, w * 3, d, w * 3, 0)
            want.append(d)
        dsts = [np.empty_like(s) for s in srcs]
        wk.enhance_batch(srcs, w, h, w * 3, dsts, w * 3, 0)
    for k in range(n):
        assert np.array_equal(dsts[k], want[k]), f"image {k}"


def test_batch_rejects_bad_sizes():
    from sdcb.gcdrnet_b200 import ArgumentError, CudaWorker
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        srcs = _docs(17, 32, 32, 0, 96)
        with pytest.raises(ArgumentError):
            wk.enhance_batch(srcs, 32, 32, 96, [s.copy() for s in srcs], 96, 0)


def test_enhancer_batch_matches_enhance():
    """The pooled enhancer's batch entry (gcdr_enhancer_enhance_batch): per image the bytes of
    GcdrEnhancer.Enhance, strided and in place; argument errors as Enhance reports them."""
    from sdcb.gcdrnet_b200 import ArgumentError, GcdrEnhancer
    n, w, h, fmt = 3, 250, 170, 2
    stride = w * 4 + 12
    srcs = _docs(n, w, h, fmt, stride, seed0=120)
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        want = []
        for s in srcs:
            d = np.full_like(s, 0x5A)
            enh.enhance(s, w, h, stride, d, stride, fmt)
            want.append(d)
        dsts = [np.full_like(s, 0x5A) for s in srcs]
        enh.enhance_batch(srcs, w, h, stride, dsts, stride, fmt)
        for k in range(n):
            assert np.array_equal(dsts[k], want[k]), f"image {k}"
        io = [s.copy() for s in srcs]
        enh.enhance_batch(io, w, h, stride, io, stride, fmt)
        for k in range(n):
            assert np.array_equal(io[k], want[k]), f"in place, image {k}"
        with pytest.raises(ArgumentError):
            enh.enhance_batch(srcs, w, h, stride, [dsts[0], dsts[1][:stride * (h - 1)], dsts[2]], stride, fmt)
        with pytest.raises(ArgumentError):
            enh.enhance_batch(srcs * 6, w, h, stride, dsts * 6, stride, fmt)


def test_batch_with_per_image_ops_matches_single(monkeypatch):
    """With the fp32 SIMT stem and head (GCDR_CUDA_STEM=simt), which run once per image, the
    batch plan interleaves those per-image launches with the batched ones in plan order: each
    image still gets the single-image bytes."""
    from sdcb.gcdrnet_b200 import CudaWorker
    monkeypatch.setenv("GCDR_CUDA_STEM", "simt")
    n, w, h = 3, 200, 130
    srcs = _docs(n, w, h, 0, w * 3, seed0=150)
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        want = []
        for s in srcs:
            d = np.empty_like(s)
            wk.enhance(s, w, h, w * 3, d, w * 3, 0)
            want.append(d)
        single_launches = wk.launch_count
        dsts = [np.empty_like(s) for s in srcs]
        wk.enhance_batch(srcs, w, h, w * 3, dsts, w * 3, 0)
        # the per-image kernels (two stems, two heads) run n times, the rest once
        assert wk.launch_count == single_launches + (n - 1) * 4, (wk.launch_count, single_launches)
    for k in range(n):
        assert np.array_equal(dsts[k], want[k]), f"image {k}"


def test_concurrent_enhance_calls_are_batched():
    """Concurrent GcdrEnhancer.enhance calls of one shape run as batched launches (fewer worker
    launches than calls); every call gets the bytes of a single-image enhance.  With batching
    off (max_batch 1) every call is its own launch."""
    import threading
    from sdcb.gcdrnet_b200 import CudaWorker, GcdrEnhancer
    threads, per, w, h = 8, 4, 320, 224
    docs = _docs(threads * per, w, h, 0, w * 3, seed0=200)
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        want = []
        for s in docs:
            d = np.empty_like(s)
            wk.enhance(s, w, h, w * 3, d, w * 3, 0)
            want.append(d)
    for max_batch in (8, 1):
        got = [np.empty_like(s) for s in docs]
        errors = []
        with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
            enh.set_batching(max_batch, 1)   # one launch at a time: the other calls queue behind it
            enh.enhance(docs[0], w, h, w * 3, got[0], w * 3, 0)   # plans the shape
            go = threading.Barrier(threads)

            def run(t):
                try:
                    go.wait()
                    for i in range(t, len(docs), threads):
                        enh.enhance(docs[i], w, h, w * 3, got[i], w * 3, 0)
                except Exception as ex:   # surfaced below
                    errors.append(repr(ex))

            th = [threading.Thread(target=run, args=(t,)) for t in range(threads)]
            for t in th:
                t.start()
            for t in th:
                t.join()
            calls, launches = enh.batch_stats
        assert not errors, errors[:3]
        for i in range(len(docs)):
            assert np.array_equal(got[i], want[i]), f"max_batch {max_batch}: document {i}"
        assert calls == len(docs) + 1
        if max_batch == 1:
            assert launches == calls
        else:
            assert launches < calls, (calls, launches)


def test_batched_calls_two_shapes_and_device_loss():
    """Concurrent enhance calls of two shapes (two lanes) while the first worker run reports a
    device loss (injected on the host): the batch that met it is retried on a fresh pool, and
    every call returns its single-image bytes."""
    import threading
    from sdcb.gcdrnet_b200 import CudaWorker, GcdrEnhancer
    shapes = [(256, 160), (192, 224)]
    docs = {s: _docs(6, s[0], s[1], 0, s[0] * 3, seed0=300 + 10 * k) for k, s in enumerate(shapes)}
    want = {}
    with CudaWorker.from_files(G.GC_PATH, G.DR_PATH) as wk:
        for s in shapes:
            for i, d in enumerate(docs[s]):
                out = np.empty_like(d)
                wk.enhance(d, s[0], s[1], s[0] * 3, out, s[0] * 3, 0)
                want[s, i] = out
    got, errors = {}, []
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        enh.set_batching(4, 1)
        evicted0 = enh.pool_stats[2]
        enh.inject_device_loss(1)
        go = threading.Barrier(6)

        def run(t):
            try:
                go.wait()
                s = shapes[t % 2]
                for i in range(t // 2, 6, 3):
                    out = np.empty_like(docs[s][i])
                    enh.enhance(docs[s][i], s[0], s[1], s[0] * 3, out, s[0] * 3, 0)
                    got[s, i] = out
            except Exception as ex:   # surfaced below
                errors.append(repr(ex))

        th = [threading.Thread(target=run, args=(t,)) for t in range(6)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert enh.pool_stats[2] > evicted0, "the pool that met the device loss was dropped"
    assert not errors, errors[:3]
    assert set(got) == set(want)
    for key in want:
        assert np.array_equal(got[key], want[key]), f"{key}"
