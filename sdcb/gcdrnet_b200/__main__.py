"""Command line: python -m sdcb.gcdrnet_b200 <command>

  enhance IN OUT [--gc M --dr M]        enhance an image file (PNG/JPEG via PIL)
  run [--width W --height H --iters N]  device-resident throughput of one worker
  prof [--width W --height H]           per-op profile (the GCDRNET_PROF analogue,
                                        bench/Sdcb.SimdGcdrNet.Benchmark/Program.cs:993-1010)
  microbench [--iters N]                isolated 3x3 conv + bias + relu layers of the GC/DR
                                        pyramid at 1600x1152 through the layer entry gcdr_k_conv
  batch [--count N]                     64 (N) Bgra32 1600x1152 documents enhanced in place with
                                        row stride width*4+64 through GcdrEnhancer (host buffers)
  corpus DIR [--mode smoke|bench] [--count N] [--synthetic]
                                        corpus harness (manifest.json + NN_<kind> / NN_gt images):
                                        PSNR against the ground truths, determinism, cold timing
  stress [--count N]                    odd-size Rgba32 documents (w 2000-4096, h 1500-3072,
                                        seed 7): first pass (plan + graph capture per shape) and
                                        a second pass (parity: tests/test_gpu_configs.py)
Models default to the copies under tests/golden/models.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
_MODELS = os.path.join(_ROOT, "tests", "golden", "models")


def _models(a):
    gc = a.gc or os.path.join(_MODELS, "gcdrnet_gcnet_sim.onnx")
    dr = a.dr or os.path.join(_MODELS, "gcdrnet_drnet_sim.onnx")
    return gc, dr


def cmd_enhance(a):
    import numpy as np
    from PIL import Image
    from . import GcdrEnhancer, GcdrPixelFormat
    im = Image.open(a.input).convert("RGB")
    rgb = np.ascontiguousarray(np.asarray(im, np.uint8))
    h, w, _ = rgb.shape
    with GcdrEnhancer.from_files(*_models(a), device=a.device) as enh:
        out = enh.enhance_image(rgb, w, h, GcdrPixelFormat.Rgb24).reshape(h, w, 3)
    Image.fromarray(out).save(a.output)
    print(f"{a.input} -> {a.output} ({w}x{h})")


def _worker_and_image(a):
    """A worker and a.batch device-resident documents (seeds 0..) with their outputs."""
    import torch
    from . import CudaWorker, synth
    torch.cuda.set_device(a.device)
    srcs = [torch.from_numpy(synth.document(a.width, a.height, seed=k, fmt=a.format).reshape(-1)).cuda()
            for k in range(a.batch)]
    dsts = [torch.empty_like(s) for s in srcs]
    wk = CudaWorker.from_files(*_models(a), device=a.device)
    return wk, srcs, dsts


def _launch(wk, a, srcs, dsts, stream):
    """One enhancement of the documents: a single-image launch, or one batched launch."""
    if a.batch == 1:
        wk.enhance_device(srcs[0].data_ptr(), a.width, a.height, dsts[0].data_ptr(), a.format, stream)
    else:
        wk.enhance_batch_device([s.data_ptr() for s in srcs], a.width, a.height, [d.data_ptr() for d in dsts],
                                a.format, stream)


def cmd_run(a):
    import torch
    wk, srcs, dsts = _worker_and_image(a)
    s = torch.cuda.Stream()
    for _ in range(2):
        _launch(wk, a, srcs, dsts, s.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(a.iters):
        _launch(wk, a, srcs, dsts, s.cuda_stream)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters / a.batch
    print(f"{a.width}x{a.height} fmt {a.format}, {a.batch} per launch: {ms:.3f} ms/image, {1000 / ms:.1f} images/s, "
          f"{wk.launch_count} kernels/launch")
    wk.close()


def cmd_prof(a):
    import torch
    wk, srcs, dsts = _worker_and_image(a)
    _launch(wk, a, srcs, dsts, 0)
    torch.cuda.synchronize()
    prof = wk.profile(reps=a.iters)
    tot = sum(p[1] for p in prof)
    print(f"{'op':26s} {'us':>9s} {'share':>6s} {'GFLOP':>8s} {'MB':>8s} {'TFLOP/s':>8s} {'GB/s':>8s}")
    for name, ms, fl, by, tc in prof:
        print(f"{name:26s} {ms * 1000:9.1f} {100 * ms / tot:5.1f}% {fl / 1e9:8.3f} {by / 1e6:8.2f} "
              f"{fl / (ms * 1e-3) / 1e12 if ms else 0:8.2f} {by / (ms * 1e-3) / 1e9 if ms else 0:8.1f}{'  tc' if tc else ''}")
    print(f"total {tot * 1000:.1f} us")
    wk.close()


def _peaks():
    import json
    p = os.path.join(_ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            d = json.load(fh)
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0)
    except OSError:
        return 6650.0, 1590.0


# (label, kind, H, W, Cin, N): kind 3 = 3x3 zero-pad stride 1, kind 2 = 1x1.  Channel
# counts below 16 are zero-padded to 16 for the tensor cores; FLOPs and bytes count the
# real channels.
_MICRO = [
    ("6->32 3x3 @1152x1600", 3, 1152, 1600, 6, 32),
    ("32->64 3x3 @576x800", 3, 576, 800, 32, 64),
    ("64->128 3x3 @288x400", 3, 288, 400, 64, 128),
    ("128->256 3x3 @144x200", 3, 144, 200, 128, 256),
    ("256->256 3x3 @72x100", 3, 72, 100, 256, 256),
    ("1x1 256->3 @1152x1600", 2, 1152, 1600, 256, 3),
]


def cmd_microbench(a):
    import ctypes
    import torch
    import numpy as np
    from . import ConvDesc, lib
    L = lib()

    torch.cuda.set_device(a.device)
    dev = torch.device("cuda", a.device)
    hbm, tf = _peaks()
    g = torch.Generator(device="cpu").manual_seed(1)
    st = torch.cuda.Stream(dev)
    print(f"{'layer':24s} {'us':>8s} {'TFLOP/s':>8s} {'%bf16':>6s} {'GB/s':>8s} {'%HBM':>6s}")
    for label, kind, H, W, cin, n in _MICRO:
        C, N = max(16, (cin + 15) // 16 * 16), max(16, (n + 15) // 16 * 16)
        taps = 9 if kind == 3 else 1
        x = torch.zeros(H, W, C, dtype=torch.float16)
        x[:, :, :cin] = torch.randn(H, W, cin, generator=g)
        w = torch.zeros(N, taps, C)
        w[:n, :, :cin] = torch.randn(n, taps, cin, generator=g) * (2.0 / (cin * taps)) ** 0.5   # Kaiming normal
        xt = x.to(dev)
        wt = w.reshape(N, taps * C).to(dev, torch.float16)
        bt = torch.zeros(N, device=dev)
        if kind == 2:
            inp = xt
        else:
            cnt = L.gcdr_k_to_layout(None, H, W, C, 3, None, None)
            inp = torch.empty(cnt, dtype=torch.float16, device=dev)
            L.gcdr_k_to_layout(xt.data_ptr(), H, W, C, 3, inp.data_ptr(), None)
        out = torch.empty(H * W * N, dtype=torch.float16, device=dev)
        d = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), 2, out.data_ptr(), None, 1, 1)
        bias_host = np.zeros(N, np.float32)          # host copy of the bias: the calls only enqueue
        d.bias_host = bias_host.ctypes.data
        for _ in range(3):
            assert L.gcdr_k_conv(ctypes.byref(d), 0, ctypes.c_void_p(st.cuda_stream)) == 0
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(a.iters):
            L.gcdr_k_conv(ctypes.byref(d), 0, ctypes.c_void_p(st.cuda_stream))
        e1.record(st)
        torch.cuda.synchronize(dev)
        us = e0.elapsed_time(e1) * 1000 / a.iters
        flops = 2.0 * H * W * n * taps * cin
        byts = 2.0 * H * W * (cin + n) + 2.0 * n * taps * cin
        tfs, gbs = flops / (us * 1e-6) / 1e12, byts / (us * 1e-6) / 1e9
        print(f"{label:24s} {us:8.1f} {tfs:8.1f} {100 * tfs / tf:5.1f}% {gbs:8.1f} {100 * gbs / hbm:5.1f}%")


def cmd_batch(a):
    import numpy as np
    from . import GcdrEnhancer, GcdrPixelFormat, synth
    w, h = a.width, a.height
    stride = w * 4 + 64
    imgs = []
    for seed in range(a.count):
        px = synth.document(w, h, seed=seed, fmt=int(GcdrPixelFormat.Bgra32))
        buf = np.zeros(stride * h, np.uint8)
        buf.reshape(h, stride)[:, :w * 4] = px.reshape(h, w * 4)
        imgs.append(buf)
    alphas = [b.reshape(h, stride)[:, 3:w * 4:4].copy() for b in imgs]
    import threading
    with GcdrEnhancer.from_files(*_models(a), device=a.device) as enh:
        warm = [imgs[0].copy() for _ in range(a.threads)]

        def warm_one(k):
            enh.enhance(warm[k], w, h, stride, warm[k], stride, GcdrPixelFormat.Bgra32)

        th = [threading.Thread(target=warm_one, args=(k,)) for k in range(a.threads)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        lat = []

        def part(k):
            # the callers share the enhancer (its worker pool): one image's copies overlap another's kernels
            for i in range(k, len(imgs), a.threads):
                t = time.perf_counter()
                enh.enhance(imgs[i], w, h, stride, imgs[i], stride, GcdrPixelFormat.Bgra32)
                lat.append(time.perf_counter() - t)

        th = [threading.Thread(target=part, args=(k,)) for k in range(a.threads)]
        t0 = time.perf_counter()
        for t in th:
            t.start()
        for t in th:
            t.join()
        total = time.perf_counter() - t0
    ok = all(np.array_equal(b.reshape(h, stride)[:, 3:w * 4:4], al) for b, al in zip(imgs, alphas))
    lat.sort()
    print(f"{a.count} x {w}x{h} Bgra32 in place, stride {stride}, {a.threads} calling thread(s): "
          f"{a.count / total:.1f} images/s, e2e per call median {1000 * lat[len(lat) // 2]:.2f} ms, "
          f"max {1000 * lat[-1]:.2f} ms, alpha bit-exact: {ok}")


def cmd_stress(a):
    import numpy as np
    from . import GcdrEnhancer, GcdrPixelFormat, synth
    rng = np.random.default_rng(7)
    shapes = [(int(rng.integers(2000, 4097)), int(rng.integers(1500, 3073))) for _ in range(a.count)]
    fmt = int(GcdrPixelFormat.Rgba32)
    imgs = [synth.document(w, h, seed=100 + i, fmt=fmt, strokes=int(200 * w * h / (1600 * 1152)))
            for i, (w, h) in enumerate(shapes)]
    with GcdrEnhancer.from_files(*_models(a), device=a.device) as enh:
        outs = []
        for rep in range(2):
            lat = []
            t0 = time.perf_counter()
            for (w, h), im in zip(shapes, imgs):
                dst = np.empty_like(im)
                t = time.perf_counter()
                enh.enhance(im, w, h, w * 4, dst, w * 4, fmt)
                lat.append(time.perf_counter() - t)
                if rep == 0:
                    outs.append(dst)
            total = time.perf_counter() - t0
            mp = sum(w * h for w, h in shapes) / 1e6
            print(f"pass {rep + 1}: {len(shapes)} Rgba32 images ({mp:.1f} MP), {len(shapes) / total:.1f} images/s, "
                  f"{mp / total:.1f} MP/s, per image ms: " + " ".join(f"{1000 * t:.1f}" for t in lat))


def cmd_corpus(a):
    import json
    from . import GcdrEnhancer, corpus
    folder = a.folder
    if a.synthetic:
        sizes = [(640, 480), (1600, 1152), (1024, 768), (2000, 1500), (640, 480), (1280, 960)][: max(1, a.count)]
        corpus.write_synthetic(folder, sizes)
    with GcdrEnhancer.from_files(*_models(a), device=a.device) as enh:
        doc = corpus.run(enh, folder, a.mode, a.count, a.max_mp)
        doc["pool"] = dict(zip(("pools", "workers", "evicted"), enh.pool_stats))
    s = doc["summary"]
    print(f"corpus[{a.mode}] {s['timed']} timed, mean {s['meanMs']} ms, {s['mpPerSec']} MP/s"
          + (f", psnr {s['psnr']} dB (input {s['psnrIn']} dB)" if s["psnr"] is not None else ""))
    for e in doc["errors"]:
        print("FAIL", e, file=sys.stderr)
    if a.out:
        with open(a.out, "w") as fh:
            json.dump(doc, fh, indent=1)
    return 0 if doc["ok"] else 3


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m sdcb.gcdrnet_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("enhance", "run", "prof", "microbench", "batch", "stress", "corpus"):
        p = sub.add_parser(name)
        p.add_argument("--gc")
        p.add_argument("--dr")
        p.add_argument("--device", type=int, default=0)
        if name == "enhance":
            p.add_argument("input")
            p.add_argument("output")
        elif name == "corpus":
            p.add_argument("folder")
            p.add_argument("--mode", choices=("smoke", "bench"), default="smoke")
            p.add_argument("--count", type=int, default=5)
            p.add_argument("--max-mp", type=float, default=1e9)
            p.add_argument("--out")
            p.add_argument("--synthetic", action="store_true", help="first write seeded synthetic pairs into folder")
        elif name == "microbench":
            p.add_argument("--iters", type=int, default=20)
        elif name in ("batch", "stress"):
            p.add_argument("--count", type=int, default=64 if name == "batch" else 16)
            if name == "batch":
                p.add_argument("--threads", type=int, default=4)
            p.add_argument("--width", type=int, default=1600)
            p.add_argument("--height", type=int, default=1152)
        else:
            p.add_argument("--width", type=int, default=1600)
            p.add_argument("--height", type=int, default=1152)
            p.add_argument("--format", type=int, default=0)
            p.add_argument("--iters", type=int, default=10)
            if name in ("run", "prof"):
                p.add_argument("--batch", type=int, default=1, help="images per launch (a batch plan)")
    a = ap.parse_args(argv)
    rc = {"enhance": cmd_enhance, "run": cmd_run, "prof": cmd_prof, "microbench": cmd_microbench, "batch": cmd_batch,
          "stress": cmd_stress, "corpus": cmd_corpus}[a.cmd](a)
    return rc or 0


if __name__ == "__main__":
    sys.exit(main())
