"""Command line: python -m sdcb.gcdrnet_b200 <command>

  enhance IN OUT [--gc M --dr M]        enhance an image file (PNG/JPEG via PIL)
  run [--width W --height H --iters N]  device-resident throughput of one worker
  prof [--width W --height H]           per-op profile (the GCDRNET_PROF analogue,
                                        bench/Sdcb.SimdGcdrNet.Benchmark/Program.cs:993-1010)
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
    import torch
    from . import CudaWorker, synth
    torch.cuda.set_device(a.device)
    img = synth.document(a.width, a.height, seed=0, fmt=a.format)
    src = torch.from_numpy(img.reshape(-1)).cuda()
    dst = torch.empty_like(src)
    wk = CudaWorker.from_files(*_models(a), device=a.device)
    return wk, src, dst


def cmd_run(a):
    import torch
    wk, src, dst = _worker_and_image(a)
    s = torch.cuda.Stream()
    for _ in range(2):
        wk.enhance_device(src.data_ptr(), a.width, a.height, dst.data_ptr(), a.format, s.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(a.iters):
        wk.enhance_device(src.data_ptr(), a.width, a.height, dst.data_ptr(), a.format, s.cuda_stream)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / a.iters
    print(f"{a.width}x{a.height} fmt {a.format}: {ms:.3f} ms/image, {1000 / ms:.1f} images/s, "
          f"{wk.launch_count} kernels/image")
    wk.close()


def cmd_prof(a):
    import torch
    wk, src, dst = _worker_and_image(a)
    wk.enhance_device(src.data_ptr(), a.width, a.height, dst.data_ptr(), a.format, 0)
    torch.cuda.synchronize()
    prof = wk.profile(reps=a.iters)
    tot = sum(p[1] for p in prof)
    print(f"{'op':26s} {'us':>9s} {'share':>6s} {'GFLOP':>8s} {'MB':>8s} {'TFLOP/s':>8s} {'GB/s':>8s}")
    for name, ms, fl, by, tc in prof:
        print(f"{name:26s} {ms * 1000:9.1f} {100 * ms / tot:5.1f}% {fl / 1e9:8.3f} {by / 1e6:8.2f} "
              f"{fl / (ms * 1e-3) / 1e12 if ms else 0:8.2f} {by / (ms * 1e-3) / 1e9 if ms else 0:8.1f}{'  tc' if tc else ''}")
    print(f"total {tot * 1000:.1f} us")
    wk.close()


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m sdcb.gcdrnet_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("enhance", "run", "prof"):
        p = sub.add_parser(name)
        p.add_argument("--gc")
        p.add_argument("--dr")
        p.add_argument("--device", type=int, default=0)
        if name == "enhance":
            p.add_argument("input")
            p.add_argument("output")
        else:
            p.add_argument("--width", type=int, default=1600)
            p.add_argument("--height", type=int, default=1152)
            p.add_argument("--format", type=int, default=0)
            p.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    {"enhance": cmd_enhance, "run": cmd_run, "prof": cmd_prof}[a.cmd](a)
    return 0


if __name__ == "__main__":
    sys.exit(main())
