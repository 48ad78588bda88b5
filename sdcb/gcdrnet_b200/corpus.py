"""Corpus harness: enhancement quality and cold per-image timing over a directory
of degraded images and their ground truths, in the reference's corpus layout
(docs/corpus.md; bench/Sdcb.SimdGcdrNet.Benchmark/CiRunner.cs):

    <dir>/manifest.json   {"images": [{"name": "01_color.webp", "w": W, "h": H}, ...]}
    <dir>/NN_<kind>.<ext> the degraded input
    <dir>/NN_gt.<ext>     its ground truth (optional; PSNR needs it)

Two modes, as the reference's `--ci smoke|bench`:

  smoke  correctness: every output differs from its input and is not flat, a
         second run gives the same bytes (determinism), and the enhanced images
         are closer to their ground truths than the inputs (mean PSNR).
  bench  timing: `count` images spread evenly over the manifest; the first warms
         up untimed, every other is timed once, cold (a new shape's plan and graph
         capture included), decoding excluded.

The RealDAE corpus itself is not in this repository; `write_synthetic` makes a
corpus of seeded synthetic document pairs in the same layout (a shaded, noisy
page and its clean page) for tests and for runs without the dataset.
"""
from __future__ import annotations

import json
import os
import time

import numpy as np


def psnr(a: np.ndarray, b: np.ndarray) -> float:
    """PSNR in dB of two u8 buffers of the same size (inf when equal)."""
    d = a.astype(np.float64) - b.astype(np.float64)
    se = float(np.mean(d * d))
    return float("inf") if se == 0 else 10.0 * np.log10(255.0 * 255.0 / se)


def read_manifest(folder: str) -> list:
    with open(os.path.join(folder, "manifest.json")) as fh:
        return [(e["name"], int(e["w"]), int(e["h"])) for e in json.load(fh)["images"]]


def select(images: list, count: int, max_mp: float = 1e9) -> list:
    """`count` images spread evenly over the manifest (after the --max-mp filter)."""
    pool = [e for e in images if e[1] * e[2] <= max_mp * 1e6]
    if not pool:
        return []
    count = max(1, min(count, len(pool)))
    return [pool[k * len(pool) // count] for k in range(count)]


def gt_name(name: str) -> str:
    stem, ext = os.path.splitext(name)
    return stem[:stem.index("_")] + "_gt" + ext if "_" in stem else stem + "_gt" + ext


def decode_bgr(path: str) -> np.ndarray:
    from PIL import Image
    rgb = np.asarray(Image.open(path).convert("RGB"), dtype=np.uint8)
    return np.ascontiguousarray(rgb[:, :, ::-1])


def run(enhancer, folder: str, mode: str = "smoke", count: int = 5, max_mp: float = 1e9, log=print) -> dict:
    """Runs the corpus through `enhancer` (a GcdrEnhancer); returns the result document
    (per-image rows, a summary, ok and errors) the reference's CI runner writes."""
    if mode not in ("smoke", "bench"):
        raise ValueError("mode must be smoke or bench")
    images = select(read_manifest(folder), count, max_mp)
    rows, errors = [], []
    psnr_in, psnr_out = [], []
    timed_ms, timed_mp = 0.0, 0.0
    for i, (name, w, h) in enumerate(images):
        src = decode_bgr(os.path.join(folder, name))
        if src.shape[:2] != (h, w):
            errors.append(f"{name}: decoded {src.shape[1]}x{src.shape[0]}, manifest {w}x{h}")
            continue
        out = np.empty_like(src)
        t0 = time.perf_counter()
        enhancer.enhance(src, w, h, w * 3, out, w * 3, 0)
        ms = (time.perf_counter() - t0) * 1000.0
        row = {"name": name, "w": w, "h": h, "ms": round(ms, 2)}
        warm = mode == "bench" and i == 0
        if warm:
            row["warmup"] = True
        else:
            timed_ms += ms
            timed_mp += w * h / 1e6
        gpath = os.path.join(folder, gt_name(name))
        if os.path.exists(gpath):
            gt = decode_bgr(gpath)
            if gt.shape == src.shape:
                pi, po = psnr(src, gt), psnr(out, gt)
                row["psnrIn"], row["psnr"] = round(pi, 2), round(po, 2)
                psnr_in.append(pi)
                psnr_out.append(po)
        if mode == "smoke":
            if np.array_equal(out, src):
                errors.append(f"{name}: output identical to input")
            if float(out.std()) <= 1.0:
                errors.append(f"{name}: output std {out.std():.2f} looks degenerate")
            again = np.empty_like(src)
            enhancer.enhance(src, w, h, w * 3, again, w * 3, 0)
            if not np.array_equal(again, out):
                errors.append(f"{name}: second run differs from the first (nondeterministic)")
        rows.append(row)
        if log:
            log(f"{name:18s} {w:5d}x{h:<5d} {ms:9.1f} ms{' (warmup)' if warm else ''}"
                + (f"  psnr {row['psnr']} dB (input {row['psnrIn']} dB)" if "psnr" in row else ""))
    if mode == "smoke" and psnr_out and sum(psnr_out) <= sum(psnr_in):
        errors.append(f"enhanced images are not closer to their ground truths: mean PSNR "
                      f"{np.mean(psnr_out):.2f} dB vs input {np.mean(psnr_in):.2f} dB")
    timed = sum(1 for r in rows if not r.get("warmup"))
    return {
        "kind": mode, "images": rows, "ok": not errors, "errors": errors,
        "summary": {"images": len(rows), "timed": timed, "totalMs": round(timed_ms, 2),
                    "meanMs": round(timed_ms / timed, 2) if timed else None,
                    "mpPerSec": round(timed_mp / (timed_ms / 1000.0), 3) if timed_ms else None,
                    "psnr": round(float(np.mean(psnr_out)), 2) if psnr_out else None,
                    "psnrIn": round(float(np.mean(psnr_in)), 2) if psnr_in else None},
    }


def write_synthetic(folder: str, sizes: list, seed0: int = 500, lossless: bool = True) -> list:
    """Writes seeded synthetic pairs into `folder` in the corpus layout: NN_shadow.webp (the
    document generator's shaded, noisy page) and NN_gt.webp (the same strokes on a flat,
    clean page), plus manifest.json.  Returns the manifest entries."""
    from PIL import Image
    from . import synth
    os.makedirs(folder, exist_ok=True)
    entries = []
    for k, (w, h) in enumerate(sizes):
        strokes = max(10, int(200 * w * h / (1600 * 1152)))    # the benchmark page's stroke density
        degraded, clean = synth.document_pair(w, h, seed=seed0 + k, strokes=strokes)
        nn = f"{k + 1:02d}"
        for name, img in ((f"{nn}_shadow.webp", degraded), (f"{nn}_gt.webp", clean)):
            Image.fromarray(np.ascontiguousarray(img[:, :, ::-1])).save(os.path.join(folder, name), lossless=lossless)
        entries.append({"name": f"{nn}_shadow.webp", "w": w, "h": h})
    with open(os.path.join(folder, "manifest.json"), "w") as fh:
        json.dump({"images": entries}, fh, indent=1)
    return entries
