"""Seeded synthetic document images (the benchmark inputs).

Stand-in for the reference's RealDAE corpus methodology (docs/corpus.md),
which is not available here.  Recipe, per image and seed:
  1. paper background, one U(200, 240) level per channel;
  2. times a smooth shading field: a 4x4 grid of U(0.35, 1.0) gains,
     bicubically upsampled to the image;
  3. about 200 dark strokes along random quadratic Bezier paths, value
     U(10, 60), width 2-6 px;
  4. plus N(0, 3) noise, clamped to [0, 255].
Returns tight interleaved u8 in the requested GcdrPixelFormat (alpha, for
4-byte formats, is U(0, 255) per pixel).
"""
from __future__ import annotations

import numpy as np


def _cubic_weights(n: int, cells: int) -> np.ndarray:
    """[n][cells] weights of bicubic (Keys, a = -0.5) interpolation of `cells` grid nodes
    spread over n pixels (node k at pixel (k + 0.5) * n / cells - 0.5), edge-clamped."""
    t = (np.arange(n, dtype=np.float64) + 0.5) * cells / n - 0.5
    i0 = np.floor(t).astype(np.int64)
    wts = np.zeros((n, cells))
    for k in range(-1, 3):
        d = np.abs(t - (i0 + k))
        kw = np.where(d <= 1, (1.5 * d - 2.5) * d * d + 1,
                      np.where(d < 2, ((-0.5 * d + 2.5) * d - 4) * d + 2, 0.0))
        np.add.at(wts, (np.arange(n), np.clip(i0 + k, 0, cells - 1)), kw)
    return wts


def _bicubic_field(gains: np.ndarray, h: int, w: int) -> np.ndarray:
    """The 4x4 gain grid bicubically upsampled to h x w (separable: two small matrix products)."""
    return _cubic_weights(h, gains.shape[0]) @ gains @ _cubic_weights(w, gains.shape[1]).T


def document(width: int = 1600, height: int = 1152, seed: int = 0, fmt: int = 0, strokes: int = 200) -> np.ndarray:
    return _render(width, height, seed, fmt, strokes)[0]


CLEAN_PAPER = 250.0   # the ground-truth page of document_pair: flat, no shading, no noise


def document_pair(width: int, height: int, seed: int = 0, strokes: int = 200):
    """(degraded, clean) Bgr24 pages of one seed: document(width, height, seed) and the same
    strokes, unshaded, on a flat CLEAN_PAPER page without noise (a ground truth in the
    corpus harness's layout)."""
    return _render(width, height, seed, 0, strokes, clean=True)


def _render(width, height, seed, fmt, strokes, clean=False):
    rng = np.random.default_rng(seed)
    paper = rng.uniform(200, 240, 3)
    gains = rng.uniform(0.35, 1.0, (4, 4))
    shade = _bicubic_field(gains, height, width).astype(np.float32)
    img = np.empty((height, width, 3), np.float32)
    for c in range(3):
        img[:, :, c] = paper[c] * shade
    ys_all, xs_all, vs_all = [], [], []
    for _ in range(strokes):
        p = rng.uniform([0, 0], [height, width], (3, 2))
        val = rng.uniform(10, 60)
        r = rng.uniform(2, 6) / 2.0
        length = np.linalg.norm(p[1] - p[0]) + np.linalg.norm(p[2] - p[1])
        n = max(8, int(length / max(r, 1.0)))
        t = np.linspace(0, 1, n)[:, None]
        pts = (1 - t) ** 2 * p[0] + 2 * (1 - t) * t * p[1] + t ** 2 * p[2]
        ir = int(np.ceil(r))
        oy, ox = np.mgrid[-ir:ir + 1, -ir:ir + 1]
        m = oy ** 2 + ox ** 2 <= r * r
        oy, ox = oy[m], ox[m]
        yy = (np.round(pts[:, 0])[:, None] + oy[None, :]).ravel().astype(np.int64)
        xx = (np.round(pts[:, 1])[:, None] + ox[None, :]).ravel().astype(np.int64)
        keep = (yy >= 0) & (yy < height) & (xx >= 0) & (xx < width)
        ys_all.append(yy[keep])
        xs_all.append(xx[keep])
        vs_all.append(np.full(keep.sum(), val, np.float32))
    gt = None
    if ys_all:
        ys, xs, vs = np.concatenate(ys_all), np.concatenate(xs_all), np.concatenate(vs_all)
        img[ys, xs, :] = vs[:, None] * shade[ys, xs][:, None]
    if clean:
        gt = np.full((height, width, 3), CLEAN_PAPER, np.float32)
        if ys_all:
            gt[ys, xs, :] = vs[:, None]
        gt = np.ascontiguousarray(np.clip(np.rint(gt), 0, 255).astype(np.uint8))
    img += rng.standard_normal(img.shape, dtype=np.float32) * np.float32(3.0)
    bgr = np.clip(np.rint(img), 0, 255).astype(np.uint8)
    if fmt in (1, 3):
        bgr = bgr[:, :, ::-1]
    if fmt >= 2:
        a = rng.integers(0, 256, (height, width, 1), dtype=np.uint8)
        bgr = np.concatenate([bgr, a], axis=2)
    return np.ascontiguousarray(bgr), gt


class DocumentMaker:
    """document(width, height, seed=i, fmt) as a picklable callable of i (worker processes)."""

    def __init__(self, width: int = 1600, height: int = 1152, fmt: int = 0):
        self.width, self.height, self.fmt = width, height, fmt

    def __call__(self, i: int) -> np.ndarray:
        return document(self.width, self.height, seed=int(i), fmt=self.fmt)
