"""The corpus harness (sdcb/gcdrnet_b200/corpus.py): the reference's corpus
layout and CI checks (docs/corpus.md, bench/Sdcb.SimdGcdrNet.Benchmark/CiRunner.cs)
on seeded synthetic pairs (the RealDAE corpus is not in this repository)."""
import os

import numpy as np
import pytest

import golden_data as G
from sdcb.gcdrnet_b200 import corpus, synth


def test_layout_selection_and_psnr(tmp_path):
    folder = str(tmp_path / "c")
    entries = corpus.write_synthetic(folder, [(96, 64), (120, 80), (64, 64)])
    assert corpus.read_manifest(folder) == [(e["name"], e["w"], e["h"]) for e in entries]
    assert corpus.gt_name("01_shadow.webp") == "01_gt.webp"
    # lossless pages round-trip exactly
    deg, clean = synth.document_pair(120, 80, seed=501, strokes=10)
    assert np.array_equal(corpus.decode_bgr(os.path.join(folder, "02_shadow.webp")), deg)
    assert np.array_equal(corpus.decode_bgr(os.path.join(folder, "02_gt.webp")), clean)
    # evenly spread selection and the --max-mp filter
    imgs = [(f"{k:02d}_x.webp", 10, 10) for k in range(10)]
    assert [n for n, *_ in corpus.select(imgs, 3)] == ["00_x.webp", "03_x.webp", "06_x.webp"]
    assert corpus.select(imgs, 3, max_mp=1e-5) == []
    a = np.zeros(100, np.uint8)
    assert corpus.psnr(a, a) == float("inf")
    assert abs(corpus.psnr(a, a + 1) - 48.13) < 0.01      # 20 log10(255)


def test_synthetic_pair_is_the_document_and_a_flat_page():
    deg, clean = synth.document_pair(160, 120, seed=9, strokes=15)
    assert np.array_equal(deg, synth.document(160, 120, seed=9, strokes=15))
    bg = clean[clean == synth.CLEAN_PAPER]
    assert bg.size > 0.5 * clean.size


@pytest.mark.gpu
def test_smoke_and_bench_on_synthetic_pairs(tmp_path):
    from sdcb.gcdrnet_b200 import GcdrEnhancer
    folder = str(tmp_path / "c")
    corpus.write_synthetic(folder, [(320, 240), (480, 352), (320, 240), (257, 199)])
    with GcdrEnhancer.from_files(G.GC_PATH, G.DR_PATH) as enh:
        smoke = corpus.run(enh, folder, "smoke", count=4, log=None)
        bench = corpus.run(enh, folder, "bench", count=4, log=None)
    assert smoke["ok"], smoke["errors"]
    assert smoke["summary"]["psnr"] > smoke["summary"]["psnrIn"]   # enhanced pages are closer to the clean ones
    assert bench["summary"]["timed"] == 3 and bench["images"][0]["warmup"]
