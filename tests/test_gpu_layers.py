"""Layer-level GPU parity of the tcgen05 implicit-GEMM convolution.

Each layer runs three ways on the same seeded inputs: the tcgen05 kernel,
the SIMT reference kernel (same epilogue code, fp32 FMA) and torch fp32 on
the CPU.  Mirrors the reference's GPU-kernel-vs-CPU-kernel tests
(tests/Sdcb.SimdGcdrNet.Tests/VkKernelTests.cs:15-65) for the conv family;
shapes are the GC/DR layer shapes at small spatial sizes.
"""
import numpy as np
import pytest

from gpu_util import run_conv, torch_conv

pytestmark = pytest.mark.gpu

# (kind, H, W, C, N, epilogue): kind 0 reflect s1, 1 stride-2 zero pad, 2 token Gemm, 3 zero-pad s1
CASES = [
    (0, 32, 48, 16, 32, 1),     # GC enc2 (+pool)
    (0, 16, 24, 32, 128, 1),    # GC enc3 (+pool)
    (0, 32, 40, 32, 64, 1),     # DR enc2 (+pool)
    (0, 16, 20, 64, 128, 1),    # DR enc3 (+pool)
    (0, 8, 10, 160, 128, 0),    # GC dec2
    (0, 4, 6, 256, 160, 0),     # GC dec1
    (0, 4, 5, 512, 256, 0),     # DR dec1 (N=256, C=512)
    (0, 64, 80, 16, 16, 0),     # GC dec5 (N=16)
    (0, 16, 20, 128, 32, 0),    # GC dec3
    (0, 3, 7, 32, 32, 0),       # odd tiny
    (1, 16, 20, 128, 160, 0),   # GC pe3 (stride 2)
    (1, 8, 10, 160, 256, 0),    # GC pe4
    (1, 8, 12, 256, 512, 0),    # DR pe4 (N=512)
    (2, 9, 13, 160, 160, 0),    # GC fc
    (2, 6, 7, 512, 512, 0),     # DR block2 fc (N=512)
    (2, 18, 25, 128, 128, 0),   # dblock2 fc
    (3, 24, 30, 32, 64, 2),     # zero-pad conv + relu (microbench form)
    (0, 66, 130, 32, 64, 1),    # pool with two x tiles
    (0, 256, 320, 16, 16, 0),   # dec5-like, 4 tiles per work unit
    (0, 128, 200, 32, 32, 0),   # 2 tiles per work unit
    (0, 96, 150, 64, 64, 2),    # thin layer + relu
    # 256-wide plain slices over several tiles
    (3, 24, 30, 128, 256, 2),   # 6 tiles, zero pad + relu (microbench form)
    (0, 10, 37, 64, 256, 0),    # odd tile count
    # row-window kernel edges: 4 rows per unit with a ragged last unit (rows past the
    # image), odd pooled-row count, segments past the right edge, zero padding
    (0, 150, 1100, 16, 32, 1),
    (0, 150, 1100, 32, 32, 0),
    (3, 150, 600, 16, 16, 2),
    # flat plain layers with between one and two waves of single tiles: two tiles per unit
    (0, 144, 200, 128, 64, 0),    # DR dec3
    (3, 144, 200, 128, 256, 2),   # the 128 -> 256 microbench conv
    # 8-row pool units (stem shapes: at least eight units per SM), one with a ragged last unit
    (0, 1100, 1500, 16, 16, 1),
    (0, 1152, 1600, 16, 32, 1),
]


def _inputs(kind, H, W, C, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((H, W, C)).astype(np.float32)
    k = 1 if kind == 2 else 3
    w = (rng.standard_normal((N, C, k, k)) * np.sqrt(2.0 / (C * k * k))).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    return x, w, b


@pytest.mark.parametrize("case", CASES, ids=lambda c: "k%d_%dx%d_c%d_n%d_e%d" % c)
def test_tc_conv_matches_reference_and_torch(case):
    from sdcb.gcdrnet_b200 import lib
    kind, H, W, C, N, ep = case
    x, w, b = _inputs(kind, H, W, C, N, hash(case) & 0xFFFF)
    L = lib()
    tc = run_conv(L, kind, x, w, b, ep, reference=False)
    ref = run_conv(L, kind, x, w, b, ep, reference=True)
    want = torch_conv(kind, x, w, b, ep)
    assert not np.isnan(tc).any(), "tcgen05 output left unwritten positions"
    scale = np.abs(want).max() + 1e-6
    # fp16 output rounding: 2^-11 relative, plus accumulation-order noise
    d_ref = np.abs(tc - ref).max() / scale
    d_torch = np.abs(tc - want).max() / scale
    rel_l2 = np.linalg.norm(tc - want) / (np.linalg.norm(want) + 1e-12)
    assert d_ref < 2e-3, f"tcgen05 vs SIMT reference max rel {d_ref}"
    assert d_torch < 4e-3, f"tcgen05 vs torch fp32 max rel {d_torch}"
    assert rel_l2 < 1e-3, f"rel L2 {rel_l2}"


# N slices (any epilogue) and split-K fp32 partials (the first stage of the
# LayerNorm layers with few tiles): (kind, H, W, C, N, epilogue, nsplit, ksplit)
SPLIT_CASES = [
    (2, 4, 5, 512, 512, 0, 4, 1),     # DR block2 fc1 at /32, 4 slices of 128
    (0, 2, 3, 256, 160, 0, 5, 1),     # GC dec1 at /32, 5 slices of 32
    (1, 4, 6, 256, 512, 3, 2, 9),     # DR pe4: 2 slices x 9 k splits (one tap each)
    (1, 6, 8, 160, 256, 3, 1, 5),     # GC pe4: 5 k splits of 9 k-blocks
    (2, 5, 7, 512, 512, 3, 2, 4),     # DR block2 fc2
    (2, 9, 10, 256, 256, 3, 1, 2),    # block1 fc2 at /16
    (0, 16, 20, 32, 64, 1, 2, 1),     # pool epilogue with 2 slices
]


@pytest.mark.parametrize("case", SPLIT_CASES, ids=lambda c: "k%d_%dx%d_c%d_n%d_e%d_ns%d_ks%d" % c)
def test_tc_conv_splits(case):
    from sdcb.gcdrnet_b200 import lib
    kind, H, W, C, N, ep, ns, ks = case
    x, w, b = _inputs(kind, H, W, C, N, hash(case) & 0xFFFF)
    L = lib()
    tc = run_conv(L, kind, x, w, b, ep, nsplit=ns, ksplit=ks)
    want = torch_conv(kind, x, w, b, 1 if ep == 1 else 0)
    assert not np.isnan(tc).any(), "unwritten outputs"
    scale = np.abs(want).max() + 1e-6
    d = np.abs(tc - want).max() / scale
    tol = 2e-4 if ep == 3 else 4e-3   # partials are fp32 (no fp16 output rounding)
    assert d < tol, f"split conv vs torch fp32: max rel {d}"


_FLAT_SCRIPT = r"""
import sys, json
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + '/tests')
import numpy as np
from gpu_util import run_conv, torch_conv
from sdcb.gcdrnet_b200 import lib
from test_gpu_layers import CASES, _inputs
L = lib()
out = []
for case in CASES[:8] + CASES[-3:]:
    kind, H, W, C, N, ep = case
    x, w, b = _inputs(kind, H, W, C, N, 7)
    tc = run_conv(L, kind, x, w, b, ep)
    want = torch_conv(kind, x, w, b, ep)
    out.append(float(np.abs(tc - want).max() / (np.abs(want).max() + 1e-6)))
print(json.dumps(out))
"""


def test_flat_kernel_still_matches_torch():
    """The flat implicit-GEMM kernel (the row-window kernel's fallback) on the
    layers the row-window kernel would otherwise take (GCDR_CUDA_CONV=flat)."""
    import json
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, GCDR_CUDA_CONV="flat")
    r = subprocess.run([sys.executable, "-c", _FLAT_SCRIPT, root], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    errs = json.loads(r.stdout.strip().splitlines()[-1])
    assert max(errs) < 4e-3, errs
