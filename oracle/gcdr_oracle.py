"""CPU oracle of the GCDRNet enhancement path (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of bench.py use this module, and only as the
checker or as the timed CPU baseline.  The product (``sdcb.gcdrnet_b200`` and
``libgcdr_cuda.so``) never imports it.

The network is restated from the ONNX graphs
``tests/testdata/models/gcdrnet_{gcnet,drnet}_sim.onnx`` of the reference
(node numbers ``gc#N`` / ``dr#N`` are graph indices); the per-operator
arithmetic lives in ``gcdr_oracle.c`` (OpenMP C).  The five-stage pipeline
follows ``src/Sdcb.SimdGcdrNet/GcdrEnhancer.cs:226-270``:
pre -> GC-Net -> div6 -> DR-Net -> post.

Pinned by ``tests/test_oracle_golden.py`` against the reference's committed
onnxruntime outputs ``tests/testdata/{small,pad,mid}_{shadow,output}.f32``
(max abs < 1e-4 per net, ``tests/Sdcb.SimdGcdrNet.Tests/GoldenTests.cs:13-50``).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import numpy as np

from .onnx_model import OnnxGraph, split_sizes

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_build", "libgcdr_oracle.so")            # AVX2 + FMA
LIB512_PATH = os.path.join(_HERE, "_build", "libgcdr_oracle_avx512.so")  # x86-64-v4 (AVX-512)
_V4_FLAGS = ("avx512f", "avx512bw", "avx512vl", "avx512dq", "avx512cd")

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_lib = None


def build(force: bool = False) -> str:
    """Compile gcdr_oracle.c (gcc, OpenMP) twice: oracle/_build/libgcdr_oracle.so for AVX2 +
    FMA hosts and libgcdr_oracle_avx512.so for AVX-512 (x86-64-v4) hosts.  The libraries
    are built once and may run on another x86 host; lib() loads the widest one the host
    runs.  Both give bit-identical results on the golden and benchmark images."""
    src = os.path.join(_HERE, "gcdr_oracle.c")
    import subprocess
    os.makedirs(os.path.dirname(LIB_PATH), exist_ok=True)
    for path, isa in ((LIB_PATH, ["-mavx2", "-mfma"]), (LIB512_PATH, ["-march=x86-64-v4", "-mprefer-vector-width=512"])):
        if not force and os.path.exists(path) and os.path.getmtime(path) >= os.path.getmtime(src):
            continue
        tmp = path + ".tmp%d" % os.getpid()
        subprocess.check_call(["gcc", "-O3"] + isa + ["-fopenmp", "-fPIC", "-shared", "-fvisibility=hidden",
                                                      "-o", tmp, src, "-lm"])
        os.replace(tmp, path)
    return LIB_PATH


def _host_flags() -> set:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def isa() -> str:
    """The instruction set of the oracle library lib() loads on this host."""
    return "avx512 (x86-64-v4)" if all(f in _host_flags() for f in _V4_FLAGS) else "avx2+fma"


def lib():
    global _lib
    if _lib is not None:
        return _lib
    path = LIB512_PATH if isa().startswith("avx512") else LIB_PATH
    if not os.path.exists(path):
        build()
    L = ctypes.CDLL(path)
    i, sz, f = ctypes.c_int, ctypes.c_size_t, ctypes.c_float
    L.orc_conv2d.argtypes = [_f32p, i, i, i, _f32p, ctypes.c_void_p, i, i, i, i, i, _f32p]
    L.orc_maxpool2_relu.argtypes = [_f32p, i, i, i, _f32p]
    L.orc_relu.argtypes = [_f32p, sz]
    L.orc_add.argtypes = [_f32p, _f32p, _f32p, sz]
    L.orc_sigmoid.argtypes = [_f32p, sz]
    L.orc_layernorm.argtypes = [_f32p, sz, i, _f32p, _f32p, f, _f32p]
    L.orc_gemm_bias.argtypes = [_f32p, sz, i, _f32p, _f32p, i, _f32p]
    L.orc_dwconv3x3.argtypes = [_f32p, i, i, i, _f32p, _f32p, _f32p]
    L.orc_gelu.argtypes = [_f32p, sz]
    L.orc_shift.argtypes = [_f32p, i, i, i, i, _i32p, _i32p, i, _f32p]
    L.orc_resize2x.argtypes = [_f32p, i, i, i, _f32p]
    L.orc_pre.argtypes = [ctypes.c_void_p, i, i, i, i, i, i, _f32p]
    L.orc_div6.argtypes = [_f32p, _f32p, sz, _f32p]
    L.orc_post.argtypes = [_f32p, i, i, i, i, ctypes.c_void_p, i, i, i, i, ctypes.c_void_p, i]
    L.orc_num_threads.restype = i
    L.orc_set_threads.argtypes = [i]
    _lib = L
    return L


def num_threads() -> int:
    return lib().orc_num_threads()


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


# ----------------------------------------------------------------- operators

def conv2d(x, w, b, stride=1, pad=1, reflect=True):
    H, W, Cin = x.shape
    Cout, wc, k, _ = w.shape
    assert wc == Cin, (wc, Cin)
    Ho = (H + 2 * pad - k) // stride + 1
    Wo = (W + 2 * pad - k) // stride + 1
    out = np.empty((Ho, Wo, Cout), np.float32)
    bias = np.ascontiguousarray(b, np.float32) if b is not None else None
    lib().orc_conv2d(np.ascontiguousarray(x), H, W, Cin, np.ascontiguousarray(w, np.float32),
                     bias.ctypes.data if bias is not None else None, Cout, k, stride, pad,
                     1 if reflect else 0, out)
    return out


def maxpool2_relu(x):
    H, W, C = x.shape
    out = np.empty((H // 2, W // 2, C), np.float32)
    lib().orc_maxpool2_relu(np.ascontiguousarray(x), H, W, C, out)
    return out


def relu(x):
    y = np.array(x, np.float32, copy=True, order="C")
    lib().orc_relu(y, y.size)
    return y


def add(a, b):
    out = np.empty_like(a)
    lib().orc_add(np.ascontiguousarray(a), np.ascontiguousarray(b), out, a.size)
    return out


def sigmoid(x):
    y = np.array(x, np.float32, copy=True, order="C")
    lib().orc_sigmoid(y, y.size)
    return y


def layernorm(x, g, b, eps=1e-5):
    C = x.shape[-1]
    out = np.empty_like(x)
    lib().orc_layernorm(np.ascontiguousarray(x), x.size // C, C, np.ascontiguousarray(g),
                        np.ascontiguousarray(b), eps, out)
    return out


def gemm(x, B, bias):
    C = x.shape[-1]
    N = B.shape[1]
    out = np.empty(x.shape[:-1] + (N,), np.float32)
    lib().orc_gemm_bias(np.ascontiguousarray(x), x.size // C, C, np.ascontiguousarray(B),
                        np.ascontiguousarray(bias), N, out)
    return out


def dwconv3x3(x, w, b):
    H, W, C = x.shape
    out = np.empty_like(x)
    lib().orc_dwconv3x3(np.ascontiguousarray(x), H, W, C, np.ascontiguousarray(w), np.ascontiguousarray(b), out)
    return out


def gelu(x):
    y = np.array(x, np.float32, copy=True, order="C")
    lib().orc_gelu(y, y.size)
    return y


def shift(x, axis, ends, offs):
    H, W, C = x.shape
    out = np.empty_like(x)
    lib().orc_shift(np.ascontiguousarray(x), H, W, C, axis, np.asarray(ends, np.int32),
                    np.asarray(offs, np.int32), len(offs), out)
    return out


def resize2x(x):
    H, W, C = x.shape
    out = np.empty((2 * H, 2 * W, C), np.float32)
    lib().orc_resize2x(np.ascontiguousarray(x), H, W, C, out)
    return out


# --------------------------------------------------------------------- glue

BPP = {0: 3, 1: 3, 2: 4, 3: 4}


def pad_amounts(h: int, w: int):
    """Top/left replicate padding to a multiple of 32 (GcdrEnhancer.cs:226-227)."""
    return (-h) & 31, (-w) & 31


def pre(src, w, h, stride, fmt):
    ph, pw = pad_amounts(h, w)
    x = np.empty((h + ph, w + pw, 3), np.float32)
    buf = np.ascontiguousarray(src, np.uint8)
    lib().orc_pre(buf.ctypes.data, w, h, stride, fmt, ph, pw, x)
    return x


def div6(x, s):
    H, W, _ = x.shape
    out = np.empty((H, W, 6), np.float32)
    lib().orc_div6(np.ascontiguousarray(x), np.ascontiguousarray(s), H * W, out)
    return out


def post(y, w, h, dst, dst_stride, fmt, alpha_src=None, alpha_stride=0):
    H, W, _ = y.shape
    ph, pw = H - h, W - w
    if BPP[fmt] == 4 and alpha_src is None:
        raise ValueError("4-byte formats need the alpha source")
    a = alpha_src if alpha_src is not None else dst
    lib().orc_post(np.ascontiguousarray(y), H, W, ph, pw, dst.ctypes.data, w, h, dst_stride, fmt,
                   a.ctypes.data, alpha_stride)
    return dst


# ------------------------------------------------------------------ network

@dataclass
class Block:
    """One shifted-MLP block (UNeXt shiftedBlock) plus the LayerNorm after it."""
    norm2: tuple
    fc1: tuple
    dw: tuple
    fc2: tuple
    shift_h: tuple   # (axis, ends, offsets) of the first shift (gc#44-80)
    shift_w: tuple   # of the second shift (gc#95-126)
    norm_out: tuple  # norm3 / norm4 / dnorm3 / dnorm4


class GcdrNet:
    """Weights of one of the two UNeXt-style nets, read from its ONNX graph."""

    def __init__(self, g: OnnxGraph):
        I = g.init
        cw = lambda n: (I(f"m.{n}.weight"), I(f"m.{n}.bias"))
        self.enc = [cw("encoder1.1"), cw("encoder2.1"), cw("encoder3.1")]
        self.pe3, self.pe4 = cw("patch_embed3.proj"), cw("patch_embed4.proj")
        self.pe3_norm, self.pe4_norm = cw("patch_embed3.norm"), cw("patch_embed4.norm")
        self.dec = [cw(f"decoder{i}.1") for i in range(1, 6)]
        self.final = cw("final")
        shifts = g.shifts()
        if len(shifts) != 8:
            raise ValueError(f"expected 8 shift groups, found {len(shifts)}")

        def block(name, norm_out, si):
            C = I(f"m.{name}.0.norm2.weight").shape[0]

            def sh(k):
                axis, sizes, offs, nout = shifts[k]
                return axis, np.cumsum(split_sizes(C, sizes, nout)).tolist(), offs
            return Block(
                norm2=cw(f"{name}.0.norm2"),
                fc1=(g.gemm_weight(f"m.{name}.0.mlp.fc1.bias"), I(f"m.{name}.0.mlp.fc1.bias")),
                dw=cw(f"{name}.0.mlp.dwconv.dwconv"),
                fc2=(g.gemm_weight(f"m.{name}.0.mlp.fc2.bias"), I(f"m.{name}.0.mlp.fc2.bias")),
                shift_h=sh(si), shift_w=sh(si + 1), norm_out=cw(norm_out))
        # Splits appear in graph order block1, block2, dblock1, dblock2 (two each)
        self.block1 = block("block1", "norm3", 0)
        self.block2 = block("block2", "norm4", 2)
        self.dblock1 = block("dblock1", "dnorm3", 4)
        self.dblock2 = block("dblock2", "dnorm4", 6)
        self.cin = self.enc[0][0].shape[1]

    @classmethod
    def load(cls, path):
        return cls(OnnxGraph.load(path))


def shifted_block(x, blk: Block):
    """x + MLP(LN2(x)) then the block's trailing LayerNorm (gc#38-130).

    MLP = shift(H) -> fc1 -> dwconv3x3 -> GELU -> shift(W) -> fc2.
    """
    h = layernorm(x, *blk.norm2)
    h = shift(h, *blk.shift_h)
    h = gemm(h, *blk.fc1)
    h = dwconv3x3(h, *blk.dw)
    h = gelu(h)
    h = shift(h, *blk.shift_w)
    h = gemm(h, *blk.fc2)
    return layernorm(add(x, h), *blk.norm_out)


def net_forward(net: GcdrNet, x: np.ndarray, trace: dict | None = None) -> np.ndarray:
    """One net on an NHWC input [H][W][Cin] (H, W multiples of 32) -> [H][W][3]."""
    H, W, C = x.shape
    if C != net.cin or H % 32 or W % 32:
        raise ValueError(f"input {x.shape} does not fit the net (cin {net.cin}, /32)")
    c1 = conv2d(x, *net.enc[0])                       # gc#22-23 (skip for the tail)
    t1 = maxpool2_relu(c1)                            # gc#24-25
    t2 = maxpool2_relu(conv2d(t1, *net.enc[1]))       # gc#26-29
    t3 = maxpool2_relu(conv2d(t2, *net.enc[2]))       # gc#30-33
    y = conv2d(t3, *net.pe3, stride=2, pad=1, reflect=False)   # gc#34
    y = layernorm(y, *net.pe3_norm)                   # gc#37
    t4 = shifted_block(y, net.block1)                 # gc#38-130
    y = conv2d(t4, *net.pe4, stride=2, pad=1, reflect=False)   # gc#134
    y = layernorm(y, *net.pe4_norm)                   # gc#137
    y = shifted_block(y, net.block2)                  # gc#138-230
    d = add(relu(resize2x(conv2d(y, *net.dec[0]))), t4)        # gc#234-240
    d = shifted_block(d, net.dblock1)                 # gc#243-335
    d = add(relu(resize2x(conv2d(d, *net.dec[1]))), t3)        # gc#339-343
    d = shifted_block(d, net.dblock2)                 # gc#346-438
    d = add(relu(resize2x(conv2d(d, *net.dec[2]))), t2)        # gc#442-446
    d = add(relu(resize2x(conv2d(d, *net.dec[3]))), t1)        # gc#447-451
    d = conv2d(d, *net.dec[4])                        # gc#452-453
    s = add(relu(resize2x(d)), relu(c1))              # gc#454-457
    out = sigmoid(conv2d(s, *net.final, stride=1, pad=0, reflect=False))  # gc#458-459
    if trace is not None:
        trace.update(c1=c1, t1=t1, t2=t2, t3=t3, t4=t4, dec5=d, head_in=s)
    return out


class Oracle:
    """Both nets and the five-stage enhancement (GcdrEnhancer.cs:226-270)."""

    def __init__(self, gc_path, dr_path):
        self.gc = GcdrNet.load(gc_path)
        self.dr = GcdrNet.load(dr_path)

    def stages(self, src, w, h, stride, fmt):
        x = pre(src, w, h, stride, fmt)
        shadow = net_forward(self.gc, x)
        x6 = div6(x, shadow)
        out = net_forward(self.dr, x6)
        return x, shadow, x6, out

    def enhance(self, src, w, h, stride, dst, dst_stride, fmt=0):
        _, _, _, out = self.stages(src, w, h, stride, fmt)
        return post(out, w, h, dst, dst_stride, fmt, src if BPP[fmt] == 4 else None, stride)
