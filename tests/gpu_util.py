"""Helpers shared by the GPU tests: device buffers through torch (plumbing only)
and the layer-level C ABI entry gcdr_k_conv."""
from __future__ import annotations

import ctypes

import numpy as np


from sdcb.gcdrnet_b200 import ConvDesc  # noqa: F401  (gcdr_conv_desc)


class Act(ctypes.Structure):
    """gcdr_act: kind 0 tokens, 1 reflect-padded, 2 phase planes, 3 zero-padded."""
    _fields_ = [("p", ctypes.c_void_p), ("H", ctypes.c_int), ("W", ctypes.c_int), ("C", ctypes.c_int),
                ("kind", ctypes.c_int)]


class Shift(ctypes.Structure):
    """gcdr_shift: cumulative channel-group ends and offsets (at most 5 groups)."""
    _fields_ = [("ngroups", ctypes.c_int), ("ends", ctypes.c_int * 5), ("offs", ctypes.c_int * 5)]

    @classmethod
    def of(cls, ends, offs):
        s = cls()
        s.ngroups = len(ends)
        for g, (e, o) in enumerate(zip(ends, offs)):
            s.ends[g] = e
            s.offs[g] = o
        return s


def to_device_layout(lib, x_hwc_f16, kind):
    """fp16 torch tensor [H][W][C] on the device -> the flat buffer of layout `kind` (1, 2, 3)."""
    import torch
    H, W, C = x_hwc_f16.shape
    n = lib.gcdr_k_to_layout(None, H, W, C, kind, None, None)
    assert n > 0
    buf = torch.empty(n, dtype=torch.float16, device=x_hwc_f16.device)
    assert lib.gcdr_k_to_layout(x_hwc_f16.data_ptr(), H, W, C, kind, buf.data_ptr(), None) == n
    return buf


def from_device_layout(buf, H, W, C, kind):
    """Interior [H][W][C] (fp32 numpy) of a layout buffer (kind 0 tokens, 1/3 padded, 2 phase)."""
    a = buf.float().cpu().numpy()
    if kind == 0:
        return a.reshape(H, W, C)
    if kind in (1, 3):
        return a.reshape(H + 2, W + 2, C)[1:H + 1, 1:W + 1]
    P, Q = (H + 2) // 2, (W + 2) // 2
    planes = a.reshape(2, 2, P, Q, C)
    out = np.empty((H, W, C), np.float32)
    for y in range(H):
        for x in range(W):
            yy, xx = y + 1, x + 1
            out[y, x] = planes[yy & 1, xx & 1, yy >> 1, xx >> 1]
    return out


def pack_weights(w_onnx: np.ndarray) -> np.ndarray:
    """ONNX [N][C][k][k] -> [N][k*k*C] (k index = (ky*k + kx)*C + c)."""
    N, C, k, _ = w_onnx.shape
    return np.ascontiguousarray(w_onnx.transpose(0, 2, 3, 1).reshape(N, k * k * C))


def run_conv(lib, kind, x_hwc, w_onnx, bias, epilogue=0, reference=False, nsplit=1, ksplit=1):
    """Runs one layer through gcdr_k_conv on cuda:0; returns fp32 numpy [Ho][Wo][N]
    (epilogue 3: the split-K partials summed in order plus the bias)."""
    import torch
    H, W, C = x_hwc.shape
    N = w_onnx.shape[0]
    dev = torch.device("cuda:0")
    xt = torch.from_numpy(np.ascontiguousarray(x_hwc)).to(dev, torch.float16)
    if kind == 2:
        inp = xt
    else:
        lay = {0: 1, 1: 2, 3: 3}[kind]
        n = lib.gcdr_k_to_layout(None, H, W, C, lay, None, None)
        assert n > 0
        inp = torch.empty(n, dtype=torch.float16, device=dev)
        assert lib.gcdr_k_to_layout(xt.data_ptr(), H, W, C, lay, inp.data_ptr(), None) == n
    wt = torch.from_numpy(pack_weights(w_onnx)).to(dev, torch.float16)
    bt = torch.from_numpy(np.ascontiguousarray(bias, np.float32)).to(dev)
    if kind == 1:
        Ho, Wo = H // 2, W // 2
    elif epilogue == 1:
        Ho, Wo = H // 2, W // 2
    else:
        Ho, Wo = H, W
    if epilogue == 3:
        out = torch.full((ksplit, Ho * Wo, N), float("nan"), dtype=torch.float32, device=dev)
    else:
        out = torch.full((Ho, Wo, N), float("nan"), dtype=torch.float16, device=dev)
    d = ConvDesc(kind, H, W, C, N, inp.data_ptr(), wt.data_ptr(), bt.data_ptr(), epilogue, out.data_ptr(), None,
                 nsplit, ksplit)
    scratch = None
    if reference:
        n = lib.gcdr_k_conv_scratch(ctypes.byref(d))
        scratch = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
        d.scratch = scratch.data_ptr()
    rc = lib.gcdr_k_conv(ctypes.byref(d), 1 if reference else 0, None)
    assert rc == 0, rc
    torch.cuda.synchronize()
    if epilogue == 3:
        tot = out[0].clone()
        for k in range(1, ksplit):
            tot += out[k]
        return (tot + bt[None, :]).reshape(Ho, Wo, N).cpu().numpy()
    return out.float().cpu().numpy()


def torch_conv(kind, x_hwc, w_onnx, bias, epilogue=0, round_operands=True):
    """fp32 torch reference of one layer.  round_operands: input and weights
    rounded to fp16 first, like the kernel's operands (the check then measures the
    accumulation and output rounding only); False keeps them fp32, so the check
    also covers the operand quantisation."""
    import torch
    import torch.nn.functional as F
    x = torch.from_numpy(np.ascontiguousarray(x_hwc)).permute(2, 0, 1)[None]
    w = torch.from_numpy(w_onnx)
    if round_operands:
        x, w = x.half().float(), w.half().float()
    b = torch.from_numpy(np.ascontiguousarray(bias, np.float32))
    if kind == 0:
        y = F.conv2d(F.pad(x, (1, 1, 1, 1), mode="reflect"), w, b)
    elif kind == 3:
        y = F.conv2d(x, w, b, padding=1)
    elif kind == 1:
        y = F.conv2d(x, w, b, stride=2, padding=1)
    else:
        y = F.conv2d(x, w, b)
    if epilogue == 1:
        y = F.relu(F.max_pool2d(y, 2))
    elif epilogue == 2:
        y = F.relu(y)
    # epilogue 3 (partials + bias) is the plain conv
    return y[0].permute(1, 2, 0).numpy()
