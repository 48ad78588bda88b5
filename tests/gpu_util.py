"""Helpers shared by the GPU tests: device buffers through torch (plumbing only)
and the layer-level C ABI entry gcdr_k_conv."""
from __future__ import annotations

import ctypes

import numpy as np


class ConvDesc(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("H", ctypes.c_int), ("W", ctypes.c_int), ("C", ctypes.c_int),
                ("N", ctypes.c_int), ("inp", ctypes.c_void_p), ("weight", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("epilogue", ctypes.c_int), ("out", ctypes.c_void_p),
                ("scratch", ctypes.c_void_p), ("nsplit", ctypes.c_int), ("ksplit", ctypes.c_int)]


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


def torch_conv(kind, x_hwc, w_onnx, bias, epilogue=0):
    """fp32 torch reference of one layer (input rounded to fp16 like the kernel's)."""
    import torch
    import torch.nn.functional as F
    x = torch.from_numpy(np.ascontiguousarray(x_hwc)).half().float().permute(2, 0, 1)[None]
    w = torch.from_numpy(w_onnx).half().float()
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
