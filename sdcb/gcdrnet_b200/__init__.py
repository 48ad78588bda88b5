"""GCDRNet document enhancement on NVIDIA B200 (sm_100a).

Python face of ``libgcdr_cuda.so`` (C ABI: ``include/gcdr_cuda.h``), shaped
like the reference's public API ``Sdcb.SimdGcdrNet.GcdrEnhancer``
(src/Sdcb.SimdGcdrNet/GcdrEnhancer.cs):

    with GcdrEnhancer.from_files(gc_onnx, dr_onnx, GcdrBackend.Cuda) as enh:
        enh.enhance(src, width, height, src_stride, dst, dst_stride, GcdrPixelFormat.Bgra32)
        out = enh.enhance_image(bgr, width, height)        # Enhance(byte[], w, h, fmt)

Errors raise the analogues of the reference's exceptions
(ArgumentOutOfRangeError, ArgumentError, NotSupportedError, DeviceLostError).
Only the CUDA backend lives here; there is no CPU fallback -- the library
must be built (``python -m sdcb.gcdrnet_b200._build``) and a B200 present.
"""
from __future__ import annotations

import ctypes
import enum
import io
import os
import threading

__all__ = ["GcdrBackend", "GcdrPixelFormat", "GcdrEnhancer", "CudaWorker", "ConvDesc", "lib", "library_path",
           "register_host", "unregister_host", "GcdrError", "ArgumentError", "ArgumentOutOfRangeError", "NotSupportedError",
           "DeviceLostError", "DeviceTimeoutError", "ModelError", "OutOfMemoryError",
           "bytes_per_pixel"]

_PKG = os.path.dirname(os.path.abspath(__file__))
library_path = os.path.join(_PKG, "libgcdr_cuda.so")


class GcdrBackend(enum.IntEnum):
    """GcdrBackend (GcdrEnhancer.cs:16-27) plus the Cuda arm this package adds."""
    Cpu = 0
    Vulkan = 1
    Auto = 2
    Metal = 3
    Cuda = 4


class GcdrPixelFormat(enum.IntEnum):
    """GcdrPixelFormat (GcdrPixelFormat.cs:7-17)."""
    Bgr24 = 0
    Rgb24 = 1
    Bgra32 = 2
    Rgba32 = 3


def bytes_per_pixel(fmt) -> int:
    f = int(fmt)
    if f in (0, 1):
        return 3
    if f in (2, 3):
        return 4
    raise ArgumentOutOfRangeError(f"unknown pixel format {fmt}")


class GcdrError(Exception):
    code = -1


class ArgumentError(GcdrError, ValueError):
    code = 1


class ArgumentOutOfRangeError(ArgumentError):
    code = 2


class NotSupportedError(GcdrError):
    code = 3


class DeviceLostError(GcdrError, RuntimeError):
    code = 4


class DeviceTimeoutError(GcdrError, RuntimeError):
    code = 5


class OutOfMemoryError(GcdrError, MemoryError):
    code = 6


class ModelError(GcdrError, ValueError):
    code = 7


_ERRORS = {c.code: c for c in (ArgumentError, ArgumentOutOfRangeError, NotSupportedError, DeviceLostError,
                               DeviceTimeoutError, OutOfMemoryError, ModelError)}


def _raise(rc: int, msg: str = ""):
    if rc:
        raise _ERRORS.get(rc, GcdrError)(msg or f"gcdr status {rc}")


class ConvDesc(ctypes.Structure):
    """gcdr_conv_desc of include/gcdr_cuda.h (the layer entries gcdr_k_conv / gcdr_k_conv_static)."""
    _fields_ = [("kind", ctypes.c_int), ("H", ctypes.c_int), ("W", ctypes.c_int), ("C", ctypes.c_int),
                ("N", ctypes.c_int), ("inp", ctypes.c_void_p), ("weight", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("epilogue", ctypes.c_int), ("out", ctypes.c_void_p),
                ("scratch", ctypes.c_void_p), ("nsplit", ctypes.c_int), ("ksplit", ctypes.c_int),
                ("bias_host", ctypes.c_void_p), ("wait_cycles", ctypes.c_longlong), ("timeout_probe", ctypes.c_int)]


_lib = None
_lib_lock = threading.Lock()


def lib():
    """The loaded libgcdr_cuda.so (raises when it has not been built)."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(library_path):
            raise ImportError(f"{library_path} is missing: build it with `python -m sdcb.gcdrnet_b200._build`")
        L = ctypes.CDLL(library_path)
        vp, sz, i, i64, cp = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int64, ctypes.c_char_p
        L.gcdr_model_load.argtypes = [vp, sz, vp, sz, ctypes.POINTER(vp), cp, sz]
        L.gcdr_model_free.argtypes = [vp]
        L.gcdr_model_describe.argtypes = [vp, cp, sz]
        L.gcdr_model_describe.restype = sz
        L.gcdr_cuda_create.argtypes = [i, vp, i, ctypes.POINTER(vp)]
        L.gcdr_cuda_create_from_onnx.argtypes = [i, vp, sz, vp, sz, i, ctypes.POINTER(vp)]
        L.gcdr_cuda_enhance.argtypes = [vp, vp, i, i, i, vp, i, i]
        L.gcdr_cuda_enhance_device.argtypes = [vp, vp, i, i, vp, i, vp]
        L.gcdr_cuda_enhance_batch.argtypes = [vp, vp, i, i, i, i, vp, i, i]
        L.gcdr_cuda_enhance_batch_device.argtypes = [vp, vp, i, i, i, vp, i, vp]
        L.gcdr_cuda_device_bytes.argtypes = [vp]
        L.gcdr_cuda_device_bytes.restype = i64
        L.gcdr_cuda_debug_intermediates.argtypes = [vp, vp, vp, vp]
        L.gcdr_cuda_debug_output.argtypes = [vp, vp]
        L.gcdr_cuda_set_debug.argtypes = [vp, i]
        L.gcdr_cuda_launch_count.argtypes = [vp]
        L.gcdr_cuda_plan_stats.argtypes = [vp, ctypes.POINTER(i), ctypes.POINTER(i)]
        L.gcdr_cuda_profile.argtypes = [vp, i, vp, i]
        L.gcdr_cuda_last_error.argtypes = [vp]
        L.gcdr_cuda_last_error.restype = cp
        L.gcdr_cuda_destroy.argtypes = [vp]
        L.gcdr_enhancer_create.argtypes = [i, vp, sz, vp, sz, i, ctypes.POINTER(vp), cp, sz]
        L.gcdr_enhancer_enhance.argtypes = [vp, vp, sz, i, i, i, vp, sz, i, i, cp, sz]
        L.gcdr_enhancer_enhance_batch.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(sz), i, i, i, i,
                                                  ctypes.POINTER(vp), ctypes.POINTER(sz), i, i, cp, sz]
        L.gcdr_enhancer_set_batching.argtypes = [vp, i, i]
        L.gcdr_enhancer_batch_stats.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.gcdr_enhancer_batch_stats.restype = None
        L.gcdr_enhancer_pool_stats.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.gcdr_enhancer_inject_device_loss.argtypes = [vp, i]
        L.gcdr_enhancer_destroy.argtypes = [vp]
        L.gcdr_k_bgr2nhwc.argtypes = [vp, i, i, i, i, vp, i, i, vp]
        L.gcdr_k_div6.argtypes = [vp, vp, sz, vp, vp]
        L.gcdr_k_nhwc2bgr.argtypes = [vp, i, i, i, i, vp, i, i, i, i, vp, i, vp]
        L.gcdr_k_conv.argtypes = [vp, i, vp]
        L.gcdr_k_conv_scratch.argtypes = [vp]
        L.gcdr_k_conv_scratch.restype = i64
        L.gcdr_k_to_layout.argtypes = [vp, i, i, i, i, vp, vp]
        L.gcdr_k_to_layout.restype = i64
        L.gcdr_device_sms.restype = i
        L.gcdr_k_conv_static.argtypes = [vp, vp]
        L.gcdr_k_status.argtypes = [vp]
        L.gcdr_host_register.argtypes = [vp, sz]
        L.gcdr_host_unregister.argtypes = [vp]
        f = ctypes.c_float
        L.gcdr_k_dw_gelu_shift.argtypes = [vp, i, i, i, vp, vp, vp, vp, vp]
        L.gcdr_k_up_add.argtypes = [vp, vp, vp, vp, vp, f, vp, vp, vp]
        L.gcdr_k_ln_finalize.argtypes = [vp, i, i, i, i, vp, vp, vp, vp, f, vp, vp, f, vp, vp, vp, vp]
        _lib = L
        return L


def register_host(buf) -> None:
    """Page-locks a C-contiguous numpy array (or other buffer) for direct DMA: enhance calls
    whose source or destination lies in it skip the staging copies.  Call unregister_host
    before the memory goes away."""
    b = _Buf(buf, writable=False)
    _raise(lib().gcdr_host_register(b.ptr, b.len), "host register failed")


def unregister_host(buf) -> None:
    b = _Buf(buf, writable=False)
    _raise(lib().gcdr_host_unregister(b.ptr), "host unregister failed")


class _Buf:
    """A writable/readable view of a bytes-like object as (pointer, length)."""

    def __init__(self, obj, writable: bool):
        self._keep = None
        if obj is None:
            raise ArgumentError("buffer is None")
        if hasattr(obj, "__array_interface__"):
            ai = obj.__array_interface__
            if ai.get("strides") not in (None,) and not getattr(obj, "flags", None).c_contiguous:
                raise ArgumentError("buffer must be C-contiguous")
            self.ptr = ai["data"][0]
            self.len = obj.nbytes
            if writable and ai["data"][1]:
                raise ArgumentError("destination buffer is read-only")
            self._keep = obj
        elif isinstance(obj, bytes):
            if writable:
                raise ArgumentError("destination must be writable (bytearray / numpy array)")
            self._keep = obj
            self.ptr = ctypes.cast(ctypes.c_char_p(obj), ctypes.c_void_p).value
            self.len = len(obj)
        else:
            mv = memoryview(obj)
            if writable and mv.readonly:
                raise ArgumentError("destination buffer is read-only")
            c = (ctypes.c_char * mv.nbytes).from_buffer(obj) if not mv.readonly else None
            if c is None:
                b = bytes(mv)
                self._keep = b
                self.ptr = ctypes.cast(ctypes.c_char_p(b), ctypes.c_void_p).value
            else:
                self._keep = c
                self.ptr = ctypes.addressof(c)
            self.len = mv.nbytes


def _read_all(x) -> bytes:
    if isinstance(x, (bytes, bytearray, memoryview)):
        return bytes(x)
    if isinstance(x, (str, os.PathLike)):
        with open(x, "rb") as fh:
            return fh.read()
    if isinstance(x, io.IOBase) or hasattr(x, "read"):
        return x.read()
    raise ArgumentError(f"cannot read model from {type(x).__name__}")


class GcdrEnhancer:
    """Thread-safe GCDRNet enhancer on one CUDA device (GcdrEnhancer.cs:36-433)."""

    def __init__(self, gc_onnx: bytes, dr_onnx: bytes, backend=GcdrBackend.Cuda, device: int = 0):
        if int(backend) not in (GcdrBackend.Cuda, GcdrBackend.Auto):
            raise NotSupportedError(f"backend {GcdrBackend(int(backend)).name} is not part of the B200 package")
        L = lib()
        h = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        rc = L.gcdr_enhancer_create(int(device), gc_onnx, len(gc_onnx), dr_onnx, len(dr_onnx), 0,
                                    ctypes.byref(h), err, 512)
        _raise(rc, err.value.decode(errors="replace"))
        self._h = h
        self.device = int(device)

    # GcdrEnhancer.FromFiles / FromBytes / FromStreams (GcdrEnhancer.cs:82-100)
    @classmethod
    def from_files(cls, gcnet_onnx_path, drnet_onnx_path, backend=GcdrBackend.Cuda, device: int = 0):
        return cls(_read_all(gcnet_onnx_path), _read_all(drnet_onnx_path), backend, device)

    @classmethod
    def from_bytes(cls, gcnet_onnx, drnet_onnx, backend=GcdrBackend.Cuda, device: int = 0):
        return cls(bytes(gcnet_onnx), bytes(drnet_onnx), backend, device)

    @classmethod
    def from_streams(cls, gcnet_onnx, drnet_onnx, backend=GcdrBackend.Cuda, device: int = 0):
        if gcnet_onnx is None or drnet_onnx is None:
            raise ArgumentError("stream is None")
        return cls(gcnet_onnx.read(), drnet_onnx.read(), backend, device)

    def enhance(self, src, width: int, height: int, src_stride: int, dst, dst_stride: int,
                format=GcdrPixelFormat.Bgr24) -> None:
        """Enhance(src, width, height, srcStride, dst, dstStride, format) (GcdrEnhancer.cs:181-271).

        src/dst are bytes-like host buffers (numpy uint8 arrays, bytearray); dst
        may be the same memory as src when the strides are equal.
        """
        if self._h is None:
            raise GcdrError("enhancer disposed")
        fmt = int(format)
        s = _Buf(src, False)
        d = _Buf(dst, True)
        err = ctypes.create_string_buffer(512)
        rc = lib().gcdr_enhancer_enhance(self._h, s.ptr, s.len, int(width), int(height), int(src_stride),
                                         d.ptr, d.len, int(dst_stride), fmt, err, 512)
        _raise(rc, err.value.decode(errors="replace"))

    def enhance_batch(self, srcs, width: int, height: int, src_stride: int, dsts, dst_stride: int,
                      format=GcdrPixelFormat.Bgr24) -> None:
        """n (1..16) same-shape images through one pooled worker's batch plan (one launch per
        layer for all of them, gcdr_enhancer_enhance_batch); each image gets the bytes that
        enhance() gives it.  dsts[k] may be the same memory as srcs[k] at equal strides."""
        if self._h is None:
            raise GcdrError("enhancer disposed")
        n = len(srcs)
        if n != len(dsts):
            raise ArgumentError("srcs and dsts differ in length")
        if n == 0:
            return
        ss = [_Buf(s, False) for s in srcs]
        ds = [_Buf(d, True) for d in dsts]
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        sp, sl = (vp * n)(*[b.ptr for b in ss]), (sz * n)(*[b.len for b in ss])
        dp, dl = (vp * n)(*[b.ptr for b in ds]), (sz * n)(*[b.len for b in ds])
        err = ctypes.create_string_buffer(512)
        rc = lib().gcdr_enhancer_enhance_batch(self._h, sp, sl, n, int(width), int(height), int(src_stride),
                                               dp, dl, int(dst_stride), int(format), err, 512)
        _raise(rc, err.value.decode(errors="replace"))

    def enhance_image(self, src, width: int, height: int, format=GcdrPixelFormat.Bgr24):
        """Enhance(byte[] src, w, h, format) (GcdrEnhancer.cs:316-322): tight in, new buffer out."""
        import numpy as np
        stride = int(width) * bytes_per_pixel(format)
        dst = np.empty(stride * int(height), np.uint8)
        self.enhance(src, width, height, stride, dst, stride, format)
        return dst

    def set_batching(self, max_batch: int = 8, max_running: int = 3) -> None:
        """Concurrent enhance() calls of one shape run together: when no batch of that shape is
        on the GPU, or a full batch is queued and fewer than max_running run, a waiting caller
        runs the oldest queued calls (a power of two, at most max_batch) as one batched launch;
        a lone call runs at once.  Results are the single-image bytes.  max_batch = 1 turns it
        off."""
        _raise(lib().gcdr_enhancer_set_batching(self._h, int(max_batch), int(max_running)), "bad batching limits")

    @property
    def batch_stats(self):
        """(enhance calls, worker launches that ran them)."""
        a, b = ctypes.c_int64(), ctypes.c_int64()
        lib().gcdr_enhancer_batch_stats(self._h, ctypes.byref(a), ctypes.byref(b))
        return a.value, b.value

    @property
    def pool_stats(self):
        """(pools, workers, evicted) (GcdrEnhancer.cs:67-68)."""
        a, b, c = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        lib().gcdr_enhancer_pool_stats(self._h, ctypes.byref(a), ctypes.byref(b), ctypes.byref(c))
        return a.value, b.value, c.value

    def inject_device_loss(self, count: int = 1) -> None:
        """Test hook: the next `count` worker runs report device loss (host-side fault injection)."""
        lib().gcdr_enhancer_inject_device_loss(self._h, int(count))

    def dispose(self) -> None:
        if self._h is not None:
            lib().gcdr_enhancer_destroy(self._h)
            self._h = None

    close = dispose

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.dispose()

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


class OpProfile(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 48), ("ms", ctypes.c_double), ("flops", ctypes.c_double),
                ("bytes", ctypes.c_double), ("tensor_core", ctypes.c_int)]


class CudaWorker:
    """One worker (gcdr_cuda_*): the VkGcdrPipeline-level object, not thread-safe."""

    def __init__(self, gc_onnx: bytes, dr_onnx: bytes, device: int = 0):
        L = lib()
        h = ctypes.c_void_p()
        _raise(L.gcdr_cuda_create_from_onnx(int(device), gc_onnx, len(gc_onnx), dr_onnx, len(dr_onnx), 0,
                                            ctypes.byref(h)), "worker creation failed")
        self._h = h

    @classmethod
    def from_files(cls, gc_path, dr_path, device: int = 0):
        return cls(_read_all(gc_path), _read_all(dr_path), device)

    def _check(self, rc):
        if rc:
            _raise(rc, lib().gcdr_cuda_last_error(self._h).decode(errors="replace"))

    def enhance(self, src, width, height, src_stride, dst, dst_stride, format=GcdrPixelFormat.Bgr24):
        s, d = _Buf(src, False), _Buf(dst, True)
        self._check(lib().gcdr_cuda_enhance(self._h, s.ptr, int(width), int(height), int(src_stride), d.ptr,
                                            int(dst_stride), int(format)))

    def enhance_device(self, d_src: int, width, height, d_dst: int, format=GcdrPixelFormat.Bgr24, stream: int = 0):
        self._check(lib().gcdr_cuda_enhance_device(self._h, d_src, int(width), int(height), d_dst, int(format),
                                                   stream or None))

    def enhance_batch(self, srcs, width, height, src_stride, dsts, dst_stride, format=GcdrPixelFormat.Bgr24):
        """n same-shape images (host buffers) in one CUDA-graph launch (gcdr_cuda_enhance_batch)."""
        if len(srcs) != len(dsts):
            raise ArgumentError("srcs and dsts differ in length")
        s = [_Buf(b, False) for b in srcs]
        d = [_Buf(b, True) for b in dsts]
        n = len(s)
        sp = (ctypes.c_void_p * n)(*[b.ptr for b in s])
        dp_ = (ctypes.c_void_p * n)(*[b.ptr for b in d])
        self._check(lib().gcdr_cuda_enhance_batch(self._h, sp, n, int(width), int(height), int(src_stride), dp_,
                                                  int(dst_stride), int(format)))

    def enhance_batch_device(self, d_srcs, width, height, d_dsts, format=GcdrPixelFormat.Bgr24, stream: int = 0):
        """n same-shape device-resident tight images in one CUDA-graph launch, asynchronous on `stream`."""
        n = len(d_srcs)
        if n != len(d_dsts):
            raise ArgumentError("d_srcs and d_dsts differ in length")
        sp = (ctypes.c_void_p * n)(*d_srcs)
        dp_ = (ctypes.c_void_p * n)(*d_dsts)
        self._check(lib().gcdr_cuda_enhance_batch_device(self._h, sp, n, int(width), int(height), dp_, int(format),
                                                         stream or None))

    def set_debug(self, on: bool = True):
        self._check(lib().gcdr_cuda_set_debug(self._h, 1 if on else 0))

    def debug_intermediates(self, H: int, W: int):
        """(gc_in, gc_out, dr_in) padded NHWC fp32 of the last enhance (gc_out needs debug mode)."""
        import numpy as np
        x = np.empty((H, W, 3), np.float32)
        s = np.empty((H, W, 3), np.float32)
        d = np.empty((H, W, 6), np.float32)
        self._check(lib().gcdr_cuda_debug_intermediates(self._h, x.ctypes.data, s.ctypes.data, d.ctypes.data))
        return x, s, d

    def debug_output(self, H: int, W: int):
        import numpy as np
        y = np.empty((H, W, 3), np.float32)
        self._check(lib().gcdr_cuda_debug_output(self._h, y.ctypes.data))
        return y

    def profile(self, reps: int = 5):
        """Per-op [(name, ms, flops, bytes, tensor_core)] of the bound shape."""
        arr = (OpProfile * 256)()
        n = lib().gcdr_cuda_profile(self._h, int(reps), arr, 256)
        if n < 0:
            self._check(-n)
        return [(arr[k].name.decode(), arr[k].ms, arr[k].flops, arr[k].bytes, arr[k].tensor_core) for k in range(n)]

    @property
    def device_bytes(self) -> int:
        return lib().gcdr_cuda_device_bytes(self._h)

    @property
    def launch_count(self) -> int:
        return lib().gcdr_cuda_launch_count(self._h)

    @property
    def plan_stats(self) -> tuple:
        """(graph captures so far, shape plans held): one capture per shape not cached."""
        c, p = ctypes.c_int(), ctypes.c_int()
        self._check(lib().gcdr_cuda_plan_stats(self._h, ctypes.byref(c), ctypes.byref(p)))
        return c.value, p.value

    def close(self):
        if self._h is not None:
            lib().gcdr_cuda_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def describe_models(gc_onnx: bytes, dr_onnx: bytes) -> dict:
    """Parses both models (no GPU) and returns the recognised topology."""
    import json
    L = lib()
    m = ctypes.c_void_p()
    err = ctypes.create_string_buffer(512)
    _raise(L.gcdr_model_load(gc_onnx, len(gc_onnx), dr_onnx, len(dr_onnx), ctypes.byref(m), err, 512),
           err.value.decode(errors="replace"))
    try:
        n = L.gcdr_model_describe(m, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        L.gcdr_model_describe(m, buf, n + 1)
        return json.loads(buf.value.decode())
    finally:
        L.gcdr_model_free(m)
