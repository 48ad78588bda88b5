"""Minimal ONNX reader for the oracle (test infrastructure only).

Decodes the protobuf wire format of an ONNX ModelProto with no dependency
beyond numpy, and extracts from the GCDRNet graphs everything the network
restatement in :mod:`oracle.gcdr_oracle` needs: initialiser tensors by name,
the Gemm weight feeding each ``m.*.mlp.fc*.bias``, the channel-group sizes of
each shift Split and the per-group shift offsets/axes encoded by its
``Mod``/``Slice`` roll pattern.

The shift recovery follows the reference's pattern pass
``Extensions/ChannelShiftOp.cs:64-188`` (FuseShiftPass): a roll by ``cut``
of a tensor zero-padded by ``pad`` and sliced back is a shift by
``((pad + cut) % L) - pad``; for the exported ``cut = c mod L`` with
``|c| <= pad`` this is ``c`` itself (offsets 2, 1, 0, -1, -2).

This module is independent of the product's C++ loader on purpose: the two
readers check each other through the parity tests.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

_DT = {1: np.float32, 6: np.int32, 7: np.int64, 11: np.float64}


def _varint(b: bytes, i: int):
    r = 0
    s = 0
    while True:
        c = b[i]
        i += 1
        r |= (c & 0x7F) << s
        s += 7
        if c < 0x80:
            return r, i


def _fields(b: bytes):
    i, n = 0, len(b)
    while i < n:
        key, i = _varint(b, i)
        f, t = key >> 3, key & 7
        if t == 0:
            v, i = _varint(b, i)
        elif t == 1:
            v = b[i:i + 8]
            i += 8
        elif t == 5:
            v = b[i:i + 4]
            i += 4
        elif t == 2:
            ln, i = _varint(b, i)
            v = b[i:i + ln]
            i += ln
        else:
            raise ValueError(f"unsupported protobuf wire type {t}")
        yield f, t, v


def _signed(v: int) -> int:
    return v - (1 << 64) if v >= (1 << 63) else v


def _ints(t: int, v) -> list[int]:
    if t == 0:
        return [_signed(v)]
    out, i = [], 0
    while i < len(v):
        x, i = _varint(v, i)
        out.append(_signed(x))
    return out


def _tensor(b: bytes):
    dims, name, dt, raw, fl, i64 = [], "", 0, b"", [], []
    for f, t, v in _fields(b):
        if f == 1:
            dims += _ints(t, v)
        elif f == 2:
            dt = v
        elif f == 4:
            fl += list(struct.unpack("<%df" % (len(v) // 4), v)) if t == 2 else [struct.unpack("<f", v)[0]]
        elif f == 7:
            i64 += _ints(t, v)
        elif f == 8:
            name = v.decode()
        elif f == 9:
            raw = v
    if raw:
        arr = np.frombuffer(raw, dtype=_DT[dt]).copy()
    elif fl:
        arr = np.array(fl, dtype=np.float32)
    elif i64:
        arr = np.array(i64, dtype=np.int64)
    else:
        arr = np.zeros(0, dtype=_DT.get(dt, np.float32))
    return name, arr.reshape(dims) if dims else arr.reshape(())


@dataclass
class Node:
    op: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


def _attr(b: bytes):
    name, val = "", None
    ints, floats = [], []
    for f, t, v in _fields(b):
        if f == 1:
            name = v.decode()
        elif f == 2:
            val = struct.unpack("<f", v)[0]
        elif f == 3:
            val = _signed(v)
        elif f == 4:
            val = v
        elif f == 7:
            floats += list(struct.unpack("<%df" % (len(v) // 4), v)) if t == 2 else [struct.unpack("<f", v)[0]]
        elif f == 8:
            ints += _ints(t, v)
    if val is None:
        val = ints or floats
    return name, val


def _node(b: bytes) -> Node:
    n = Node("", [], [])
    for f, t, v in _fields(b):
        if f == 1:
            n.inputs.append(v.decode())
        elif f == 2:
            n.outputs.append(v.decode())
        elif f == 4:
            n.op = v.decode()
        elif f == 5:
            k, a = _attr(v)
            n.attrs[k] = a
    return n


class OnnxGraph:
    """Nodes and initialisers of one ONNX model."""

    def __init__(self, data: bytes):
        graph = None
        for f, t, v in _fields(data):
            if f == 7:
                graph = v
        if graph is None:
            raise ValueError("no GraphProto in model")
        self.nodes: list[Node] = []
        self.inits: dict[str, np.ndarray] = {}
        for f, t, v in _fields(graph):
            if f == 1:
                self.nodes.append(_node(v))
            elif f == 5:
                name, arr = _tensor(v)
                self.inits[name] = arr
        for n in self.nodes:  # Constant nodes behave as initialisers
            if n.op == "Constant" and "value" in n.attrs:
                _, arr = _tensor(n.attrs["value"])
                self.inits[n.outputs[0]] = arr
        self._producer = {o: n for n in self.nodes for o in n.outputs}

    @classmethod
    def load(cls, path) -> "OnnxGraph":
        with open(path, "rb") as fh:
            return cls(fh.read())

    def init(self, name: str) -> np.ndarray:
        return self.inits[name]

    def consumers(self, value: str):
        return [n for n in self.nodes if value in n.inputs]

    def gemm_weight(self, bias_name: str) -> np.ndarray:
        """[K][N] B operand of the Gemm whose C operand is `bias_name` (transB=0)."""
        for n in self.nodes:
            if n.op == "Gemm" and len(n.inputs) > 2 and n.inputs[2] == bias_name:
                if n.attrs.get("transB", 0) not in (0, [], None):
                    raise ValueError("transB Gemm not expected")
                return self.inits[n.inputs[1]]
        raise KeyError(bias_name)

    def shifts(self):
        """Per shift-MLP Split (graph order): (axis, group_ends, offsets)."""
        out = []
        for n in self.nodes:
            if n.op != "Split":
                continue
            pad = self._producer[n.inputs[0]]
            if pad.op != "Pad":
                raise ValueError("Split not fed by Pad")
            pads = self.inits[pad.inputs[1]].astype(np.int64)
            C = None
            if len(n.inputs) > 1 and n.inputs[1]:
                sizes = [int(s) for s in self.inits[n.inputs[1]]]
            else:
                sizes = None  # num_outputs: ceil chunks, resolved once C is known
            axis, offs = None, []
            for o in n.outputs:
                sl = [m for m in self.consumers(o) if m.op == "Slice"]
                first = None
                for m in sl:  # the head slice starts at constant 0
                    if m.inputs[1] in self.inits and int(self.inits[m.inputs[1]].reshape(-1)[0]) == 0:
                        first = m
                if first is None:
                    raise ValueError("roll pattern not found")
                ax = int(self.inits[first.inputs[3]].reshape(-1)[0])
                mod = self._producer[first.inputs[2]]
                if mod.op != "Mod":
                    raise ValueError("roll cut is not a Mod")
                c = int(self.inits[mod.inputs[0]].reshape(-1)[0])
                p = int(pads[ax])
                # ChannelShiftOp.cs:158-161 offset = ((pad + cut) % L) - pad, cut = c mod L
                # with L = n + 2*pad > 2*pad >= |c| this is exactly c.
                if abs(c) > p:
                    raise ValueError("shift larger than its zero pad")
                offs.append(c)
                if axis is None:
                    axis = ax
                elif axis != ax:
                    raise ValueError("mixed shift axes")
            out.append((axis, sizes, offs, n.attrs.get("num_outputs")))
        return out


def split_sizes(C: int, sizes, num_outputs):
    if sizes is not None:
        if sum(sizes) != C:
            raise ValueError("split sizes do not cover C")
        return list(sizes)
    k = int(num_outputs)
    chunk = -(-C // k)  # ONNX Split num_outputs: ceil chunks, last smaller
    s = [chunk] * (k - 1) + [C - chunk * (k - 1)]
    return s
