"""Node-by-node CPU interpreter of an mlvc AOT graph (NCHW, FP16 storage).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg as the checker.  The product never imports it.

Semantics follow the reference runtime contract:
  * graph decoding / operand order: runtime/src/aot_graph.cpp:110-283
  * per-op arithmetic and FP16 rounding points: backends/driver_cubin/kernels/
    elementwise.cu:23-79, tensor_ops.cu:1-116, generic_conv.cu:1-82 and the CPU
    scalar kernels backends/cpu/src/kernels_scalar.cpp:112-196 (restated in C
    in mlvc_oracle.c)
  * Slice reads starts/axes/steps from int64 initialisers and takes the output
    extent from the output tensor (backends/driver_cubin/src/execution_plan.cpp:493-535)
  * the same interpreter shape as the reference's own independent replay
    tests/unit/aot_tests.py:21-61, but with explicit FP32-accumulate FP16
    arithmetic instead of PyTorch.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

from .wire_schema import OP_NAMES, parse_graph

_HERE = Path(__file__).resolve().parent
_LIB = None


def lib():
    """Load liboracle.so (built by `make -C oracle oracle`)."""
    global _LIB
    if _LIB is None:
        path = _HERE / "liboracle.so"
        if not path.exists():
            raise RuntimeError(f"oracle library missing: {path} (run make -C oracle)")
        l = ctypes.CDLL(str(path))
        u16p = ctypes.POINTER(ctypes.c_uint16)
        l.oracle_conv2d.argtypes = [u16p, u16p, u16p, u16p] + [ctypes.c_int] * 15 + [ctypes.c_float, u16p]
        l.oracle_unary.argtypes = [u16p, u16p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float]
        i64p = ctypes.POINTER(ctypes.c_int64)
        l.oracle_binary.argtypes = [u16p, u16p, u16p, i64p, i64p, i64p, ctypes.c_int]
        _LIB = l
    return _LIB


def _p16(a):
    if a is None:
        return None
    assert a.dtype == np.float16 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))


def conv2d(x, w, b=None, stride=(1, 1), pad=(0, 0), groups=1, epilogue=0, alpha=0.01, residual=None):
    """NCHW FP16 conv, FP32 accumulation, bias-first, one FP16 rounding; optional
    fused LeakyReLU (1) / residual add (2) with a second rounding."""
    x = np.ascontiguousarray(x, np.float16)
    w = np.ascontiguousarray(w, np.float16)
    n, ic, ih, iw = x.shape
    oc, _, kh, kw = w.shape
    oh = (ih + 2 * pad[0] - kh) // stride[0] + 1
    ow = (iw + 2 * pad[1] - kw) // stride[1] + 1
    y = np.empty((n, oc, oh, ow), np.float16)
    bb = None if b is None else np.ascontiguousarray(b, np.float16).reshape(-1)
    rr = None if residual is None else np.ascontiguousarray(residual, np.float16)
    lib().oracle_conv2d(_p16(x), _p16(w), _p16(bb), _p16(y), n, ic, ih, iw, oc, oh, ow, kh, kw,
                        stride[0], stride[1], pad[0], pad[1], groups, epilogue, alpha, _p16(rr))
    return y


def conv2d_gemm(x, w, b=None, stride=(1, 1), pad=(0, 0), groups=1):
    """Same operator as conv2d (bias added to the FP32 accumulator, one FP16
    rounding) computed as an im2col FP32 GEMM with numpy.  The summation order
    differs from the scalar loop, so results agree to FP32 accumulation error,
    not bit for bit; used for shapes the scalar loop would take minutes on."""
    x = np.asarray(x, np.float16)
    w = np.asarray(w, np.float16)
    n, ic, ih, iw = x.shape
    oc, icg, kh, kw = w.shape
    oh = (ih + 2 * pad[0] - kh) // stride[0] + 1
    ow = (iw + 2 * pad[1] - kw) // stride[1] + 1
    xp = np.zeros((n, ic, ih + 2 * pad[0], iw + 2 * pad[1]), np.float32)
    xp[:, :, pad[0]:pad[0] + ih, pad[1]:pad[1] + iw] = x
    ocg = oc // groups
    y = np.empty((n, oc, oh * ow), np.float32)
    for g in range(groups):
        cols = np.empty((n, icg, kh, kw, oh, ow), np.float32)
        for ky in range(kh):
            for kx in range(kw):
                cols[:, :, ky, kx] = xp[:, g * icg:(g + 1) * icg, ky:ky + stride[0] * oh:stride[0],
                                        kx:kx + stride[1] * ow:stride[1]]
        wg = w[g * ocg:(g + 1) * ocg].reshape(ocg, -1).astype(np.float32)
        for b_ in range(n):
            y[b_, g * ocg:(g + 1) * ocg] = wg @ cols[b_].reshape(icg * kh * kw, -1)
    if b is not None:
        y += np.asarray(b, np.float16).astype(np.float32).reshape(1, oc, 1)
    return y.reshape(n, oc, oh, ow).astype(np.float16)


def unary(x, op, alpha=0.01, lo=-np.inf, hi=np.inf):
    x = np.ascontiguousarray(x, np.float16)
    y = np.empty_like(x)
    lib().oracle_unary(_p16(x), _p16(y), x.size, op, alpha, lo, hi)
    return y


def _dims4(shape):
    s = list(shape)
    return [1] * (4 - len(s)) + s


def binary(a, b, op):
    a = np.ascontiguousarray(a, np.float16)
    b = np.ascontiguousarray(b, np.float16)
    out_shape = np.broadcast_shapes(a.shape, b.shape)
    y = np.empty(out_shape, np.float16)
    arr = lambda s: (ctypes.c_int64 * 4)(*_dims4(s))
    lib().oracle_binary(_p16(a), _p16(b), _p16(y), arr(out_shape), arr(a.shape), arr(b.shape), op)
    return y


def depth_to_space(x, r):
    n, c, h, w = x.shape
    return np.ascontiguousarray(x.reshape(n, c // (r * r), r, r, h, w).transpose(0, 1, 4, 2, 5, 3).reshape(n, c // (r * r), h * r, w * r))


def space_to_depth(x, r):
    n, c, h, w = x.shape
    return np.ascontiguousarray(x.reshape(n, c, h // r, r, w // r, r).transpose(0, 1, 3, 5, 2, 4).reshape(n, c * r * r, h // r, w // r))


class GraphOracle:
    """Loads graph.pb + weights.bin and runs the graph on NCHW numpy inputs."""

    def __init__(self, graph_bytes: bytes, weights: bytes, conv_impl: str = "c"):
        """conv_impl "c": scalar FP32 loop in the reference's summation order
        (bit-exact against the reference CPU backend's scalar kernels);
        "gemm": numpy FP32 GEMM for large graphs."""
        self.conv_impl = conv_impl
        self.g = parse_graph(graph_bytes)
        if self.g.schema_version != 3:
            raise ValueError("unsupported schema")
        self.tensors = {t.id: t for t in self.g.tensors}
        self.consts = {}
        for t in self.g.tensors:
            if t.WhichOneof("storage") == "weight":
                dt = {1: np.float16, 3: np.int64}[t.dtype]
                cnt = t.weight.size_bytes // np.dtype(dt).itemsize
                self.consts[t.id] = np.frombuffer(weights, dt, cnt, t.weight.offset).reshape(tuple(t.shape)).copy()

    @classmethod
    def from_dir(cls, model_dir, part, conv_impl="c"):
        d = Path(model_dir) / "aot" / part
        return cls((d / "graph.pb").read_bytes(), (d / "weights.bin").read_bytes(), conv_impl)

    def input_names(self):
        return [self.tensors[i].name for i in self.g.inputs]

    def output_names(self):
        return [self.tensors[i].name for i in self.g.outputs]

    def run(self, inputs, keep_all=False):
        vals = dict(self.consts)
        for tid, arr in zip(self.g.inputs, inputs, strict=True):
            t = self.tensors[tid]
            want = np.int32 if t.dtype == 2 else np.float16
            arr = np.asarray(arr)
            if arr.dtype != want or list(arr.shape) != list(t.shape):
                raise ValueError(f"input {t.name}: expected {want} {list(t.shape)}, got {arr.dtype} {list(arr.shape)}")
            vals[tid] = arr
        for node in self.g.nodes:
            out_t = self.tensors[node.outputs[0]]
            vals[node.outputs[0]] = self._exec(node, vals, out_t)
        result = [vals[i] for i in self.g.outputs]
        return (result, {self.tensors[k].name: v for k, v in vals.items()}) if keep_all else result

    def _scalar(self, vals, tid, default):
        if tid == 0:
            return default
        return float(np.asarray(vals[tid], np.float32).reshape(-1)[0])

    def _exec(self, node, vals, out_t):
        op = OP_NAMES[node.op]
        ins = list(node.inputs)
        a = lambda i: vals[ins[i]]
        out_shape = tuple(out_t.shape)
        if op == "Conv":
            c = node.conv
            b = a(2) if len(ins) > 2 and ins[2] != 0 else None
            f = conv2d if self.conv_impl == "c" else conv2d_gemm
            y = f(a(0), a(1), b, tuple(c.strides), tuple(c.pads[:2]), c.groups)
        elif op in ("Add", "Mul", "Sub"):
            y = binary(a(0), a(1), {"Add": 0, "Mul": 1, "Sub": 2}[op])
        elif op == "LeakyRelu":
            y = unary(a(0), 0, alpha=node.activation.alpha)
        elif op == "Clip":
            lo = self._scalar(vals, ins[1], -np.inf) if len(ins) > 1 else -np.inf
            hi = self._scalar(vals, ins[2], np.inf) if len(ins) > 2 else np.inf
            y = unary(a(0), 1, lo=lo, hi=hi)
        elif op in ("Sigmoid", "Reciprocal", "Round"):
            y = unary(a(0), {"Sigmoid": 2, "Reciprocal": 3, "Round": 4}[op])
        elif op == "Slice":
            x = a(0)
            starts = vals[ins[1]].reshape(-1)
            axes = vals[ins[3]].reshape(-1) if len(ins) > 3 and ins[3] else np.arange(len(starts))
            steps = vals[ins[4]].reshape(-1) if len(ins) > 4 and ins[4] else np.ones(len(starts), np.int64)
            sl = [slice(None)] * x.ndim
            for s, ax, st in zip(starts, axes, steps):
                ax = int(ax) + (x.ndim if ax < 0 else 0)
                s = int(s) + (x.shape[ax] if s < 0 else 0)
                # clamped to [0, dim] (backends/cpu/src/execution_plan.cpp:596-599)
                s = min(max(s, 0), x.shape[ax])
                sl[ax] = slice(s, s + int(st) * out_shape[ax], int(st))
            y = np.ascontiguousarray(x[tuple(sl)])
        elif op == "Concat":
            y = np.concatenate([vals[i] for i in ins], axis=node.axis.axis)
        elif op == "Gather":
            data, idx = a(0), int(np.asarray(a(1)).reshape(-1)[0])
            if idx < 0:
                idx += data.shape[0]
            y = np.ascontiguousarray(data[idx:idx + 1])
        elif op == "DepthToSpace":
            y = depth_to_space(a(0), node.pixel.block_size)
        elif op == "SpaceToDepth":
            y = space_to_depth(a(0), node.pixel.block_size)
        else:
            raise ValueError(f"unsupported op {op}")
        y = np.asarray(y)
        if y.dtype == np.float32:
            y = y.astype(np.float16)
        return y.reshape(out_shape)
