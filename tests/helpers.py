"""Shared test helpers: seeded inputs, single-op graphs, tolerance checks."""

from __future__ import annotations

import numpy as np

from mlvc_b200.graph import GraphBuilder

# Per-op tolerance of the north-star contract: FP16 outputs within max-abs
# 2e-2 and relative L2 1e-3 of an FP32-accumulation reference.
MAX_ABS = 2e-2
REL_L2 = 1e-3


def lcg_values(count, seed):
    """The reference kernel tests' generator (tests/unit/cutlass_kernel_tests.cpp:26-34):
    seed = seed*1664525 + 1013904223 (mod 2^32); value = (int(seed >> 24) - 128) / 256."""
    out = np.empty(count, np.float32)
    s = seed & 0xFFFFFFFF
    for i in range(count):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = ((s >> 24) - 128) / 256.0
    return out.astype(np.float16)


def lcg_fast(count, seed):
    """Vectorised form of lcg_values (same sequence)."""
    a, c, m = 1664525, 1013904223, 1 << 32
    out = np.empty(count, np.uint64)
    s = seed % m
    # jump ahead in blocks to keep it vectorised
    block = 4096
    mult = np.empty(block, np.uint64)
    add = np.empty(block, np.uint64)
    ma, ca = 1, 0
    for i in range(block):
        ma, ca = (ma * a) % m, (ca * a + c) % m
        mult[i], add[i] = ma, ca
    for start in range(0, count, block):
        n = min(block, count - start)
        out[start:start + n] = (mult[:n] * np.uint64(s) + add[:n]) % np.uint64(m)
        s = int(out[start + n - 1])
    return ((((out >> np.uint64(24)).astype(np.int64)) - 128) / 256.0).astype(np.float16)


def compare(actual, expected, max_abs=MAX_ABS, rel_l2=REL_L2):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.isfinite(a).all(), "non-finite output"
    err = np.abs(a - e)
    mx = float(err.max()) if err.size else 0.0
    rl = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
    assert mx <= max_abs and rl <= rel_l2, f"max-abs {mx:.3g} (<= {max_abs}), rel-L2 {rl:.3g} (<= {rel_l2})"
    return mx, rl


def bits_equal(actual, expected):
    a = np.ascontiguousarray(actual, np.float16).view(np.uint16)
    e = np.ascontiguousarray(expected, np.float16).view(np.uint16)
    mism = int((a != e).sum())
    assert mism == 0, f"{mism} of {a.size} FP16 values differ"


def conv_graph(x_shape, w, b=None, stride=(1, 1), pad=(0, 0), groups=1, epilogue=None, residual_shape=None):
    """One conv (+ optional fused-pattern tail) as a graph."""
    gb = GraphBuilder()
    x = gb.input("x", x_shape)
    wn = gb.weight("w", w)
    bn = gb.weight("b", b) if b is not None else None
    y = gb.conv(x, wn, bn, stride, pad, groups)
    if epilogue == "leaky":
        y = gb.leaky_relu(y, 0.01)
    elif epilogue == "residual":
        r = gb.input("r", residual_shape or gb.shape(y))
        y = gb.add(r, y)
    elif epilogue == "reglu":
        c = gb.shape(y)[1] // 2
        g = gb.slice(y, 1, 0, c)
        lin = gb.slice(y, 1, c, 2 * c)
        y = gb.mul(gb.clip(g, 0.0, 1.0), lin)
    gb.output(y, "y")
    return gb


# FP16 spacing grows with magnitude (2^-7 at |x| = 8, 2^-5 at 32), so an
# absolute bound only means something near unit scale.  The per-op contract
# (max-abs 2e-2, rel-L2 1e-3 against FP32 accumulation) is applied with the
# absolute bound scaled by max(1, m / 8), m = |expected| or, for elementwise
# operators, the largest magnitude among the operator's inputs at that element
# (a one-ulp difference of a large operand survives cancellation): 2e-2 at
# m <= 8, about 2.5 FP16 ulps of m above.
def compare_scaled(actual, expected, max_abs=MAX_ABS, rel_l2=REL_L2, magnitude=None):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.isfinite(a).all(), "non-finite output"
    m = np.abs(e) if magnitude is None else np.maximum(np.abs(e), magnitude)
    scale = np.maximum(1.0, m / 8.0)
    se = np.abs(a - e) / scale
    err = float(se.max()) if a.size else 0.0
    rl = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
    if not (err <= max_abs and rl <= rel_l2):
        i = np.unravel_index(int(np.argmax(se)), se.shape)
        raise AssertionError(f"scaled max-abs {err:.3g} (<= {max_abs}), rel-L2 {rl:.3g} (<= {rel_l2}); "
                             f"{int((se > max_abs).sum())} of {se.size} over; worst at {tuple(int(v) for v in i)}: "
                             f"got {a[i]!r} want {e[i]!r} magnitude {m[i]!r}")
    return err, rl


# Whole-graph limits when rounding differences compound through many layers:
# the reference's own tensor conformance rule (docs/codec-compatibility.md:
# FP16 tensors max-abs <= 0.25), scaled as above, with rel-L2 1e-3.
STACK_MAX_ABS = 0.25


def per_op_parity(backend, graph, weights, inputs, conv_impl="c"):
    """Checks every tensor the GPU materialised against the oracle applied to the
    GPU's own inputs of that step (so errors do not compound across steps).
    Chain-internal values of fused steps are recomputed by the oracle from the
    GPU's chain input.  Returns the number of checked tensors."""
    from oracle.graph_oracle import GraphOracle
    o = GraphOracle(graph, weights, conv_impl)
    vals = dict(o.consts)
    for tid, arr in zip(o.g.inputs, inputs):
        vals[tid] = np.asarray(arr)
    checked = 0
    for node in o.g.nodes:
        out_t = o.tensors[node.outputs[0]]
        want = o._exec(node, vals, out_t)
        dt = np.int32 if out_t.dtype == 2 else np.float16
        got = backend.read_tensor(out_t.name, tuple(out_t.shape), dt)
        if got is not None:
            mag = None
            if node.op in (1, 2, 3):  # Add / Sub / Mul: operand magnitudes
                ops = [np.abs(np.asarray(vals[i], np.float64)) for i in node.inputs]
                mag = np.broadcast_to(np.maximum(*np.broadcast_arrays(*ops)), want.shape)
            try:
                compare_scaled(got, want, magnitude=mag)
            except AssertionError as e:
                ctx = ""
                if node.op in (1, 2, 3):
                    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
                    i = np.unravel_index(int(np.argmax(d)), d.shape)
                    ctx = "; operands " + ", ".join(
                        repr(np.broadcast_to(np.asarray(vals[k]), want.shape)[i]) for k in node.inputs)
                raise AssertionError(f"node {out_t.name} (op {node.op}): {e}{ctx}") from None
            vals[node.outputs[0]] = got
            checked += 1
        else:
            vals[node.outputs[0]] = want
    return checked
