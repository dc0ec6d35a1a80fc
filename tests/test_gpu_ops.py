"""Operator parity on the B200: each case is a one-operator (or one fused
chain) graph run through the product's C ABI (load -> run) and compared with
the CPU oracle on the same seeded inputs.

Conv cases mirror the reference's kernel tests (tests/unit/cutlass_kernel_tests.cpp:
GEMM shapes M=OC, N=H*W, K=IC at :345-348 with the LCG inputs of :26-34, the
spatial convs of :355-358 on a 13x17 image, pixel (un)shuffle order for
factors 2 and 8 at :43-89) plus the shapes of the benchmark workloads.
Tolerance for convolutions: max-abs 2e-2 and relative L2 1e-3 against FP32
accumulation; elementwise, layout and data-movement operators are bit-exact.
"""

import numpy as np
import pytest

from helpers import bits_equal, compare, conv_graph, lcg_fast
from mlvc_b200 import Backend
from mlvc_b200.graph import GraphBuilder
from oracle.graph_oracle import GraphOracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def device():
    return 0


def run_both(gb, inputs, conv_impl="c", state_bindings=()):
    graph, weights = gb.finish()
    be = Backend(0)
    be.load_memory(graph, weights, state_bindings)
    got = be.run(inputs)
    want = GraphOracle(graph, weights, conv_impl).run(inputs)
    return got, want, be


# ------------------------------------------------------------ convolutions
GEMM_SHAPES = [  # (OC, H, W, IC): reference shapes (OC, HW, IC) with HW = H*W
    (136, 23, 40, 24), (136, 23, 40, 72), (136, 23, 40, 128), (128, 16, 16, 32), (8, 2, 4, 8), (256, 24, 40, 512),
    # benchmark block-stack shapes
    (256, 92, 160, 128), (128, 92, 160, 256), (512, 92, 160, 128), (64, 13, 17, 64),
]


@pytest.mark.parametrize("oc,h,w,ic", GEMM_SHAPES)
@pytest.mark.parametrize("epilogue", [None, "leaky", "residual"])
def test_conv1x1(oc, h, w, ic, epilogue):
    x = lcg_fast(ic * h * w, 1).reshape(1, ic, h, w)
    wt = lcg_fast(oc * ic, 2).reshape(oc, ic, 1, 1)
    b = lcg_fast(oc, 3)
    gb = conv_graph(x.shape, wt, b, epilogue=epilogue)
    inputs = [x]
    if epilogue == "residual":
        inputs.append(lcg_fast(oc * h * w, 4).reshape(1, oc, h, w))
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    kernels = {s["kernel"] for s in be.steps()}
    assert "mlvc_conv1x1_tc" in kernels, kernels


@pytest.mark.parametrize("c,h,w", [(128, 92, 160), (64, 13, 17), (256, 8, 8)])
def test_conv1x1_reglu(c, h, w):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16)
    wt = (rng.standard_normal((4 * c, c, 1, 1), dtype=np.float32) * np.sqrt(2.0 / c)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, 4 * c).astype(np.float16)
    gb = conv_graph(x.shape, wt, b, epilogue="reglu")
    got, want, be = run_both(gb, [x])
    compare(got[0], want[0])
    steps = be.steps()
    assert len([s for s in steps if s["kernel"] != "mlvc_boundary_f16"]) == 1, steps


FFN_CASES = [  # (C, hidden, C_out, H, W, epilogue of the second conv)
    (128, 256, 128, 92, 160, "residual"),  # block-stack FFN (residual = FFN input)
    (64, 64, 64, 13, 17, None),            # one hidden chunk, ragged last tile
    (256, 128, 128, 8, 20, "leaky"),       # four input panels
    (128, 256, 128, 160, 160, "residual"), # 200 tiles: two tiles per CTA, two X buffers
    (64, 192, 64, 20, 30, "residual"),     # three hidden chunks
    (64, 128, 64, 20, 30, "residual_other"),  # residual is not the FFN input: two separate convs
]


def _ffn_graph(c, hidden, c_out, h, w, epilogue, seed=21):
    rng = np.random.default_rng(seed)
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    w1 = gb.weight("w1", (rng.standard_normal((2 * hidden, c, 1, 1), dtype=np.float32) * np.sqrt(2.0 / c)).astype(np.float16))
    b1 = gb.weight("b1", rng.uniform(-0.1, 0.1, 2 * hidden).astype(np.float16))
    w2 = gb.weight("w2", (rng.standard_normal((c_out, hidden, 1, 1), dtype=np.float32) * np.sqrt(1.0 / hidden)).astype(np.float16))
    b2 = gb.weight("b2", rng.uniform(-0.1, 0.1, c_out).astype(np.float16))
    t = gb.conv(x, w1, b1)
    gate = gb.slice(t, 1, 0, hidden)
    lin = gb.slice(t, 1, hidden, 2 * hidden)
    hid = gb.mul(gb.clip(gate, 0.0, 1.0), lin)  # node order of the exported ReGLU tail
    y = gb.conv(hid, w2, b2)
    inputs = [rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16)]
    if epilogue == "residual":
        y = gb.add(y, x)
    elif epilogue == "residual_other":
        r = gb.input("r", [1, c_out, h, w])
        y = gb.add(r, y)
        inputs.append(rng.standard_normal((1, c_out, h, w), dtype=np.float32).astype(np.float16))
    elif epilogue == "leaky":
        y = gb.leaky_relu(y, 0.01)
    gb.output(y, "y")
    return gb, inputs


@pytest.mark.parametrize("c,hidden,c_out,h,w,epilogue", FFN_CASES)
def test_ffn_fused(c, hidden, c_out, h, w, epilogue, monkeypatch):
    """Conv1x1 -> ReGLU -> Conv1x1 (+ residual / LeakyReLU) as one kernel with
    the hidden tensor on chip: parity with the oracle, and bit-identical to the
    same graph planned as separate tensor-core convs (same accumulation order,
    same FP16 roundings)."""
    gb, inputs = _ffn_graph(c, hidden, c_out, h, w, epilogue)
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    kernels = [s["kernel"] for s in be.steps() if s["kernel"] != "mlvc_boundary_f16"]
    if epilogue == "residual_other":
        assert kernels == ["mlvc_conv1x1_tc", "mlvc_conv1x1_tc"], kernels
        return
    assert kernels == ["mlvc_ffn_tc"], kernels
    graph, weights = gb.finish()
    monkeypatch.setenv("MLVC_B200_FFN_FUSION", "0")
    split = Backend(0)
    split.load_memory(graph, weights)
    assert "mlvc_ffn_tc" not in {s["kernel"] for s in split.steps()}
    bits_equal(split.run(inputs)[0], got[0])


DW_CASES = [  # (C, C_out, H, W, epilogue of the 1x1 conv)
    (256, 128, 92, 160, "residual"),  # block-stack shape (bottom tile row half inside the image)
    (64, 64, 13, 21, None),           # ragged tiles on both edges, odd width
    (128, 128, 9, 300, "leaky"),      # wide image
    (64, 64, 160, 160, "residual"),   # 200 tiles: two tiles per CTA
    (64, 256, 8, 8, None),            # 256 output columns (four staging panels)
    (512, 256, 34, 60, "residual"),   # taps in two 256-channel boxes (MLVC-width block)
    (320, 128, 13, 21, None),         # taps in a 256- and a 64-channel box
]


@pytest.mark.parametrize("c,c_out,h,w,epilogue", DW_CASES)
def test_dwconv_fused(c, c_out, h, w, epilogue, monkeypatch):
    """Depthwise 3x3 -> 1x1 conv (+ residual / LeakyReLU) as one kernel, the
    depthwise result written straight into the tensor-core A operand: parity
    with the oracle, and bit-identical to the two stand-alone kernels."""
    rng = np.random.default_rng(31)
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    dw = gb.weight("dw", (rng.standard_normal((c, 1, 3, 3), dtype=np.float32) / 3.0).astype(np.float16))
    db = gb.weight("db", rng.uniform(-0.1, 0.1, c).astype(np.float16))
    d = gb.conv(x, dw, db, (1, 1), (1, 1), groups=c)
    wt = gb.weight("w", (rng.standard_normal((c_out, c, 1, 1), dtype=np.float32) * np.sqrt(1.0 / c)).astype(np.float16))
    b = gb.weight("b", rng.uniform(-0.1, 0.1, c_out).astype(np.float16))
    y = gb.conv(d, wt, b)
    inputs = [rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16)]
    if epilogue == "residual":
        r = gb.input("r", [1, c_out, h, w])
        y = gb.add(y, r)
        inputs.append(rng.standard_normal((1, c_out, h, w), dtype=np.float32).astype(np.float16))
    elif epilogue == "leaky":
        y = gb.leaky_relu(y, 0.01)
    gb.output(y, "y")
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    kernels = [s["kernel"] for s in be.steps() if s["kernel"] != "mlvc_boundary_f16"]
    assert kernels == ["mlvc_dwconv_tc"], kernels
    graph, weights = gb.finish()
    monkeypatch.setenv("MLVC_B200_DW_FUSION", "0")
    split = Backend(0)
    split.load_memory(graph, weights)
    assert "mlvc_dwconv_tc" not in {s["kernel"] for s in split.steps()}
    bits_equal(split.run(inputs)[0], got[0])


MB_CASES = [  # (C, E, C_out, H, W, LeakyReLU after the expand conv, epilogue of the projection)
    (128, 256, 128, 92, 160, True, "residual_x"),  # the block stack's block (residual = block input)
    (64, 128, 64, 13, 21, False, None),            # ragged tiles on both edges, odd width
    (128, 256, 128, 9, 300, True, "leaky"),        # wide image
    (64, 64, 64, 160, 160, True, "residual"),      # one expand chunk; 200 tiles: two tiles per CTA
    (64, 192, 64, 8, 8, True, "residual_x"),       # three expand chunks (odd), one tile, half outside
    (128, 128, 64, 23, 40, True, "residual"),      # two chunks, residual from another tensor
]


@pytest.mark.parametrize("c,e,c_out,h,w,leaky,epilogue", MB_CASES)
def test_mbconv_fused(c, e, c_out, h, w, leaky, epilogue, monkeypatch):
    """1x1 expand (+ LeakyReLU) -> depthwise 3x3 -> 1x1 projection (+ residual /
    LeakyReLU) as one kernel, the expanded tensor and the depthwise result kept
    in shared memory: parity with the oracle, and bit-identical to the
    expand-conv + fused-depthwise schedule."""
    rng = np.random.default_rng(37)
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    w1 = gb.weight("w1", (rng.standard_normal((e, c, 1, 1), dtype=np.float32) * np.sqrt(2.0 / c)).astype(np.float16))
    b1 = gb.weight("b1", rng.uniform(-0.1, 0.1, e).astype(np.float16))
    t = gb.conv(x, w1, b1)
    if leaky:
        t = gb.leaky_relu(t, 0.01)
    dw = gb.weight("dw", (rng.standard_normal((e, 1, 3, 3), dtype=np.float32) / 3.0).astype(np.float16))
    db = gb.weight("db", rng.uniform(-0.1, 0.1, e).astype(np.float16))
    d = gb.conv(t, dw, db, (1, 1), (1, 1), groups=e)
    w2 = gb.weight("w2", (rng.standard_normal((c_out, e, 1, 1), dtype=np.float32) * np.sqrt(1.0 / e)).astype(np.float16))
    b2 = gb.weight("b2", rng.uniform(-0.1, 0.1, c_out).astype(np.float16))
    y = gb.conv(d, w2, b2)
    inputs = [rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16)]
    if epilogue == "residual_x":
        assert c_out == c
        y = gb.add(x, y)
    elif epilogue == "residual":
        r = gb.input("r", [1, c_out, h, w])
        y = gb.add(y, r)
        inputs.append(rng.standard_normal((1, c_out, h, w), dtype=np.float32).astype(np.float16))
    elif epilogue == "leaky":
        y = gb.leaky_relu(y, 0.01)
    gb.output(y, "y")
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    kernels = [s["kernel"] for s in be.steps() if s["kernel"] != "mlvc_boundary_f16"]
    assert kernels == ["mlvc_mbconv_tc"], kernels
    graph, weights = gb.finish()
    monkeypatch.setenv("MLVC_B200_MB_FUSION", "0")
    split = Backend(0)
    split.load_memory(graph, weights)
    assert "mlvc_mbconv_tc" not in {s["kernel"] for s in split.steps()}
    bits_equal(split.run(inputs)[0], got[0])


SPATIAL = [  # (IC, OC, stride, kernel, pad, H, W)
    (24, 24, 1, 3, 1, 13, 17), (40, 264, 2, 3, 1, 13, 17), (8, 8, 2, 2, 0, 13, 17), (128, 256, 2, 2, 0, 13, 17),
    (64, 64, 1, 3, 1, 13, 17), (64, 128, 2, 3, 1, 13, 17), (64, 64, 1, 3, 1, 46, 300), (128, 64, 1, 3, 1, 9, 140),
    (64, 64, 1, 1, 0, 13, 17), (64, 96, 2, 3, 1, 24, 258),
]


@pytest.mark.parametrize("ic,oc,stride,k,pad,h,w", SPATIAL)
def test_conv_spatial(ic, oc, stride, k, pad, h, w):
    x = lcg_fast(ic * h * w, 5).reshape(1, ic, h, w)
    wt = lcg_fast(oc * ic * k * k, 6).reshape(oc, ic, k, k)
    b = lcg_fast(oc, 7)
    gb = conv_graph(x.shape, wt, b, (stride, stride), (pad, pad))
    got, want, be = run_both(gb, [x])
    compare(got[0], want[0])
    if ic % 64 == 0 and oc % 16 == 0 and k > 1:
        assert "mlvc_convkxk_tc" in {s["kernel"] for s in be.steps()}


@pytest.mark.parametrize("epilogue", ["leaky", "residual"])
def test_conv3x3_fused(epilogue):
    x = lcg_fast(64 * 20 * 33, 8).reshape(1, 64, 20, 33)
    wt = lcg_fast(64 * 64 * 9, 9).reshape(64, 64, 3, 3)
    b = lcg_fast(64, 10)
    gb = conv_graph(x.shape, wt, b, (1, 1), (1, 1), epilogue=epilogue)
    inputs = [x] + ([lcg_fast(64 * 20 * 33, 11).reshape(1, 64, 20, 33)] if epilogue == "residual" else [])
    got, want, _ = run_both(gb, inputs)
    compare(got[0], want[0])


def test_conv3x3_config1_full():
    """Config 1 at its real size (3x3 64->64 @ 184x320), FP32-GEMM oracle."""
    from mlvc_b200.graph import build_conv3x3
    gb, inputs = build_conv3x3(0)
    got, want, be = run_both(gb, inputs, conv_impl="gemm")
    compare(got[0], want[0])
    assert "mlvc_convkxk_tc" in {s["kernel"] for s in be.steps()}


@pytest.mark.parametrize("c,h,w,stride", [(256, 92, 160, 1), (64, 13, 17, 1), (64, 13, 17, 2), (24, 7, 9, 1)])
def test_depthwise(c, h, w, stride):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16)
    wt = (rng.standard_normal((c, 1, 3, 3), dtype=np.float32) * 0.3).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, c).astype(np.float16)
    gb = conv_graph(x.shape, wt, b, (stride, stride), (1, 1), groups=c)
    got, want, _ = run_both(gb, [x])
    compare(got[0], want[0])


def test_grouped_conv():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 12, 9, 10), dtype=np.float32).astype(np.float16)
    wt = (rng.standard_normal((6, 4, 3, 3), dtype=np.float32) * 0.3).astype(np.float16)
    gb = conv_graph(x.shape, wt, None, (1, 1), (1, 1), groups=3)
    got, want, _ = run_both(gb, [x])
    compare(got[0], want[0])


def test_conv_rgb_input():
    """IC = 3 (the codec's first conv) takes the direct fallback."""
    rng = np.random.default_rng(5)
    x = rng.random((1, 3, 16, 24), dtype=np.float32).astype(np.float16)
    wt = (rng.standard_normal((32, 3, 3, 3), dtype=np.float32) * 0.3).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, 32).astype(np.float16)
    gb = conv_graph(x.shape, wt, b, (2, 2), (1, 1))
    got, want, _ = run_both(gb, [x])
    compare(got[0], want[0])


# ---------------------------------------------------- elementwise / layout
def _rand(shape, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * scale).astype(np.float16)


@pytest.mark.parametrize("op", ["add", "sub", "mul"])
@pytest.mark.parametrize("bshape", [(1, 24, 6, 10), (1, 24, 1, 1), (1, 1, 6, 10), (1,), (24, 1, 1)])
def test_binary(op, bshape):
    gb = GraphBuilder()
    a = gb.input("a", [1, 24, 6, 10])
    if bshape == (1, 24, 6, 10):
        b = gb.input("b", list(bshape))
        inputs = [_rand((1, 24, 6, 10), 1), _rand(bshape, 2)]
    else:
        b = gb.weight("b", _rand(bshape, 2))
        inputs = [_rand((1, 24, 6, 10), 1)]
    gb.output(getattr(gb, op)(a, b), "y")
    got, want, _ = run_both(gb, inputs)
    bits_equal(got[0], want[0])


@pytest.mark.parametrize("op", ["LeakyRelu", "Clip", "Sigmoid", "Reciprocal", "Round"])
def test_unary(op):
    gb = GraphBuilder()
    x = gb.input("x", [1, 16, 9, 11])
    if op == "LeakyRelu":
        y = gb.leaky_relu(x, 0.2)
    elif op == "Clip":
        y = gb.clip(x, -0.5, 0.75)
    else:
        y = gb.unary(op, x)
    gb.output(y, "y")
    inputs = [_rand((1, 16, 9, 11), 3, 4.0)]
    got, want, _ = run_both(gb, inputs)
    if op == "Sigmoid":  # expf may differ by an FP32 ulp between libm and CUDA
        compare(got[0], want[0], max_abs=1e-3, rel_l2=1e-3)
    else:
        bits_equal(got[0], want[0])


def test_slice_concat_gather():
    gb = GraphBuilder()
    x = gb.input("x", [1, 32, 8, 12])
    q = gb.input("q", [1], "int32")
    table = gb.weight("table", _rand((5, 32, 1, 1), 9))
    s1 = gb.slice(x, 1, 8, 24)            # channel slice
    s2 = gb.slice(x, 3, 1, 12, 2)         # strided width slice
    s3 = gb.slice(x, 2, 0, 4)
    cat = gb.concat([s1, gb.slice(x, 1, 0, 8)], 1)
    scale = gb.gather(table, q)
    y = gb.mul(x, scale)
    gb.output(cat, "cat")
    gb.output(s2, "s2")
    gb.output(gb.concat([s3, s3], 2), "cat_h")
    gb.output(y, "scaled")
    inputs = [_rand((1, 32, 8, 12), 5), np.array([3], np.int32)]
    got, want, _ = run_both(gb, inputs)
    for g, w_ in zip(got, want):
        bits_equal(g, w_)


@pytest.mark.parametrize("factor", [2, 8])
def test_pixel_shuffle_order(factor):
    """Native CRD channel order, factors 2 and 8 (reference cutlass_kernel_tests.cpp:43-89):
    unshuffle then shuffle must restore the input, and both match the oracle."""
    c, h, w = 3, factor * 2, factor * 3
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    u = gb.output(gb.space_to_depth(x, factor), "unshuffled")
    gb.output(gb.depth_to_space(u, factor), "restored")
    inputs = [np.arange(c * h * w, dtype=np.float32).reshape(1, c, h, w).astype(np.float16)]
    got, want, _ = run_both(gb, inputs)
    bits_equal(got[0], want[0])
    bits_equal(got[1], inputs[0])


@pytest.mark.parametrize("factor,c", [(2, 2), (2, 6), (4, 2), (8, 3)])
def test_pixel_shuffle_boundary_vector_paths(factor, c):
    """Unshuffle at a graph input and shuffle at a graph output with extents
    that take the boundary kernel's 16-byte paths (device channels and host
    row spans multiples of 8), a partial 32-pixel band included."""
    h, w = factor * 3, factor * 40
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    u = gb.space_to_depth(x, factor)
    gb.output(gb.depth_to_space(gb.mul(u, gb.weight("s", _rand((1, c * factor * factor, 1, 1), 4))), factor), "y")
    inputs = [_rand((1, c, h, w), 6)]
    got, want, _ = run_both(gb, inputs)
    bits_equal(got[0], want[0])


@pytest.mark.parametrize("c1,c2,oc,epilogue", [(128, 128, 256, "leaky"), (64, 192, 96, None), (256, 256, 256, "residual"),
                                                (128, 64, 256, "reglu")])
def test_conv1x1_concat_read_in_place(c1, c2, oc, epilogue):
    """Concat -> 1x1 conv with the concat never materialised (the conv streams
    its K panels from both tensors): parity with the oracle."""
    rng = np.random.default_rng(23)
    h, w = 23, 40
    gb = GraphBuilder()
    a = gb.input("a", [1, c1, h, w])
    b = gb.input("b", [1, c2, h, w])
    wt = gb.weight("w", (rng.standard_normal((oc, c1 + c2, 1, 1), dtype=np.float32) *
                         np.sqrt(1.0 / (c1 + c2))).astype(np.float16))
    y = gb.conv(gb.concat([a, b], 1), wt, gb.weight("bias", rng.uniform(-0.1, 0.1, oc).astype(np.float16)))
    inputs = [rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16) for c in (c1, c2)]
    if epilogue == "leaky":
        y = gb.leaky_relu(y, 0.01)
    elif epilogue == "residual":
        y = gb.add(y, gb.input("r", [1, oc, h, w]))
        inputs.append(rng.standard_normal((1, oc, h, w), dtype=np.float32).astype(np.float16))
    elif epilogue == "reglu":  # node order of the exported ReGLU tail: slice, slice, clip, mul
        gate, lin = gb.slice(y, 1, 0, oc // 2), gb.slice(y, 1, oc // 2, oc)
        y = gb.mul(gb.clip(gate, 0.0, 1.0), lin)
    gb.output(y, "y")
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    kernels = [s["kernel"] for s in be.steps() if s["kernel"] != "mlvc_boundary_f16"]
    assert kernels == ["mlvc_conv1x1_tc"], kernels


@pytest.mark.parametrize("first,second", [((256, 128, 256), None), (None, (192, 64, 128)), ((128, 0, 64), (128, 64, 128))])
def test_conv1x1_concat_of_channel_slices_read_in_place(first, second):
    """Concat operands that are channel slices of wider tensors (each slice's
    only reader being the concat) are read in place too: the conv's A map
    starts at the slice's first channel and steps by the wider tensor's row.
    first / second: (channels of the wider tensor, slice start, slice end), or
    None for a plain tensor of 128 channels."""
    rng = np.random.default_rng(29)
    h, w = 17, 30
    gb = GraphBuilder()
    inputs = []

    def operand(spec, name):
        if spec is None:
            inputs.append(rng.standard_normal((1, 128, h, w), dtype=np.float32).astype(np.float16))
            return gb.input(name, [1, 128, h, w]), 128
        c, lo, hi = spec
        wide = gb.input(name, [1, c, h, w])
        inputs.append(rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16))
        # the wider tensor is produced on the device (a LeakyReLU), as in the decoder graphs
        return gb.slice(gb.leaky_relu(wide, 0.1), 1, lo, hi), hi - lo

    a, c1 = operand(first, "a")
    b, c2 = operand(second, "b")
    wt = gb.weight("w", (rng.standard_normal((128, c1 + c2, 1, 1), dtype=np.float32) *
                         np.sqrt(1.0 / (c1 + c2))).astype(np.float16))
    gb.output(gb.conv(gb.concat([a, b], 1), wt, gb.weight("bias", rng.uniform(-0.1, 0.1, 128).astype(np.float16))), "y")
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    kernels = [s["kernel"] for s in be.steps() if s["kernel"] not in ("mlvc_boundary_f16", "mlvc_unary_f16")]
    assert kernels == ["mlvc_conv1x1_tc"], kernels


@pytest.mark.parametrize("c,h,w", [(64, 6, 10), (32, 4, 14), (24, 4, 6)])
def test_pixel_shuffle_mid_graph(c, h, w):
    """Pixel shuffle / unshuffle between two other operators (not folded into
    the NCHW <-> NHWC boundary): 16-byte vector kernels for r = 2 when the
    8-channel blocks allow (c % 32 for the shuffle, c % 8 for the unshuffle),
    element kernels otherwise; CRD order bit-exact against the oracle."""
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    one = gb.weight("one", np.ones((1, 1, 1, 1), np.float16))
    shuffled = gb.depth_to_space(gb.mul(x, one), 2)
    gb.output(gb.mul(shuffled, one), "shuffled")
    unshuffled = gb.space_to_depth(gb.mul(x, one), 2)
    gb.output(gb.mul(unshuffled, one), "unshuffled")
    inputs = [np.arange(c * h * w, dtype=np.float32).reshape(1, c, h, w).astype(np.float16)]
    got, want, be = run_both(gb, inputs)
    bits_equal(got[0], want[0])
    bits_equal(got[1], want[1])
    kernels = {s["kernel"] for s in be.steps()}
    assert ("mlvc_depth_to_space_r2_v8_f16" in kernels) == (c % 32 == 0), kernels
    assert ("mlvc_space_to_depth_r2_v8_f16" in kernels) == (c % 8 == 0), kernels


@pytest.mark.parametrize("c,h,w,ic,epilogue", [(64, 6, 10, 64, None), (128, 9, 120, 256, "leaky"),
                                               (64, 5, 240, 128, None), (256, 4, 130, 256, "leaky"),
                                               (128, 3, 17, 64, "leaky")])
def test_conv1x1_pixel_shuffle_folded(c, h, w, ic, epilogue, monkeypatch):
    """1x1 conv (4c outputs, + LeakyReLU) -> DepthToSpace(2): the shuffle is
    folded into the conv's store (row-aligned tiles, weights in sub-pixel
    order, 5-D output view), so the 4c-channel tensor is never written.
    Widths below, at and above the 128-pixel tile (partial last tiles of a
    row).  Against the oracle, and bit-identical to the two-step plan."""
    x = lcg_fast(ic * h * w, 11).reshape(1, ic, h, w)
    wt = lcg_fast(4 * c * ic, 12).reshape(4 * c, ic, 1, 1)
    b = lcg_fast(4 * c, 13)
    gb = GraphBuilder()
    xi = gb.input("x", [1, ic, h, w])
    y = gb.conv(xi, gb.weight("w", wt), gb.weight("b", b))
    if epilogue == "leaky":
        y = gb.leaky_relu(y, 0.01)
    one = gb.weight("one", np.ones((1, 1, 1, 1), np.float16))
    gb.output(gb.mul(gb.depth_to_space(y, 2), one), "y")
    got, want, be = run_both(gb, [x])
    compare(got[0], want[0])
    kernels = [s["kernel"] for s in be.steps()]
    assert "mlvc_depth_to_space_r2_v8_f16" not in kernels and "mlvc_conv1x1_tc" in kernels, kernels
    monkeypatch.setenv("MLVC_B200_D2S_FUSION", "0")
    got2, _, be2 = run_both(gb, [x])
    assert "mlvc_depth_to_space_r2_v8_f16" in [s["kernel"] for s in be2.steps()]
    bits_equal(got[0], got2[0])


def test_reglu_standalone():
    gb = GraphBuilder()
    x = gb.input("x", [1, 48, 5, 7])
    g = gb.slice(x, 1, 0, 24)
    lin = gb.slice(x, 1, 24, 48)
    gb.output(gb.mul(gb.clip(g, 0.0, 1.0), lin), "y")
    got, want, be = run_both(gb, [_rand((1, 48, 5, 7), 6)])
    bits_equal(got[0], want[0])
    assert "mlvc_reglu_f16" in {s["kernel"] for s in be.steps()}


def test_state_binding_and_slots():
    """State binding (reference backend.hpp:34-46): output `feature` feeds input
    `ref` of the next run; reset_state zeroes it.  The slot path must give the
    same numbers as run()."""
    rng = np.random.default_rng(8)
    gb = GraphBuilder()
    x = gb.input("x", [1, 64, 6, 10])
    ref = gb.input("ref", [1, 64, 6, 10])
    w = gb.weight("w", (rng.standard_normal((64, 64, 1, 1), dtype=np.float32) * 0.1).astype(np.float16))
    feat = gb.add(gb.conv(x, w), ref)
    gb.output(gb.leaky_relu(feat, 0.1), "y")
    gb.output(feat, "feature")
    graph, weights = gb.finish()
    be = Backend(0)
    be.load_memory(graph, weights, [(1, 1)])
    with pytest.raises(RuntimeError, match="reset_state"):
        be.run([_rand((1, 64, 6, 10), 1)])
    be.reset_state()
    oracle = GraphOracle(graph, weights)
    state = np.zeros((1, 64, 6, 10), np.float16)
    frames = [_rand((1, 64, 6, 10), 10 + i) for i in range(3)]
    outs = []
    for f in frames:
        (y,) = be.run([f])
        want_y, want_feat = oracle.run([f, state])
        compare(y, want_y)
        state = want_feat
        outs.append(y)
    be.reset_state()
    be.configure_slots(2)
    for i, f in enumerate(frames):
        slot = i % 2
        be.slot_input(slot, 0)[...] = f
        be.submit(slot)
        be.wait_slot(slot)
        bits_equal(be.slot_output(slot, 0), outs[i])


def test_state_output_written_in_place():
    """When every read of the state input precedes the step that writes the
    bound output, the output is written straight into the state buffer (no
    copy step; the reference requires the state to alias the final node's
    output): frames still chain through the state exactly as with a copy."""
    rng = np.random.default_rng(12)
    gb = GraphBuilder()
    x = gb.input("x", [1, 64, 6, 10])
    ref = gb.input("ref", [1, 64, 6, 10])
    w1 = gb.weight("w1", (rng.standard_normal((64, 64, 1, 1), dtype=np.float32) * 0.1).astype(np.float16))
    w2 = gb.weight("w2", (rng.standard_normal((64, 64, 1, 1), dtype=np.float32) * 0.1).astype(np.float16))
    y = gb.leaky_relu(gb.add(gb.conv(x, w1), ref), 0.1)  # last read of the state
    feat = gb.conv(y, w2)                                # written after it
    gb.output(y, "y")
    gb.output(feat, "feature")
    graph, weights = gb.finish()
    be = Backend(0)
    be.load_memory(graph, weights, [(1, 1)])
    assert "state-copy" not in {s["kernel"] for s in be.steps()}
    be.reset_state()
    oracle = GraphOracle(graph, weights)
    state = np.zeros((1, 64, 6, 10), np.float16)
    frames = [_rand((1, 64, 6, 10), 20 + i) for i in range(3)]
    outs = []
    for f in frames:
        (got,) = be.run([f])
        want_y, want_feat = oracle.run([f, state])
        compare(got, want_y)
        state = want_feat
        outs.append(got)
    be.reset_state()
    be.configure_slots(2)
    for i, f in enumerate(frames):
        be.slot_input(i % 2, 0)[...] = f
        be.submit(i % 2)
        be.wait_slot(i % 2)
        bits_equal(be.slot_output(i % 2, 0), outs[i])


def test_slot_pipeline_overlapped_frames():
    """Two slots in flight (host->device of one frame, the schedule of the
    previous one and its device->host copy overlap on separate streams):
    frames still run in submission order, the recurrent state passes from
    frame to frame, and every slot returns the bits run() gives."""
    rng = np.random.default_rng(9)
    gb = GraphBuilder()
    x = gb.input("x", [1, 32, 64, 96])
    ref = gb.input("ref", [1, 64, 32, 48])
    w = gb.weight("w", (rng.standard_normal((64, 128, 1, 1), dtype=np.float32) * 0.1).astype(np.float16))
    feat = gb.add(gb.conv(gb.space_to_depth(x, 2), w), ref)
    gb.output(gb.depth_to_space(gb.leaky_relu(feat, 0.1), 2), "y")
    gb.output(feat, "feature")
    graph, weights = gb.finish()
    be = Backend(0)
    be.load_memory(graph, weights, [(1, 1)])
    frames = [_rand((1, 32, 64, 96), 20 + i) for i in range(7)]
    be.reset_state()
    want = [be.run([f])[0].copy() for f in frames]
    be.reset_state()
    be.configure_slots(2)
    got = [None] * len(frames)
    for i, f in enumerate(frames):
        slot = i % 2
        if i >= 2:
            be.wait_slot(slot)
            got[i - 2] = be.slot_output(slot, 0).copy()
        be.slot_input(slot, 0)[...] = f
        be.submit(slot)
    for i in range(len(frames) - 2, len(frames)):
        be.wait_slot(i % 2)
        got[i] = be.slot_output(i % 2, 0).copy()
    for g, w_ in zip(got, want):
        bits_equal(g, w_)


def test_rejects_bad_input_shape():
    gb = GraphBuilder()
    x = gb.input("x", [1, 8, 4, 4])
    gb.output(gb.leaky_relu(x), "y")
    graph, weights = gb.finish()
    be = Backend(0)
    be.load_memory(graph, weights)
    with pytest.raises(RuntimeError, match="shape"):
        be.run([np.zeros((1, 8, 4, 5), np.float16)])


@pytest.mark.parametrize("c,h,w,decoder", [(64, 23, 40, False), (128, 46, 80, True), (16, 7, 9, False)])
def test_feature_update_fused(c, h, w, decoder, monkeypatch):
    """Recurrent-feature update as one kernel (reference
    recurrent_feature.cu:5-107): parity with the oracle (sigmoid within its
    tolerance), and bit-identical to the same graph run operator by operator."""
    from feature_graphs import feature_update_graph
    gb, inputs = feature_update_graph(c, h, w, decoder)
    got, want, be = run_both(gb, inputs)
    for g, wnt in zip(got, want):
        compare(g, wnt)
    assert "mlvc_feature_update_f16" in {s["kernel"] for s in be.steps()}
    graph, weights = gb.finish()
    monkeypatch.setenv("MLVC_B200_TAIL_FUSION", "0")
    split = Backend(0)
    split.load_memory(graph, weights)
    assert "mlvc_feature_update_f16" not in {s["kernel"] for s in split.steps()}
    for g, s in zip(got, split.run(inputs)):
        bits_equal(s, g)


@pytest.mark.parametrize("q,h,w", [(64, 23, 40), (16, 5, 7), (128, 12, 20)])
def test_quantisation_tails_fused(q, h, w, monkeypatch):
    """y0 and y1 quantisation tails as one kernel each (reference
    quantization_tail.cu): every output bit-identical to the oracle and to the
    operator-by-operator schedule (all operators are elementwise)."""
    from quant_graphs import quant_tails_graph
    gb, inputs = quant_tails_graph(q, h, w)
    got, want, be = run_both(gb, inputs)
    for g, wnt in zip(got, want):
        bits_equal(g, wnt)
    kernels = {s["kernel"] for s in be.steps()}
    assert {"mlvc_y0_tail_f16", "mlvc_y1_tail_f16"} <= kernels, kernels
    graph, weights = gb.finish()
    monkeypatch.setenv("MLVC_B200_TAIL_FUSION", "0")
    split = Backend(0)
    split.load_memory(graph, weights)
    for g, s in zip(got, split.run(inputs)):
        bits_equal(s, g)


def test_slice_views_keep_their_source_alive():
    """Contiguous slices are views into their source's buffer (no copy step).
    The source stays allocated until the view's last reader: the convs
    planned between the slice and its reader must not reuse its memory."""
    from mlvc_b200.graph import kaiming_normal, small_bias
    rng = np.random.default_rng(31)
    gb = GraphBuilder()
    x = gb.input("x", [1, 64, 16, 24])

    def conv(v, cin, cout, name):
        return gb.conv(v, gb.weight(name + ".w", kaiming_normal(rng, (cout, cin, 1, 1), 1.0)),
                       gb.weight(name + ".b", small_bias(rng, cout)))

    t = conv(x, 64, 64, "c1")
    s = gb.slice(t, 2, 4, 12)                  # rows 4..11 of t: a view at 12,288 bytes
    u = gb.leaky_relu(conv(x, 64, 128, "c2"), 0.1)
    u = conv(conv(u, 128, 64, "c3"), 64, 64, "c4")
    y = gb.add(gb.slice(u, 2, 4, 12), s)      # both operands are views
    gb.output(conv(y, 64, 64, "c5"), "y")
    inputs = [rng.standard_normal((1, 64, 16, 24), dtype=np.float32).astype(np.float16)]
    got, want, be = run_both(gb, inputs)
    compare(got[0], want[0])
    assert not [s_ for s_ in be.steps() if s_["kernel"].startswith("mlvc_strided_copy")], be.steps()
    # the views are readable like any materialised tensor
    graph, weights = gb.finish()
    dbg = Backend(0, debug_tensors=True)
    dbg.load_memory(graph, weights)
    dbg.run(inputs)
    from helpers import per_op_parity
    assert per_op_parity(dbg, graph, weights, inputs) >= 6
