"""Workload-level parity on the B200 (configs 1 and 2 of the benchmark).

Each materialised step is checked against the oracle applied to the GPU's own
step inputs (per-op contract: max-abs 2e-2 scaled by FP16 magnitude, rel-L2
1e-3).  That is the hard criterion.

The whole-stack output is then compared with the reference's own CPU backend
(oracle/_ref, compiled from the reference sources).  The 8-block FP16 stack
amplifies summation-order rounding differences: two CPU implementations of
the same graph (the reference's AVX2 kernels and the oracle's FP32 GEMM form)
already differ by ~6% relative L2 at the output of config 2, and by ~8e-4 for
a 3-block stack.  The GPU is therefore required to stay within 2x of that
CPU-vs-CPU spread (or within 1e-3), measured on the same inputs.
"""

import numpy as np
import pytest

from helpers import bits_equal, compare_scaled, per_op_parity
from mlvc_b200 import Backend
from mlvc_b200.graph import build_block_stack, build_conv3x3, build_mlvc_decoder_standin
from oracle.graph_oracle import GraphOracle
from oracle.ref_backend import RefCpuBackend

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def _stack_check(y, graph, weights, inputs, tmp_path):
    """Every graph output (y: one array or a list) against the reference CPU
    backend, within twice the spread between the two CPU implementations (the
    reference backend and the oracle) or rel-L2 1e-3, whichever is larger."""
    ys = y if isinstance(y, (list, tuple)) else [y]
    part = tmp_path / "aot" / "m"
    part.mkdir(parents=True)
    (part / "graph.pb").write_bytes(graph)
    (part / "weights.bin").write_bytes(weights)
    refs = RefCpuBackend(tmp_path, "m", 0).run(inputs)
    alts = GraphOracle(graph, weights, "gemm").run(inputs)
    assert len(refs) == len(ys) == len(alts)
    for k, (yk, ref, alt) in enumerate(zip(ys, refs, alts)):
        spread = _rel(alt, ref)
        got = _rel(yk, ref)
        assert np.isfinite(yk.astype(np.float32)).all()
        assert got <= max(1e-3, 2.0 * spread), \
            f"output {k}: GPU vs reference CPU rel-L2 {got:.3g}, CPU-vs-CPU spread {spread:.3g}"


def _load(gb):
    graph, weights = gb.finish()
    be = Backend(0, debug_tensors=True)
    be.load_memory(graph, weights)
    return be, graph, weights


@pytest.mark.parametrize("channels,h,w,blocks", [(32, 8, 12, 2), (64, 24, 40, 2), (128, 23, 40, 3)])
def test_block_stack_small(channels, h, w, blocks, tmp_path):
    gb, inputs = build_block_stack(seed=3, channels=channels, height=h, width=w, blocks=blocks)
    be, graph, weights = _load(gb)
    (y,) = be.run(inputs)
    assert per_op_parity(be, graph, weights, inputs) >= 2 * blocks
    _stack_check(y, graph, weights, inputs, tmp_path)


def test_block_stack_config2_full(tmp_path):
    """Config 2 at full size: 8 blocks, C=128 @ 92x160, [1,32,184,320] input."""
    gb, inputs = build_block_stack(seed=0)
    be, graph, weights = _load(gb)
    (y,) = be.run(inputs)
    kernels = [s["kernel"] for s in be.steps()]
    assert kernels.count("mlvc_mbconv_tc") == 8 and kernels.count("mlvc_ffn_tc") == 8, kernels
    assert per_op_parity(be, graph, weights, inputs, conv_impl="gemm") >= 16
    _stack_check(y, graph, weights, inputs, tmp_path)
    # run-to-run determinism of the captured graph
    (y2,) = be.run(inputs)
    assert np.array_equal(y.view(np.uint16), y2.view(np.uint16))


@pytest.mark.parametrize("width,height", [(256, 128), (640, 368), (1920, 1088)])
def test_mlvc_decoder_standin(width, height, tmp_path):
    """The MLVC-shaped decoder stand-in (256-channel blocks on the unfused
    tensor-core path, pixel shuffle x2 / x8, spatial crops, channel concats,
    QP-indexed Gather): every materialised step against the oracle, then the
    whole graph against the reference CPU backend.  1920x1088 is the
    benchmark's configuration: 510-tile 1x1 convs and the
    512-channel fused depthwise + projection at 136 x 240."""
    gb, inputs = build_mlvc_decoder_standin(seed=5, width=width, height=height)
    be, graph, weights = _load(gb)
    x_hat, feature = be.run(inputs)
    assert x_hat.shape == (1, 3, height, width) and feature.shape == (1, 256, height // 8, width // 8)
    assert per_op_parity(be, graph, weights, inputs, conv_impl="gemm") >= 30
    _stack_check([x_hat, feature], graph, weights, inputs, tmp_path)


@pytest.mark.parametrize("width,height", [(256, 128), (640, 368)])
def test_mlvcs_decoder_standin(width, height, tmp_path):
    """The MLVC-S-shaped stand-in (96 / 192-channel blocks, 48-channel
    latents, x4 mini-hyperprior up-sampling): every materialised step against
    the oracle, then the whole graph against the reference CPU backend."""
    from mlvc_b200.graph import build_mlvcs_decoder_standin
    gb, inputs = build_mlvcs_decoder_standin(seed=5, width=width, height=height)
    be, graph, weights = _load(gb)
    x_hat, feature = be.run(inputs)
    assert x_hat.shape == (1, 3, height, width) and feature.shape == (1, 96, height // 8, width // 8)
    assert per_op_parity(be, graph, weights, inputs, conv_impl="gemm") >= 40
    _stack_check([x_hat, feature], graph, weights, inputs, tmp_path)


def test_conv3x3_config1_per_op():
    gb, inputs = build_conv3x3(0)
    be, graph, weights = _load(gb)
    (y,) = be.run(inputs)
    (want,) = GraphOracle(graph, weights, "gemm").run(inputs)
    compare_scaled(y, want)


@pytest.mark.parametrize("width,height", [(256, 128), (640, 368), (1920, 1088)])
def test_mlvc_encoder_standin(width, height, tmp_path):
    """The MLVC-shaped encoder stand-in (strided 3x3 analysis convs, the y0 /
    y1 quantisation tails and the encoder-form feature update as fused
    kernels): every materialised step against the oracle on the GPU's own
    step inputs -- integer-valued z_raw / y_raw_0 / y_raw_1 exactly, since
    Round outputs pass the per-op check only when equal.  That is the exact
    criterion.  The whole graph is then compared with the reference CPU
    backend as a sanity check with explicit bounds: a symbol differs only
    where an upstream FP16 rounding difference crosses a rounding boundary,
    and one z_raw symbol that flips changes the prior of every y symbol below
    it, so whole-graph differences come in cascades.  Measured between two
    CPU implementations (the reference backend and the oracle's GEMM form)
    on these graphs: up to 2.4 % of the y symbols and a feature rel-L2 up to
    4.7e-2; the GPU against the reference lies in the same range (up to 3.4 %
    and 7.5e-2 at 640x368 with seed 4, where two z symbols flip).  Bounds: at
    most 0.3 % of z_raw symbols differ (2 of 1920 measured), by 1; at most 6 %
    of y symbols; the
    feature within 0.15 rel-L2.  A P-frame: the reference feature is a
    previous feature (not zero)."""
    from mlvc_b200.graph import build_mlvc_encoder_standin
    gb, inputs = build_mlvc_encoder_standin(seed=4, width=width, height=height)
    inputs[1] = (inputs[1].astype(np.float32) * 0.15).astype(np.float16)
    be, graph, weights = _load(gb)
    outs = be.run(inputs)
    kernels = {s["kernel"] for s in be.steps()}
    assert {"mlvc_y0_tail_f16", "mlvc_y1_tail_f16", "mlvc_feature_update_f16", "mlvc_convkxk_tc"} <= kernels
    assert [o.shape for o in outs] == [(1, 256, height // 8, width // 8), (1, 128, -(-height // 128), -(-width // 128)),
                                       (1, 64, height // 16, width // 16), (1, 64, height // 16, width // 16)]
    for o in outs[1:]:
        assert np.array_equal(o, np.rint(o)), "latents must be integer-valued"
    assert per_op_parity(be, graph, weights, inputs, conv_impl="gemm") >= 40
    part = tmp_path / "aot" / "m"
    part.mkdir(parents=True)
    (part / "graph.pb").write_bytes(graph)
    (part / "weights.bin").write_bytes(weights)
    refs = RefCpuBackend(tmp_path, "m", 0).run(inputs)
    z, zr = outs[1].astype(np.float64), refs[1].astype(np.float64)
    assert (z != zr).mean() <= 3e-3 and np.abs(z - zr).max() <= 1, (int((z != zr).sum()), z.size)
    for k in (2, 3):
        y, yr = outs[k].astype(np.float64), refs[k].astype(np.float64)
        assert (y != yr).mean() <= 0.06, (k, int((y != yr).sum()), y.size)
    assert _rel(outs[0], refs[0]) <= 0.15


def test_mlvc_encoder_slot_path_with_yuv_input(tmp_path):
    """Encoder through the slot API with the codec's YUV420 input conversion
    and submit(slot, shifted_q) (the reference's encoder_input_yuv /
    submit_encoder / encoder_outputs, cuda_graph_executor.cpp:243-312): the
    outputs equal run() on the tensor the reference's prepare_model_input
    makes from the same frame, frame after frame with the state carried."""
    from mlvc_b200.graph import build_mlvc_encoder_standin, synthetic_yuv420
    from oracle.ref_backend import ref_yuv_to_tensor
    W, H, MW, MH = 256, 120, 256, 128
    gb, inputs = build_mlvc_encoder_standin(seed=6, width=MW, height=MH)
    graph, weights = gb.finish()
    slots, plain = Backend(0), Backend(0)
    for b in (slots, plain):
        b.load_memory(graph, weights, [(1, 0)])
        b.reset_state()
    slots.configure_codec_io(W, H, MW, MH, 1.0, slots=2, input_index=0)
    for frame, q in enumerate((21, 21, 0, 51)):
        slot = frame % 2
        y, u, v = synthetic_yuv420(frame, W, H)
        py, pu, pv = slots.slot_input_yuv(slot)
        py[...], pu[...], pv[...] = y, u, v
        slots.submit(slot, shifted_q=q)
        slots.wait_slot(slot)
        x, _ = ref_yuv_to_tensor(np.concatenate([y.reshape(-1), u.reshape(-1), v.reshape(-1)]), W, H, MW, MH)
        want = plain.run([x, np.array([q], np.int32)])
        for k, w in enumerate(want):
            bits_equal(slots.slot_output(slot, k), w)
