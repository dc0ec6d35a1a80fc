"""Workload-level parity on the B200 (configs 1 and 2 of the benchmark).

Each materialised step is checked against the oracle applied to the GPU's own
step inputs (per-op contract: max-abs 2e-2 scaled by FP16 magnitude, rel-L2
1e-3); the final output is checked against an independent oracle run with the
reference's whole-tensor conformance bound (max-abs 0.25, scaled, rel-L2 1e-3).
At full size the oracle's convolutions use the FP32 GEMM form (same operator,
FP32 accumulation, different summation order).
"""

import numpy as np
import pytest

from helpers import STACK_MAX_ABS, compare_scaled, per_op_parity
from mlvc_b200 import Backend
from mlvc_b200.graph import build_block_stack, build_conv3x3
from oracle.graph_oracle import GraphOracle

pytestmark = pytest.mark.gpu


def _load(gb):
    graph, weights = gb.finish()
    be = Backend(0, debug_tensors=True)
    be.load_memory(graph, weights)
    return be, graph, weights


@pytest.mark.parametrize("channels,h,w,blocks", [(32, 8, 12, 2), (64, 24, 40, 2), (128, 23, 40, 3)])
def test_block_stack_small(channels, h, w, blocks):
    gb, inputs = build_block_stack(seed=3, channels=channels, height=h, width=w, blocks=blocks)
    be, graph, weights = _load(gb)
    (y,) = be.run(inputs)
    assert per_op_parity(be, graph, weights, inputs) >= 4 * blocks
    (want,) = GraphOracle(graph, weights).run(inputs)
    compare_scaled(y, want, max_abs=STACK_MAX_ABS)


def test_block_stack_config2_full():
    """Config 2 at full size: 8 blocks, C=128 @ 92x160, [1,32,184,320] input."""
    gb, inputs = build_block_stack(seed=0)
    be, graph, weights = _load(gb)
    (y,) = be.run(inputs)
    kernels = [s["kernel"] for s in be.steps()]
    assert kernels.count("mlvc_conv1x1_tc") == 32 and kernels.count("mlvc_depthwise_v8_f16") == 8, kernels
    assert per_op_parity(be, graph, weights, inputs, conv_impl="gemm") >= 40
    (want,) = GraphOracle(graph, weights, "gemm").run(inputs)
    compare_scaled(y, want, max_abs=STACK_MAX_ABS)
    # run-to-run determinism of the captured graph
    (y2,) = be.run(inputs)
    assert np.array_equal(y.view(np.uint16), y2.view(np.uint16))


def test_conv3x3_config1_per_op():
    gb, inputs = build_conv3x3(0)
    be, graph, weights = _load(gb)
    (y,) = be.run(inputs)
    (want,) = GraphOracle(graph, weights, "gemm").run(inputs)
    compare_scaled(y, want)
