"""Graphs compiled by the reference's own AOT compiler (tests/golden/) run on
the B200 through the C ABI and match the reference CPU backend's outputs
(per-op contract, FP16-magnitude-scaled max-abs 2e-2 and rel-L2 1e-3), and
every materialised intermediate matches the oracle on the GPU's own inputs."""

from pathlib import Path

import numpy as np
import pytest

from helpers import compare_scaled, per_op_parity
from mlvc_b200 import Backend

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("case", ["example_q", "block_stack_tiny", "spatial_convs"])
def test_reference_compiled_graph(case):
    d = np.load(GOLDEN / case / "inputs.npz")
    inputs = [d[k] for k in sorted(d.files)]
    e = np.load(GOLDEN / case / "expected.npz")
    be = Backend(0, debug_tensors=True)
    be.load(GOLDEN / case, "model")
    outs = be.run(inputs)
    for i, o in enumerate(outs):
        compare_scaled(o, e[f"ref_cpu_scalar_{i}"])
    part = GOLDEN / case / "aot" / "model"
    per_op_parity(be, (part / "graph.pb").read_bytes(), (part / "weights.bin").read_bytes(), inputs)


def test_example_q_all_qp_rows():
    """The per-QP Gather row follows the int32 q input (reference aot_tests: QPs 0, 1, 3)."""
    from oracle.graph_oracle import GraphOracle
    d = np.load(GOLDEN / "example_q" / "inputs.npz")
    x, ref, _ = [d[k] for k in sorted(d.files)]
    be = Backend(0)
    be.load(GOLDEN / "example_q", "model")
    oracle = GraphOracle.from_dir(GOLDEN / "example_q", "model")
    for q in (0, 1, 3, -1):
        ins = [x, ref, np.array([q], np.int32)]
        for got, want in zip(be.run(ins), oracle.run(ins)):
            compare_scaled(got, want)
