"""Graphs compiled by the reference's own AOT compiler (tests/golden/) run on
the B200 through the C ABI and match the reference CPU backend's outputs
(per-op contract, FP16-magnitude-scaled max-abs 2e-2 and rel-L2 1e-3), and
every materialised intermediate matches the oracle on the GPU's own inputs.

The tail cases (recurrent-feature update in its encoder and decoder forms,
y0 / y1 latent quantisation tails) are the chains the reference fuses; they
run as the fused tail kernels here.  Their integer-valued and reciprocal
arithmetic (y_raw_0 / y_raw_1 and every other quantisation-tail output) must
equal the reference CPU backend bit for bit, fused and operator by operator;
outputs that pass through a Sigmoid are held to the per-op tolerance, since
CUDA's expf and the host libm's may differ by one FP32 ulp."""

from pathlib import Path

import numpy as np
import pytest

from helpers import bits_equal, compare_scaled, per_op_parity
from mlvc_b200 import Backend

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


TAIL_KERNELS = {"feature_update_enc": {"mlvc_feature_update_f16"},
                "feature_update_dec": {"mlvc_feature_update_f16"},
                "quant_tails": {"mlvc_y0_tail_f16", "mlvc_y1_tail_f16"}}


@pytest.mark.parametrize("case", ["example_q", "block_stack_tiny", "spatial_convs", "feature_update_enc",
                                  "feature_update_dec", "quant_tails"])
def test_reference_compiled_graph(case):
    d = np.load(GOLDEN / case / "inputs.npz")
    inputs = [d[k] for k in sorted(d.files)]
    e = np.load(GOLDEN / case / "expected.npz")
    be = Backend(0, debug_tensors=True)
    be.load(GOLDEN / case, "model")
    outs = be.run(inputs)
    if case in TAIL_KERNELS:
        assert TAIL_KERNELS[case] <= {s["kernel"] for s in be.steps()}
    for i, o in enumerate(outs):
        refs = [e[f"ref_cpu_scalar_{i}"]]
        if f"ref_cpu_scalar_unfused_{i}" in e.files:
            refs.append(e[f"ref_cpu_scalar_unfused_{i}"])
        for ref in refs:
            if case == "quant_tails":
                bits_equal(o, ref)
            else:
                compare_scaled(o, ref)
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
    # an index outside the 4-row table is an error, as in the reference CPU
    # backend ("cpu: GATHER index out of range"), and the backend stays usable
    for q in (4, -5):
        with pytest.raises(RuntimeError, match="GATHER index out of range"):
            be.run([x, ref, np.array([q], np.int32)])
    ins = [x, ref, np.array([1], np.int32)]
    for got, want in zip(be.run(ins), oracle.run(ins)):
        compare_scaled(got, want)
