"""Failure detection on the GPU without a fault: a bounded device wait that runs
out.  The 1x1 tensor-core conv is relaunched with its waits limited to 1 ms
and CTA 0's TMA producer withholding one activation panel (no copy issued, no
barrier armed), i.e. a flag that nothing sets.  A bounded wait stalled
behind it must expire, the CTA must wind down and the kernel return, the
host must read a wait bit (and nothing else), and the context must stay
usable: the same backend and a fresh one then reproduce the normal output
bit for bit."""

import numpy as np
import pytest

from helpers import bits_equal, conv_graph
from mlvc_b200 import Backend
from mlvc_b200.graph import kaiming_normal, small_bias

pytestmark = pytest.mark.gpu

# wait-timeout bits of csrc/kernels/conv_tc.cu: producer, MMA issuer, epilogue
ERR_WAIT_PRODUCER, ERR_WAIT_MMA, ERR_WAIT_EPILOGUE = 0x1, 0x2, 0x4


@pytest.mark.parametrize("epilogue", [None, "residual"])
def test_bounded_wait_expires_and_backend_recovers(epilogue):
    rng = np.random.default_rng(8)
    w = kaiming_normal(rng, (128, 64, 1, 1))
    b = small_bias(rng, 128)
    gb = conv_graph([1, 64, 32, 64], w, b, epilogue=epilogue)
    graph, weights = gb.finish()
    inputs = [rng.standard_normal((1, 64, 32, 64), dtype=np.float32).astype(np.float16)]
    if epilogue == "residual":
        inputs.append(rng.standard_normal((1, 128, 32, 64), dtype=np.float32).astype(np.float16))
    be = Backend(0)
    be.load_memory(graph, weights)
    (want,) = be.run(inputs)
    index = [s["kernel"] for s in be.steps()].index("mlvc_conv1x1_tc")

    # The withheld panel stalls the issuer directly and, behind it, the
    # epilogue (its accumulator never completes) and the producer (its slot is
    # never released): whichever role's 1 ms wait started first runs out and
    # aborts the CTA.  Only wait bits may be set.
    status = be.test_wait_expiry(index, 1_000_000)
    waits = ERR_WAIT_PRODUCER | ERR_WAIT_MMA | ERR_WAIT_EPILOGUE
    assert status != 0 and status & ~waits == 0, hex(status)

    (again,) = be.run(inputs)  # same backend, same context: normal 2 s limit restored
    bits_equal(again, want)
    fresh = Backend(0)
    fresh.load_memory(graph, weights)
    (third,) = fresh.run(inputs)
    bits_equal(third, want)
    fresh.close()
    be.close()


def test_wait_expiry_hook_rejects_other_steps():
    rng = np.random.default_rng(9)
    gb = conv_graph([1, 16, 8, 8], kaiming_normal(rng, (16, 1, 3, 3), 1.0), small_bias(rng, 16), pad=(1, 1),
                    groups=16)
    graph, weights = gb.finish()
    be = Backend(0)
    be.load_memory(graph, weights)
    be.run([rng.standard_normal((1, 16, 8, 8), dtype=np.float32).astype(np.float16)])
    for i, s in enumerate(be.steps()):
        assert s["kernel"] != "mlvc_conv1x1_tc"
        with pytest.raises(RuntimeError, match="mlvc_conv1x1_tc"):
            be.test_wait_expiry(i, 1_000_000)
    be.close()
