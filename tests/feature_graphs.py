"""Graph builders for the recurrent-feature update pattern (shared by the CPU
planner tests and the GPU parity tests).  Node order is the exported graph's
(reference matcher: backends/driver_cubin/src/fusion_registry.cpp:405-709)."""

import numpy as np

from mlvc_b200.graph import GraphBuilder


def feature_update_graph(c, h, w, decoder=False, seed=41):
    """encoder form: Concat(scaled, blended) right after the chain (the new
    feature); decoder form: scaled and blended also feed a conv, the concat
    comes later."""
    rng = np.random.default_rng(seed)
    gb = GraphBuilder()
    t = gb.input("t", [1, 3 * c, h, w])
    hist = gb.input("hist", [1, c, h, w])
    a = gb.slice(t, 1, 0, c)
    b = gb.slice(t, 1, c, 2 * c)
    cc = gb.slice(t, 1, 2 * c, 3 * c)
    sb = gb.unary("Sigmoid", b)
    sc = gb.unary("Sigmoid", cc)
    wb = gb.mul(sb, hist)
    ig = gb.sub(gb.weight("one", np.array([1.0], np.float16)), sb)
    wa = gb.mul(ig, a)
    blended = gb.add(wb, wa)
    gated = gb.mul(sc, blended)
    scale = gb.weight("scale", rng.uniform(0.5, 1.5, (1, c, 1, 1)).astype(np.float16))
    scaled = gb.mul(gated, scale)
    inputs = [rng.standard_normal((1, 3 * c, h, w), dtype=np.float32).astype(np.float16),
              rng.standard_normal((1, c, h, w), dtype=np.float32).astype(np.float16)]
    if decoder:
        wt = gb.weight("w", (rng.standard_normal((c, 2 * c, 1, 1), dtype=np.float32) * 0.1).astype(np.float16))
        recon = gb.conv(gb.concat([scaled, blended], 1), wt)
        gb.output(recon, "recon")
        gb.output(gb.leaky_relu(scaled, 0.1), "side")
        gb.output(gb.concat([scaled, blended], 1), "feature")
    else:
        gb.output(gb.concat([scaled, blended], 1), "feature")
    return gb, inputs
