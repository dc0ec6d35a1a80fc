"""Graph builder for the latent quantisation tails (y0 then y1), in the node
order the reference's matchers expect (backends/driver_cubin/src/
fusion_registry.cpp:14-404).  Shared by the CPU planner tests and the GPU
parity tests."""

import numpy as np

from mlvc_b200.graph import GraphBuilder


def quant_tails_graph(q, h, w, seed=51):
    rng = np.random.default_rng(seed)
    gb = GraphBuilder()
    names = {}

    def inp(name, ch, kind):
        names[name] = gb.input(name, [1, ch, h, w])
        if kind == "prior":
            v = rng.uniform(-0.2, 2.0, (1, ch, h, w))
        elif kind == "latent":
            v = rng.standard_normal((1, ch, h, w)) * 3.0
        else:  # scales
            v = rng.uniform(0.25, 2.0, (1, ch, h, w))
        return v.astype(np.float16)

    values = [inp("prior", 4 * q, "prior"), inp("latent", 2 * q, "latent"), inp("qs0", 2 * q, "scale"),
              inp("us00", q, "scale"), inp("us01", q, "scale"), inp("prior2", 2 * q, "latent"),
              inp("qs1", 2 * q, "scale"), inp("us10", q, "scale"), inp("us11", q, "scale")]
    n = names
    # y0 tail (19 operators)
    s0 = gb.slice(n["prior"], 1, 0, 2 * q)
    s1 = gb.slice(n["prior"], 1, 2 * q, 4 * q)
    clipped = gb.clip(s0, 0.11)
    rec = gb.unary("Reciprocal", clipped)
    norm = gb.mul(n["latent"], rec)
    diff = gb.sub(norm, s1)
    scaled = gb.mul(diff, n["qs0"])
    a0 = gb.slice(scaled, 1, 0, q)
    a1 = gb.slice(scaled, 1, q, 2 * q)
    y0 = gb.unary("Round", gb.add(a0, a1))
    p0 = gb.slice(s1, 1, 0, q)
    p1 = gb.slice(s1, 1, q, 2 * q)
    u0 = gb.mul(gb.add(y0, p0), n["us00"])
    u1 = gb.mul(gb.add(y0, p1), n["us01"])
    c2 = gb.concat([u0, u1], 1)
    c3 = gb.concat([c2, n["prior"]], 1)
    # y1 tail (15 operators)
    sc = gb.mul(gb.sub(norm, n["prior2"]), n["qs1"])
    b0 = gb.slice(sc, 1, 0, q)
    b1 = gb.slice(sc, 1, q, 2 * q)
    y1 = gb.unary("Round", gb.add(b0, b1))
    q0 = gb.slice(n["prior2"], 1, 0, q)
    q1 = gb.slice(n["prior2"], 1, q, 2 * q)
    v0 = gb.mul(gb.add(y1, q0), n["us10"])
    v1 = gb.mul(gb.add(y1, q1), n["us11"])
    c4 = gb.concat([v0, v1], 1)
    result = gb.mul(gb.add(c2, c4), clipped)
    gb.output(y0, "y_raw_0")
    gb.output(y1, "y_raw_1")
    gb.output(result, "decoder_input")
    gb.output(c3, "prior_concat")
    return gb, values
