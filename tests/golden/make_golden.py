"""Regenerates the golden fixtures in this directory (run in a checkout that has
the reference tree; the fixtures are committed, the tests never need it).

For each case the reference's own AOT compiler (tools/python/mlvc_tools/aot.py,
compile_module) traces a small FP16 PyTorch module into graph.pb + weights.bin,
then two reference implementations produce the expected outputs:
  * ref_cpu   - the reference's backends/cpu, compiled from its sources
                (oracle/_ref), scalar ISA (MLVC_CPU_ISA=scalar) and AVX2;
  * replay    - the reference's independent PyTorch replay of the graph
                (tests/unit/aot_tests.py:21-61, execute_graph), FP32 upcast.
The tail cases (feature_update_enc, feature_update_dec, quant_tails) hold
the operator chains the reference fuses into one kernel each (Sigmoid,
Reciprocal, Round; backends/cpu/src/fusion_matcher.cpp:413-850, kernels at
backends/cpu/src/kernels_scalar.cpp:324-537); they also record the reference
CPU backend with fusion disabled (MLVC_CPU_DISABLE_FUSION=1), i.e. operator
by operator.  The AVX2 sigmoid is an approximation, so the scalar ISA is the
bit-level reference for sigmoid-bearing cases.
Inputs are seeded; everything is stored in <case>.npz next to the bundle.

    python tests/golden/make_golden.py REFERENCE_TREE [CASE ...]
    MLVC_REFERENCE_DIR=REFERENCE_TREE python tests/golden/make_golden.py [CASE ...]
"""

import os
import subprocess
import sys
from collections import namedtuple
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
_ARGS = sys.argv[1:]
if _ARGS and Path(_ARGS[0]).is_dir():
    REF = Path(_ARGS.pop(0))
elif os.environ.get("MLVC_REFERENCE_DIR"):
    REF = Path(os.environ["MLVC_REFERENCE_DIR"])
else:
    sys.exit("usage: make_golden.py REFERENCE_TREE [CASE ...] (or set MLVC_REFERENCE_DIR)")
ONLY = set(_ARGS)
sys.path[:0] = [str(REF / "tools" / "python"), str(REF / "tests" / "unit"), str(ROOT)]

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402
from mlvc_tools.aot import compile_module  # noqa: E402

CASES = {}


def case(fn):
    CASES[fn.__name__] = fn
    return fn


class ExampleQ(torch.nn.Module):
    """Pixel unshuffle, 1x1 conv, per-QP gather, chunk, shuffle, clamp, concat,
    add and rsub: the operator mix of the reference's aot_tests Example."""
    InputType = namedtuple("Inputs", "x ref q")
    OutputType = namedtuple("Outputs", "reconstruction feature")

    def __init__(self):
        super().__init__()
        self.conv = torch.nn.Conv2d(12, 12, 1).half()
        self.scales = torch.nn.Parameter(torch.arange(1, 5, dtype=torch.float16).reshape(4, 1, 1, 1))

    def forward(self, x, ref, q):
        y = self.conv(F.pixel_unshuffle(x, 2)) * self.scales[q]
        a, b = y.chunk(2, 1)
        return self.OutputType(F.pixel_shuffle(y, 2).clamp_(0, 1), torch.cat((a + ref[:, :6], 1.0 - b), 1))


class Block(torch.nn.Module):
    def __init__(self, c):
        super().__init__()
        self.expand = torch.nn.Conv2d(c, 2 * c, 1)
        self.dw = torch.nn.Conv2d(2 * c, 2 * c, 3, padding=1, groups=2 * c)
        self.project = torch.nn.Conv2d(2 * c, c, 1)
        self.ffn_in = torch.nn.Conv2d(c, 4 * c, 1)
        self.ffn_out = torch.nn.Conv2d(2 * c, c, 1)

    def forward(self, x):
        t = F.leaky_relu(self.expand(x), 0.01)
        x = x + self.project(self.dw(t))
        g, lin = self.ffn_in(x).chunk(2, 1)
        return x + self.ffn_out(g.clamp(0, 1) * lin)


class Stack(torch.nn.Module):
    InputType = namedtuple("Inputs", "x")
    OutputType = namedtuple("Outputs", "y")

    def __init__(self, c, blocks):
        super().__init__()
        self.blocks = torch.nn.ModuleList(Block(c) for _ in range(blocks))

    def forward(self, x):
        h = F.pixel_unshuffle(x, 2)
        for b in self.blocks:
            h = b(h)
        return self.OutputType(F.pixel_shuffle(h, 2))


class Spatial(torch.nn.Module):
    InputType = namedtuple("Inputs", "x")
    OutputType = namedtuple("Outputs", "y s2 k2")

    def __init__(self):
        super().__init__()
        self.c3 = torch.nn.Conv2d(16, 16, 3, padding=1)
        self.s2 = torch.nn.Conv2d(16, 24, 3, stride=2, padding=1)
        self.k2 = torch.nn.Conv2d(16, 8, 2, stride=2)

    def forward(self, x):
        y = F.leaky_relu(self.c3(x), 0.1)
        return self.OutputType(y, self.s2(y), self.k2(x) + 0.5)


class FeatureUpdate(torch.nn.Module):
    """The recurrent-feature update: three channel thirds (a, b, g) of t, a
    sigmoid-gated blend of the history with a, a sigmoid gate and a
    per-channel scale.  encoder form: the concat of (scaled, blended) is the
    next node (fusion_matcher.cpp Case A); decoder form: scaled also feeds a
    LeakyReLU -> conv branch first and the concat comes later (Case B)."""

    def __init__(self, c, decoder):
        super().__init__()
        self.decoder = decoder
        self.scale = torch.nn.Parameter((torch.rand(1, c, 1, 1) + 0.5).half())
        if decoder:
            self.out = torch.nn.Conv2d(c, c, 1).half()
        names = "recon feature" if decoder else "feature"
        self.OutputType = namedtuple("Outputs", names)

    InputType = namedtuple("Inputs", "t hist")

    def forward(self, t, hist):
        a, b, g = t.chunk(3, 1)
        sb = torch.sigmoid(b)
        sg = torch.sigmoid(g)
        blended = sb * hist + (1 - sb) * a
        scaled = sg * blended * self.scale
        if not self.decoder:
            return self.OutputType(torch.cat((scaled, blended), 1))
        recon = self.out(F.leaky_relu(scaled, 0.1))
        return self.OutputType(recon, torch.cat((scaled, blended), 1))


class QuantTails(torch.nn.Module):
    """The latent quantisation tails in the node order the reference fuses
    (fusion_matcher.cpp try_y0_tail / try_y1_tail): y0 = round of the summed
    halves of (latent / clip(prior head, 0.11) - prior tail) * qs0, the
    dequantised update of both halves, the concat with the prior; y1 the same
    against prior2, added to the y0 update and multiplied by the clipped
    prior head."""
    InputType = namedtuple("Inputs", "prior latent qs0 us00 us01 prior2 qs1 us10 us11")
    OutputType = namedtuple("Outputs", "y_raw_0 y_raw_1 decoder_input prior_concat")

    def forward(self, prior, latent, qs0, us00, us01, prior2, qs1, us10, us11):
        s0, s1 = prior.chunk(2, 1)
        clipped = s0.clamp_min(0.11)
        norm = latent * clipped.reciprocal()
        scaled = (norm - s1) * qs0
        a0, a1 = scaled.chunk(2, 1)
        y0 = (a0 + a1).round()
        p0, p1 = s1.chunk(2, 1)
        c2 = torch.cat(((y0 + p0) * us00, (y0 + p1) * us01), 1)
        c3 = torch.cat((c2, prior), 1)
        sc = (norm - prior2) * qs1
        b0, b1 = sc.chunk(2, 1)
        y1 = (b0 + b1).round()
        q0, q1 = prior2.chunk(2, 1)
        c4 = torch.cat(((y1 + q0) * us10, (y1 + q1) * us11), 1)
        return self.OutputType(y0, y1, (c2 + c4) * clipped, c3)


@case
def example_q():
    torch.manual_seed(7)
    m = ExampleQ().eval()
    inputs = (torch.rand(1, 3, 8, 8).half(), torch.rand(1, 12, 4, 4).half(), torch.tensor([2], dtype=torch.int32))
    return m, inputs


@case
def block_stack_tiny():
    torch.manual_seed(11)
    m = Stack(16, 2).eval().half()
    with torch.no_grad():
        for p in m.parameters():
            p.mul_(0.5)
    return m, (torch.randn(1, 4, 12, 20).half(),)


@case
def spatial_convs():
    torch.manual_seed(13)
    m = Spatial().eval().half()
    return m, (torch.randn(1, 16, 13, 17).half(),)


@case
def feature_update_enc():
    torch.manual_seed(17)
    m = FeatureUpdate(8, decoder=False).eval()
    return m, (torch.randn(1, 24, 6, 10).half() * 2, torch.randn(1, 8, 6, 10).half())


@case
def feature_update_dec():
    torch.manual_seed(19)
    m = FeatureUpdate(16, decoder=True).eval()
    return m, (torch.randn(1, 48, 5, 9).half() * 2, torch.randn(1, 16, 5, 9).half())


@case
def quant_tails():
    torch.manual_seed(23)
    q, h, w = 8, 5, 7

    def u(c, lo, hi):
        return (torch.rand(1, c, h, w) * (hi - lo) + lo).half()

    inputs = (u(4 * q, -0.2, 2.0), (torch.randn(1, 2 * q, h, w) * 3).half(), u(2 * q, 0.25, 2.0),
              u(q, 0.25, 2.0), u(q, 0.25, 2.0), (torch.randn(1, 2 * q, h, w) * 3).half(), u(2 * q, 0.25, 2.0),
              u(q, 0.25, 2.0), u(q, 0.25, 2.0))
    return QuantTails().eval(), inputs


TAIL_CASES = {"feature_update_enc", "feature_update_dec", "quant_tails"}


def ref_cpu(bundle, part, inputs, isa, fusion=True):
    code = (
        "import sys, numpy as np; sys.path.insert(0, %r);"
        "from oracle.ref_backend import RefCpuBackend;"
        "d = np.load(%r); ins = [d[k] for k in sorted(d.files) if k.startswith('in')];"
        "outs = RefCpuBackend(%r, %r, 1).run(ins);"
        "np.savez(%r, *outs)" % (str(ROOT), str(bundle / "inputs.npz"), str(bundle), part,
                                 str(bundle / f"out_{isa}.npz")))
    env = dict(os.environ, MLVC_CPU_ISA=isa)
    if not fusion:
        env["MLVC_CPU_DISABLE_FUSION"] = "1"
    subprocess.run([sys.executable, "-c", code], check=True, env=env)
    d = np.load(bundle / f"out_{isa}.npz")
    outs = [d[f"arr_{i}"] for i in range(len(d.files))]
    (bundle / f"out_{isa}.npz").unlink()
    return outs


def main():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), "ref", f"REF={REF}"], check=True)
    from aot_tests import execute_graph
    for name, make in CASES.items():
        if ONLY and name not in ONLY:
            continue
        model, inputs = make()
        bundle = HERE / name
        part = bundle / "aot" / "model"
        part.mkdir(parents=True, exist_ok=True)
        with torch.inference_mode():
            compile_module(model, inputs, part, "00" * 32)
        np_inputs = [t.numpy() for t in inputs]
        np.savez(bundle / "inputs.npz", **{f"in{i}": a for i, a in enumerate(np_inputs)})
        scalar = ref_cpu(bundle, "model", np_inputs, "scalar")
        avx2 = ref_cpu(bundle, "model", np_inputs, "avx2")
        extra = {}
        if name in TAIL_CASES:
            unfused = ref_cpu(bundle, "model", np_inputs, "scalar", fusion=False)
            extra = {f"ref_cpu_scalar_unfused_{i}": a for i, a in enumerate(unfused)}
        replay = [t.float().numpy().astype(np.float16) for t in execute_graph(part, inputs)]
        with torch.inference_mode():
            eager = [t.float().numpy().astype(np.float16) for t in model(*inputs)]
        np.savez(bundle / "expected.npz",
                 **{f"ref_cpu_scalar_{i}": a for i, a in enumerate(scalar)},
                 **{f"ref_cpu_avx2_{i}": a for i, a in enumerate(avx2)},
                 **{f"replay_{i}": a for i, a in enumerate(replay)},
                 **{f"eager_{i}": a for i, a in enumerate(eager)}, **extra)
        print(name, [a.shape for a in scalar])


if __name__ == "__main__":
    main()
