"""Builder for mlvc AOT graph bundles (aot/<part>/graph.pb + weights.bin).

The on-disk contract is the reference's graph schema 3
(proto/mlvc_model.proto:30-83) as validated by runtime/src/aot_graph.cpp:110-283:
tensor IDs are dense from 1, weights live 256-byte aligned in weights.bin,
runtime tensors carry a 256-byte aligned arena slot whose `birth` is the index
of the producing node, inputs have no storage, and both SHA-256 fields are 32
bytes.  The reference produces such bundles by tracing a PyTorch module
(tools/python/mlvc_tools/aot.py:233-278); this builder emits the same operator
vocabulary directly, which lets the benchmark and the GPU tests generate their
seeded synthetic models on a machine that has no PyTorch model code.

The protobuf wire format is written by hand (varints, length-delimited
submessages, packed repeated scalars) so this module has no dependency on a
generated protobuf class.
"""

from __future__ import annotations

import hashlib
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

ALIGN = 256
DTYPE_CODE = {"fp16": 1, "int32": 2, "int64": 3}
DTYPE_BYTES = {"fp16": 2, "int32": 4, "int64": 8}
OP_CODE = dict(Add=1, Sub=2, Mul=3, Clip=4, Concat=5, Conv=6, DepthToSpace=7, Gather=8, LeakyRelu=9,
               Reciprocal=10, Round=11, Sigmoid=12, Slice=13, SpaceToDepth=14)


def _align(v: int) -> int:
    return (v + ALIGN - 1) // ALIGN * ALIGN


# ---------------------------------------------------------------- wire writer
def _varint(v: int) -> bytes:
    if v < 0:
        v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(field_no: int, wire: int) -> bytes:
    return _varint(field_no << 3 | wire)


def _f_varint(field_no, v):
    return _key(field_no, 0) + _varint(v) if v else b""


def _f_bytes(field_no, data: bytes):
    return _key(field_no, 2) + _varint(len(data)) + data


def _f_packed(field_no, values):
    values = list(values)
    if not values:
        return b""
    return _f_bytes(field_no, b"".join(_varint(int(v)) for v in values))


def _zigzag(v: int) -> int:
    return (v << 1) ^ (v >> 31)


@dataclass
class _Tensor:
    name: str
    dtype: str
    shape: list
    kind: str  # "input" | "weight" | "value"
    data: np.ndarray | None = None
    producer: int = -1
    last_use: int = -1
    tid: int = 0


@dataclass
class _Node:
    op: str
    inputs: list
    output: str
    attrs: dict = field(default_factory=dict)


class GraphBuilder:
    """Emits one graph part.  Tensors are referenced by name."""

    def __init__(self):
        self.tensors: dict[str, _Tensor] = {}
        self.nodes: list[_Node] = []
        self.inputs: list[str] = []
        self.outputs: list[str] = []
        self._lit = 0

    # -------------------------------------------------------------- values
    def input(self, name, shape, dtype="fp16"):
        self.tensors[name] = _Tensor(name, dtype, list(shape), "input")
        self.inputs.append(name)
        return name

    def weight(self, name, array):
        array = np.ascontiguousarray(array)
        dtype = {np.dtype(np.float16): "fp16", np.dtype(np.int64): "int64"}[array.dtype]
        self.tensors[name] = _Tensor(name, dtype, list(array.shape), "weight", array)
        return name

    def literal(self, values, dtype=np.int64):
        name = f"literal_{self._lit:05d}"
        self._lit += 1
        return self.weight(name, np.asarray(values, dtype).reshape(-1))

    def _emit(self, op, inputs, shape, attrs=None, dtype="fp16", name=None):
        index = len(self.nodes)
        name = name or f"value_{index:05d}"
        self.tensors[name] = _Tensor(name, dtype, list(shape), "value", producer=index)
        self.nodes.append(_Node(op, list(inputs), name, attrs or {}))
        return name

    def shape(self, name):
        return list(self.tensors[name].shape)

    # ----------------------------------------------------------------- ops
    def conv(self, x, w, b=None, stride=(1, 1), pad=(0, 0), groups=1, name=None):
        n, ic, ih, iw = self.shape(x)
        oc, icg, kh, kw = self.shape(w)
        if icg * groups != ic:
            raise ValueError("conv channel mismatch")
        oh = (ih + 2 * pad[0] - kh) // stride[0] + 1
        ow = (iw + 2 * pad[1] - kw) // stride[1] + 1
        attrs = dict(strides=list(stride), pads=list(pad) * 2, dilations=[1, 1], groups=groups)
        return self._emit("Conv", [x, w] + ([b] if b is not None else []), [n, oc, oh, ow], attrs, name=name)

    def _binary(self, op, a, b, name=None):
        shape = list(np.broadcast_shapes(tuple(self.shape(a)), tuple(self.shape(b))))
        return self._emit(op, [a, b], shape, name=name)

    def add(self, a, b, name=None):
        return self._binary("Add", a, b, name)

    def sub(self, a, b, name=None):
        return self._binary("Sub", a, b, name)

    def mul(self, a, b, name=None):
        return self._binary("Mul", a, b, name)

    def leaky_relu(self, x, alpha=0.01, name=None):
        return self._emit("LeakyRelu", [x], self.shape(x), dict(alpha=alpha), name=name)

    def clip(self, x, lo=None, hi=None, name=None):
        ins = [x, self.literal([lo], np.float16) if lo is not None else "",
               self.literal([hi], np.float16) if hi is not None else ""]
        while ins and ins[-1] == "":
            ins.pop()
        return self._emit("Clip", ins, self.shape(x), name=name)

    def unary(self, op, x, name=None):
        return self._emit(op, [x], self.shape(x), name=name)

    def slice(self, x, axis, start, end, step=1, name=None):
        shape = self.shape(x)
        start, end, step = slice(start, end, step).indices(shape[axis])
        shape[axis] = len(range(start, end, step))
        ins = [x] + [self.literal([v]) for v in (start, end, axis, step)]
        return self._emit("Slice", ins, shape, name=name)

    def concat(self, xs, axis, name=None):
        shape = self.shape(xs[0])
        shape[axis] = sum(self.shape(v)[axis] for v in xs)
        return self._emit("Concat", list(xs), shape, dict(axis=axis), name=name)

    def gather(self, data, index, name=None):
        shape = [1] + self.shape(data)[1:]
        return self._emit("Gather", [data, index], shape, dict(axis=0), name=name)

    def depth_to_space(self, x, r, name=None):
        n, c, h, w = self.shape(x)
        return self._emit("DepthToSpace", [x], [n, c // (r * r), h * r, w * r], dict(block_size=r), name=name)

    def space_to_depth(self, x, r, name=None):
        n, c, h, w = self.shape(x)
        return self._emit("SpaceToDepth", [x], [n, c * r * r, h // r, w // r], dict(block_size=r), name=name)

    def output(self, value, name):
        """Marks `value` as a graph output, renaming it to `name`."""
        if value != name:
            t = self.tensors.pop(value)
            t.name = name
            self.tensors[name] = t
            for node in self.nodes:
                node.inputs = [name if v == value else v for v in node.inputs]
                if node.output == value:
                    node.output = name
            self.outputs = [name if v == value else v for v in self.outputs]
        self.outputs.append(name)
        return name

    # ------------------------------------------------------------ finalise
    def _plan_arena(self):
        for index, node in enumerate(self.nodes):
            for v in node.inputs:
                if v:
                    self.tensors[v].last_use = max(self.tensors[v].last_use, index)
        values = [t for t in self.tensors.values() if t.kind == "value"]
        events = []
        for t in values:
            size = _align(int(np.prod(t.shape)) * DTYPE_BYTES[t.dtype])
            death = len(self.nodes) if t.name in self.outputs else max(t.last_use, t.producer)
            events.append((t.producer, death, size, t))
        live, end, plan = [], 0, {}
        for birth, death, size, t in sorted(events, key=lambda e: (e[0], e[3].name)):
            live = [e for e in live if e[0] >= birth]  # (death, offset, size)
            taken = sorted((o, o + s) for _, o, s in live)
            offset, cursor = None, 0
            for lo, hi in taken:  # first gap that fits
                if lo - cursor >= size:
                    offset = cursor
                    break
                cursor = max(cursor, hi)
            if offset is None:
                offset = cursor
            end = max(end, offset + size)
            live.append((death, offset, size))
            plan[t.name] = (offset, size, birth, death)
        return plan, end

    def finish(self, checkpoint_sha256: bytes = b"\0" * 32):
        used = set(self.inputs) | set(self.outputs)
        for node in self.nodes:
            used.update(v for v in node.inputs if v)
            used.add(node.output)
        names = sorted(n for n in self.tensors if n in used)
        ids = {n: i for i, n in enumerate(names, 1)}
        weights = bytearray()
        woff = {}
        for n in names:
            t = self.tensors[n]
            if t.kind == "weight":
                weights.extend(b"\0" * (_align(len(weights)) - len(weights)))
                woff[n] = len(weights)
                weights.extend(t.data.tobytes())
        plan, arena_bytes = self._plan_arena()
        out = bytearray()
        out += _f_varint(1, 3)
        out += _f_bytes(2, checkpoint_sha256)
        for n in names:
            t = self.tensors[n]
            body = _f_varint(1, ids[n]) + _f_bytes(2, n.encode()) + _f_varint(3, DTYPE_CODE[t.dtype])
            body += _f_packed(4, t.shape)
            if t.kind == "weight":
                body += _f_bytes(6, _f_varint(1, woff[n]) + _f_varint(2, t.data.nbytes))
            elif t.kind == "value":
                o, s, b, d = plan[n]
                body += _f_bytes(5, _f_varint(1, o) + _f_varint(2, s) + _f_varint(3, b) + _f_varint(4, d))
            out += _f_bytes(3, body)
        out += _f_packed(4, [ids[n] for n in self.inputs])
        out += _f_packed(5, [ids[n] for n in self.outputs])
        for node in self.nodes:
            body = _f_varint(1, OP_CODE[node.op])
            body += _f_packed(2, [ids[v] if v else 0 for v in node.inputs])
            body += _f_packed(3, [ids[node.output]])
            a = node.attrs
            if node.op == "Conv":
                body += _f_bytes(4, _f_packed(1, a["strides"]) + _f_packed(2, a["pads"]) +
                                 _f_packed(3, a["dilations"]) + _f_varint(4, a["groups"]))
            elif node.op in ("Concat", "Gather"):
                body += _f_bytes(5, _f_varint(1, _zigzag(int(a["axis"]))))
            elif node.op == "LeakyRelu":
                body += _f_bytes(6, _key(1, 5) + struct.pack("<f", a["alpha"]))
            elif node.op in ("DepthToSpace", "SpaceToDepth"):
                body += _f_bytes(7, _f_varint(1, a["block_size"]))
            out += _f_bytes(6, body)
        out += _f_varint(7, arena_bytes)
        out += _f_varint(8, ALIGN)
        out += _f_varint(9, len(weights))
        out += _f_bytes(10, hashlib.sha256(weights).digest())
        return bytes(out), bytes(weights)

    def save(self, model_dir, part):
        graph, weights = self.finish()
        d = Path(model_dir) / "aot" / part
        d.mkdir(parents=True, exist_ok=True)
        (d / "graph.pb").write_bytes(graph)
        (d / "weights.bin").write_bytes(weights)
        return d


# ------------------------------------------------------ synthetic workloads
def _fp16(a):
    return np.asarray(a, np.float32).astype(np.float16)


def kaiming_normal(rng, shape, gain=np.sqrt(2.0)):
    """He/Kaiming normal, fan-in mode: N(0, gain^2 / fan_in).  gain sqrt(2) is the
    ReLU-family gain (torch.nn.init.kaiming_normal_ default); gain 1 is the
    linear gain."""
    fan_in = int(np.prod(shape[1:]))
    return _fp16(rng.standard_normal(shape, dtype=np.float32) * np.float32(gain / np.sqrt(fan_in)))


def small_bias(rng, n):
    return _fp16(rng.uniform(-0.1, 0.1, n).astype(np.float32))


def build_conv3x3(seed=0, channels=64, height=184, width=320):
    """Config 1: one FP16 3x3 s1 p1 conv C->C with bias.  W ~ N(0, sqrt(2/(9C))),
    b ~ U(-0.1, 0.1), x ~ N(0, 1), all drawn from one seeded generator."""
    rng = np.random.default_rng(seed)
    gb = GraphBuilder()
    x = gb.input("x", [1, channels, height, width])
    w = gb.weight("conv.weight", kaiming_normal(rng, (channels, channels, 3, 3)))
    b = gb.weight("conv.bias", small_bias(rng, channels))
    gb.output(gb.conv(x, w, b, (1, 1), (1, 1)), "y")
    inputs = [_fp16(rng.standard_normal((1, channels, height, width), dtype=np.float32))]
    return gb, inputs


def build_block_stack(seed=0, channels=128, height=92, width=160, blocks=8):
    """Config 2: pixel_unshuffle(2) -> `blocks` x [1x1 C->2C + LeakyReLU(0.01);
    depthwise 3x3 (2C); 1x1 2C->C + residual; 1x1 C->4C -> ReGLU (clip(gate, 0, 1)
    * linear) -> 1x1 2C->C + residual] -> pixel_shuffle(2).  Input [1, C/4, 2H, 2W]
    ~ N(0, 1); biases U(-0.1, 0.1).

    Kaiming-normal weights with the gain of the operator that follows each conv:
    sqrt(2) for the expand conv (followed by LeakyReLU, the case He
    initialisation is derived for), 1 for the convs feeding linear operators
    (depthwise -> project, project/ffn_out -> residual add, ffn_in -> ReGLU).
    With sqrt(2) everywhere the un-normalised residual stream grows about 6x in
    variance per block and overflows FP16 (inf) inside block 7, which would make
    the workload's output meaningless; with these gains it stays in range."""
    rng = np.random.default_rng(seed)
    c = channels
    gb = GraphBuilder()
    x = gb.input("x", [1, c // 4, height * 2, width * 2])
    h = gb.space_to_depth(x, 2)
    for i in range(blocks):
        p = f"block{i}."
        w1 = gb.weight(p + "expand.weight", kaiming_normal(rng, (2 * c, c, 1, 1), np.sqrt(2.0)))
        b1 = gb.weight(p + "expand.bias", small_bias(rng, 2 * c))
        wd = gb.weight(p + "dw.weight", kaiming_normal(rng, (2 * c, 1, 3, 3), 1.0))
        bd = gb.weight(p + "dw.bias", small_bias(rng, 2 * c))
        w2 = gb.weight(p + "project.weight", kaiming_normal(rng, (c, 2 * c, 1, 1), 1.0))
        b2 = gb.weight(p + "project.bias", small_bias(rng, c))
        w3 = gb.weight(p + "ffn_in.weight", kaiming_normal(rng, (4 * c, c, 1, 1), 1.0))
        b3 = gb.weight(p + "ffn_in.bias", small_bias(rng, 4 * c))
        w4 = gb.weight(p + "ffn_out.weight", kaiming_normal(rng, (c, 2 * c, 1, 1), 1.0))
        b4 = gb.weight(p + "ffn_out.bias", small_bias(rng, c))
        t = gb.leaky_relu(gb.conv(h, w1, b1), 0.01)
        t = gb.conv(t, wd, bd, (1, 1), (1, 1), groups=2 * c)
        h = gb.add(h, gb.conv(t, w2, b2))
        f = gb.conv(h, w3, b3)
        g = gb.slice(f, 1, 0, 2 * c)
        lin = gb.slice(f, 1, 2 * c, 4 * c)
        f = gb.mul(gb.clip(g, 0.0, 1.0), lin)
        h = gb.add(h, gb.conv(f, w4, b4))
    gb.output(gb.depth_to_space(h, 2), "y")
    inputs = [_fp16(rng.standard_normal((1, c // 4, height * 2, width * 2), dtype=np.float32))]
    return gb, inputs


def _depth_conv_block(gb, rng, h, c, prefix, branch_gain=1.0):
    """One block of the profile's depth_conv_block_params (models/profiles/
    profiles.json: LeakyReLU, gated chunk mode, ReLU1 FFN gate), as in config 2:
    1x1 C->2C + LeakyReLU(0.01); depthwise 3x3 (2C); 1x1 2C->C + residual; 1x1
    C->4C -> ReGLU (clip(gate, 0, 1) * linear) -> 1x1 2C->C + residual.
    branch_gain scales the two residual-branch output convs (the profile's
    zero_init_residual starts them at zero)."""
    w1 = gb.weight(prefix + "expand.weight", kaiming_normal(rng, (2 * c, c, 1, 1), np.sqrt(2.0)))
    b1 = gb.weight(prefix + "expand.bias", small_bias(rng, 2 * c))
    wd = gb.weight(prefix + "dw.weight", kaiming_normal(rng, (2 * c, 1, 3, 3), 1.0))
    bd = gb.weight(prefix + "dw.bias", small_bias(rng, 2 * c))
    w2 = gb.weight(prefix + "project.weight", _fp16(kaiming_normal(rng, (c, 2 * c, 1, 1), 1.0) * branch_gain))
    b2 = gb.weight(prefix + "project.bias", small_bias(rng, c))
    w3 = gb.weight(prefix + "ffn_in.weight", kaiming_normal(rng, (4 * c, c, 1, 1), 1.0))
    b3 = gb.weight(prefix + "ffn_in.bias", small_bias(rng, 4 * c))
    w4 = gb.weight(prefix + "ffn_out.weight", _fp16(kaiming_normal(rng, (c, 2 * c, 1, 1), 1.0) * branch_gain))
    b4 = gb.weight(prefix + "ffn_out.bias", small_bias(rng, c))
    t = gb.leaky_relu(gb.conv(h, w1, b1), 0.01)
    t = gb.conv(t, wd, bd, (1, 1), (1, 1), groups=2 * c)
    h = gb.add(h, gb.conv(t, w2, b2))
    f = gb.conv(h, w3, b3)
    g = gb.slice(f, 1, 0, 2 * c)
    lin = gb.slice(f, 1, 2 * c, 4 * c)
    f = gb.mul(gb.clip(g, 0.0, 1.0), lin)
    return gb.add(h, gb.conv(f, w4, b4))


def _recon_out(gb, rng, r, cin, name, gain):
    """Final 1x1 conv to 3 x 64 channels ahead of the x8 pixel shuffle: weights
    Kaiming-normal scaled by `gain`, bias 0.5 + U(-0.1, 0.1), so that x_hat
    lies mostly inside [0, 1] (the range the codec's YUV conversion keeps;
    with unit gain nearly every sample would clip to 0 or 255)."""
    w = gb.weight(name + ".weight", _fp16(kaiming_normal(rng, (3 * 64, cin, 1, 1), 1.0) * gain))
    b = gb.weight(name + ".bias", _fp16(small_bias(rng, 3 * 64).astype(np.float32) + 0.5))
    return gb.depth_to_space(gb.conv(r, w, b), 8)


def synthetic_yuv420(frame, width, height, seed=0, shift=2, sigma=8.0):
    """Seeded synthetic 8-bit YUV420 content of BASELINE configs 3-5: a smooth
    diagonal luma gradient and two chroma gradients plus Gaussian noise
    (sigma 8 on luma, sigma / 2 on chroma), moving `shift` pixels to the
    right per frame (a global translation: frame f is the content window at
    x offset shift * f).  Returns (Y [h, w], U [h/2, w/2], V [h/2, w/2]) uint8."""
    rng = np.random.default_rng(seed)
    span = width + shift * 64  # a window that holds 64 frames of motion
    noise_y = rng.standard_normal((height, span)).astype(np.float32) * sigma
    noise_c = rng.standard_normal((2, height // 2, span // 2)).astype(np.float32) * (sigma / 2)
    off = (shift * frame) % (span - width + 1)
    xs = np.arange(off, off + width, dtype=np.float32)[None, :]
    ys = np.arange(height, dtype=np.float32)[:, None]
    y = 32.0 + 160.0 * (xs / span + ys / height) / 2.0 + noise_y[:, off:off + width]
    cx, cy = xs[:, ::2] / span, ys[::2] / height
    coff = off // 2
    u = 96.0 + 64.0 * cx + noise_c[0, :, coff:coff + width // 2]
    v = 160.0 - 64.0 * cy + noise_c[1, :, coff:coff + width // 2]
    q = lambda a: np.clip(np.rint(a), 0, 255).astype(np.uint8)
    return q(y), q(u), q(v)


def build_mlvc_decoder_standin(seed=0, width=1920, height=1088, feature=256, latent=128, hyper=128, qp_num=72,
                               q_index=21, blocks_y=2, blocks_feature=2, blocks_recon=2, recon_gain=0.02):
    """MLVC-shaped decoder STAND-IN.  The upstream MLVC architecture source is
    absent from the reference (tools/python/mlvc_tools/source.py imports it from
    an external package), so this is not the MLVC network; it is assembled from
    what the reference documents:

    * decoder I/O and plane sizes (docs/design.md, "Fixed graph I/O"):
      z_raw [1, hyper, ceil(H/128), ceil(W/128)], y_raw_0 / y_raw_1
      [1, latent/2, ceil(H/16), ceil(W/16)], ref_feature [1, feature, H/8, W/8],
      q_index_shifted [1] int32 -> x_hat [1, 3, H, W], feature [1, feature, H/8, W/8];
    * the blocks of the profile's depth_conv_block_params (_depth_conv_block);
    * native CRD pixel shuffle for up-sampling (graph schema 3) and a QP-indexed
      Gather of per-QP scale rows (qp_num = 72 tables).

    Layout: hyperprior decoder z -> 1x1 + LeakyReLU -> block -> three
    [1x1 to 4 x channels, pixel shuffle 2] stages -> crop to the y plane ->
    prior (means | context); y = concat(y_raw_0, y_raw_1) * qscale[q] + means;
    contextual decoder concat(y, context) -> 1x1 -> blocks_y blocks at 1/16 ->
    1x1 + pixel shuffle 2 -> concat(ref_feature) -> 1x1 -> blocks_feature
    blocks at 1/8 = new feature; reconstruction blocks_recon blocks -> 1x1 to
    3 x 64 (gain recon_gain, bias 0.5: x_hat within [0, 1]) -> pixel shuffle
    8 = x_hat.  Weights Kaiming-normal (gain as in
    build_block_stack), the residual-branch output convs scaled by 0.25 (with
    full gain the un-normalised 256-channel residual stream grows to std ~100
    and the two CPU implementations differ by 10 % rel-L2 at the output; at
    0.25 the outputs have std ~1 and the CPU-vs-CPU spread is ~1e-3), biases
    U(-0.1, 0.1), seeded; inputs: integer-valued latents, N(0, 1) reference
    feature."""
    rng = np.random.default_rng(seed)
    h8, w8 = -(-height // 8), -(-width // 8)
    h16, w16 = -(-height // 16), -(-width // 16)
    hz, wz = -(-height // 128), -(-width // 128)
    if h8 != 2 * h16 or w8 != 2 * w16 or height != 8 * h8 or width != 8 * w8:
        raise ValueError("stand-in needs H and W multiples of 16")
    gb = GraphBuilder()
    z = gb.input("z_raw", [1, hyper, hz, wz])
    y0 = gb.input("y_raw_0", [1, latent // 2, h16, w16])
    y1 = gb.input("y_raw_1", [1, latent // 2, h16, w16])
    ref = gb.input("ref_feature", [1, feature, h8, w8])
    q = gb.input("q_index_shifted", [1], "int32")

    def conv1x1(x, cin, cout, name, gain=1.0):
        w = gb.weight(name + ".weight", kaiming_normal(rng, (cout, cin, 1, 1), gain))
        return gb.conv(x, w, gb.weight(name + ".bias", small_bias(rng, cout)))

    # hyperprior decoder: 1/128 -> 1/16 (x8), cropped to the y plane
    t = gb.leaky_relu(conv1x1(z, hyper, feature, "hyper.in", np.sqrt(2.0)), 0.01)
    t = _depth_conv_block(gb, rng, t, feature, "hyper.block0.", 0.25)
    for i in range(3):
        t = gb.depth_to_space(conv1x1(t, feature, 4 * feature, f"hyper.up{i}"), 2)
    t = gb.slice(gb.slice(t, 2, 0, h16), 3, 0, w16)
    means = gb.slice(t, 1, 0, latent)
    context = gb.slice(t, 1, latent, feature)
    # QP-indexed dequantisation of the latents
    table = gb.weight("qscale", rng.uniform(0.5, 2.0, (qp_num, latent, 1, 1)).astype(np.float16))
    y = gb.add(gb.mul(gb.concat([y0, y1], 1), gb.gather(table, q)), means)
    # contextual decoder: 1/16 -> 1/8, joined with the reference feature
    t = conv1x1(gb.concat([y, context], 1), latent + feature - latent, feature, "ctx.in")
    for i in range(blocks_y):
        t = _depth_conv_block(gb, rng, t, feature, f"ctx.block{i}.", 0.25)
    t = gb.depth_to_space(conv1x1(t, feature, 4 * feature, "ctx.up"), 2)
    t = conv1x1(gb.concat([t, ref], 1), 2 * feature, feature, "feat.in")
    for i in range(blocks_feature):
        t = _depth_conv_block(gb, rng, t, feature, f"feat.block{i}.", 0.25)
    new_feature = t
    # reconstruction: 1/8 -> full resolution
    r = t
    for i in range(blocks_recon):
        r = _depth_conv_block(gb, rng, r, feature, f"recon.block{i}.", 0.25)
    x_hat = _recon_out(gb, rng, r, feature, "recon.out", recon_gain)
    gb.output(x_hat, "x_hat")
    gb.output(new_feature, "feature")
    inputs = [np.rint(rng.standard_normal((1, hyper, hz, wz)) * 4).astype(np.float16),
              np.rint(rng.standard_normal((1, latent // 2, h16, w16)) * 3).astype(np.float16),
              np.rint(rng.standard_normal((1, latent // 2, h16, w16)) * 3).astype(np.float16),
              _fp16(rng.standard_normal((1, feature, h8, w8), dtype=np.float32)),
              np.array([q_index], np.int32)]
    return gb, inputs


def build_mlvc_encoder_standin(seed=0, width=1920, height=1088, feature=256, latent=128, hyper=128, qp_num=72,
                               q_index=21, blocks_analysis=1, blocks_latent=1, blocks_mirror=1, ref_gain=0.25,
                               mirror_gain=0.25):
    """MLVC-shaped encoder STAND-IN (the upstream MLVC architecture is absent).
    Built from what the reference documents about the encoder:

    * graph I/O (docs/design.md, "Fixed graph I/O"): x [1, 3, H, W] pixels in
      [0, 1], ref_feature [1, feature, H/8, W/8], q_index_shifted [1] int32 ->
      feature [1, feature, H/8, W/8] (the new DPB feature, the final node, so a
      state binding input 1 <- output 0 aliases it), z_raw
      [1, hyper, ceil(H/128), ceil(W/128)], y_raw_0 / y_raw_1
      [1, latent/2, ceil(H/16), ceil(W/16)], all integer-valued latents;
    * the latent quantisation tails in the node order the reference fuses
      (y0 then y1: backends/cpu/src/fusion_matcher.cpp:543-850,
      backends/driver_cubin/src/fusion_registry.cpp:14-404), fed by a
      hyperprior that mirrors the decoder stand-in's;
    * the recurrent-feature update in its encoder form (three channel thirds,
      two sigmoids, a gated blend with the previous feature, a per-channel
      scale, then the concat: fusion_matcher.cpp:413-541 Case A);
    * the profile's depth-conv block (_depth_conv_block), native CRD pixel
      (un)shuffle and strided 3 x 3 convolutions for down-sampling.

    Layout: x -> pixel unshuffle 8 -> 1x1 + LeakyReLU -> concat(ref_feature)
    -> 1x1 -> blocks_analysis blocks at 1/8 -> 3x3 s2 + LeakyReLU ->
    blocks_latent blocks at 1/16 -> 1x1 = y; hyperprior encoder: three 3x3 s2
    convs (1/32, 1/64, 1/128) -> Round = z_raw; hyperprior decoder as in the
    decoder stand-in -> prior (4 x latent/2 channels); quantisation scales
    qs0 / qs1 = clip(1x1(prior), 0.25, 4) x the QP-indexed scale row,
    update scales clip(1x1(prior), 0.25, 4), second prior 1x1(prior); y0
    tail -> y_raw_0, y1 tail -> y_raw_1 and the dequantised latent; the
    mirror of the decoder's context path: concat(dequantised latent, prior
    concat) -> 1x1 to 4 x feature -> pixel shuffle 2 -> concat(ref_feature)
    -> 1x1 -> blocks_mirror blocks -> 1x1 to 3 x feature/2 -> feature update
    with the previous feature's second half as history = feature.  Weights
    as in build_mlvc_decoder_standin, seeded."""
    rng = np.random.default_rng(seed)
    h8, w8 = -(-height // 8), -(-width // 8)
    h16, w16 = -(-height // 16), -(-width // 16)
    if h8 != 2 * h16 or w8 != 2 * w16 or height != 8 * h8 or width != 8 * w8:
        raise ValueError("stand-in needs H and W multiples of 16")
    q = latent // 2
    gb = GraphBuilder()
    x = gb.input("x", [1, 3, height, width])
    ref = gb.input("ref_feature", [1, feature, h8, w8])
    qi = gb.input("q_index_shifted", [1], "int32")

    def conv1x1(v, cin, cout, name, gain=1.0, damp_from=None):
        """damp_from: input channels from this index on (the previous
        feature's part of a concat) get weights scaled by ref_gain."""
        w = kaiming_normal(rng, (cout, cin, 1, 1), gain)
        if damp_from is not None:
            w = w.astype(np.float32)
            w[:, damp_from:] *= ref_gain
            w = _fp16(w)
        return gb.conv(v, gb.weight(name + ".weight", w), gb.weight(name + ".bias", small_bias(rng, cout)))

    def conv3x3s2(v, cin, cout, name, gain=1.0):
        w = gb.weight(name + ".weight", kaiming_normal(rng, (cout, cin, 3, 3), gain))
        return gb.conv(v, w, gb.weight(name + ".bias", small_bias(rng, cout)), (2, 2), (1, 1))

    # analysis: 1/8 with the reference feature, then 1/16
    t = gb.leaky_relu(conv1x1(gb.space_to_depth(x, 8), 3 * 64, feature, "ana.in", np.sqrt(2.0)), 0.01)
    t = conv1x1(gb.concat([t, ref], 1), 2 * feature, feature, "ana.ctx", damp_from=feature)
    for i in range(blocks_analysis):
        t = _depth_conv_block(gb, rng, t, feature, f"ana.block{i}.", 0.25)
    t = gb.leaky_relu(conv3x3s2(t, feature, feature, "ana.down", np.sqrt(2.0)), 0.01)
    for i in range(blocks_latent):
        t = _depth_conv_block(gb, rng, t, feature, f"lat.block{i}.", 0.25)
    y = conv1x1(t, feature, latent, "lat.out")
    # hyperprior encoder: 1/16 -> 1/128, rounded
    hz = gb.leaky_relu(conv3x3s2(y, latent, hyper, "hyenc.0", np.sqrt(2.0)), 0.01)
    hz = gb.leaky_relu(conv3x3s2(hz, hyper, hyper, "hyenc.1", np.sqrt(2.0)), 0.01)
    z = gb.unary("Round", conv3x3s2(hz, hyper, hyper, "hyenc.2", 2.0))
    # hyperprior decoder (as in the decoder stand-in), cropped to the y plane
    p = gb.leaky_relu(conv1x1(z, hyper, feature, "hyper.in", np.sqrt(2.0)), 0.01)
    p = _depth_conv_block(gb, rng, p, feature, "hyper.block0.", 0.25)
    for i in range(3):
        p = gb.depth_to_space(conv1x1(p, feature, 4 * feature, f"hyper.up{i}"), 2)
    prior = gb.slice(gb.slice(p, 2, 0, h16), 3, 0, w16)  # [1, feature = 4q, h16, w16]
    table = gb.weight("qscale", rng.uniform(0.5, 2.0, (qp_num, latent, 1, 1)).astype(np.float16))
    qrow = gb.gather(table, qi)
    qs0 = gb.mul(gb.clip(conv1x1(prior, feature, latent, "qs0"), 0.25, 4.0), qrow)
    qs1 = gb.mul(gb.clip(conv1x1(prior, feature, latent, "qs1"), 0.25, 4.0), qrow)
    us0 = gb.clip(conv1x1(prior, feature, q, "us0"), 0.25, 4.0)
    us1 = gb.clip(conv1x1(prior, feature, q, "us1"), 0.25, 4.0)
    prior2 = conv1x1(prior, feature, latent, "prior2")
    # y0 tail (19 operators in the exported order)
    s0 = gb.slice(prior, 1, 0, 2 * q)
    s1 = gb.slice(prior, 1, 2 * q, 4 * q)
    clipped = gb.clip(s0, 0.11, 65504.0)
    norm = gb.mul(y, gb.unary("Reciprocal", clipped))
    scaled = gb.mul(gb.sub(norm, s1), qs0)
    a0, a1 = gb.slice(scaled, 1, 0, q), gb.slice(scaled, 1, q, 2 * q)
    y0 = gb.unary("Round", gb.add(a0, a1))
    p0, p1 = gb.slice(s1, 1, 0, q), gb.slice(s1, 1, q, 2 * q)
    c2 = gb.concat([gb.mul(gb.add(y0, p0), us0), gb.mul(gb.add(y0, p1), us1)], 1)
    c3 = gb.concat([c2, prior], 1)
    # y1 tail (15 operators)
    sc = gb.mul(gb.sub(norm, prior2), qs1)
    b0, b1 = gb.slice(sc, 1, 0, q), gb.slice(sc, 1, q, 2 * q)
    y1 = gb.unary("Round", gb.add(b0, b1))
    r0, r1 = gb.slice(prior2, 1, 0, q), gb.slice(prior2, 1, q, 2 * q)
    c4 = gb.concat([gb.mul(gb.add(y1, r0), us0), gb.mul(gb.add(y1, r1), us1)], 1)
    y_hat = gb.mul(gb.add(c2, c4), clipped)
    # mirror of the decoder's context path, then the recurrent-feature update
    m = conv1x1(gb.concat([y_hat, c3], 1), 2 * latent + feature, 4 * feature, "mir.up", mirror_gain)
    m = conv1x1(gb.concat([gb.depth_to_space(m, 2), ref], 1), 2 * feature, feature, "mir.in", damp_from=feature)
    for i in range(blocks_mirror):
        m = _depth_conv_block(gb, rng, m, feature, f"mir.block{i}.", 0.25)
    half = feature // 2
    u = conv1x1(m, feature, 3 * half, "upd.in")
    hist = gb.slice(ref, 1, half, feature)
    ua, ub, ug = gb.slice(u, 1, 0, half), gb.slice(u, 1, half, 2 * half), gb.slice(u, 1, 2 * half, 3 * half)
    sb, sg = gb.unary("Sigmoid", ub), gb.unary("Sigmoid", ug)
    blended = gb.add(gb.mul(sb, hist), gb.mul(gb.sub(gb.weight("upd.one", np.array([1.0], np.float16)), sb), ua))
    scale = gb.weight("upd.scale", rng.uniform(0.5, 1.5, (1, half, 1, 1)).astype(np.float16))
    new_feature = gb.concat([gb.mul(gb.mul(sg, blended), scale), blended], 1)
    gb.output(new_feature, "feature")
    gb.output(z, "z_raw")
    gb.output(y0, "y_raw_0")
    gb.output(y1, "y_raw_1")
    Y, U, V = synthetic_yuv420(0, width, height - 8 if height % 16 == 0 else height, seed)
    xin = np.zeros((1, 3, height, width), np.float16)
    xin[0, 0, :Y.shape[0]] = Y / 255.0
    xin[0, 1, :Y.shape[0]] = np.repeat(np.repeat(U, 2, 0), 2, 1) / 255.0
    xin[0, 2, :Y.shape[0]] = np.repeat(np.repeat(V, 2, 0), 2, 1) / 255.0
    inputs = [xin, _fp16(rng.standard_normal((1, feature, h8, w8), dtype=np.float32)),
              np.array([q_index], np.int32)]
    return gb, inputs


def build_mlvcs_decoder_standin(seed=0, width=640, height=368, feature=96, latent=48, hyper=48, hidden=192,
                                recon=192, y_scale_repeat=4, qp_num=72, q_index=21, hyper_blocks=2, blocks_y=2,
                                blocks_feature=2, blocks_recon=2, recon_gain=0.02):
    """MLVC-S-shaped decoder STAND-IN (the upstream MLVC-S architecture is
    absent, like MLVC's).  Built from what the reference documents about the
    small profile (models/profiles/profiles.json "mlvc-s-psnr-v1": hidden and
    recon channels 192, two hyperprior blocks, y_scale_repeat 4, z and y 48
    channels, the same depth-conv block; docs/design.md: feature 96 channels,
    a mini hyperprior with a 6 x 10 z plane at 640x368, i.e. z at 1/64):

    z_raw [1, 48, ceil(H/64), ceil(W/64)] -> 1x1 + LeakyReLU to 192 ->
    hyper_blocks blocks -> two [1x1 to 4 x 192, pixel shuffle 2] stages ->
    crop to the y plane -> prior (means 48 | context 144); y =
    concat(y_raw_0, y_raw_1) * qscale[q] + means; concat(y, context) -> 1x1
    -> blocks_y blocks at 1/16 (192) -> 1x1 to 4 x 96 + pixel shuffle 2 ->
    concat(ref_feature) -> 1x1 -> blocks_feature blocks at 1/8 (96) = new
    feature; 1x1 to 192 -> blocks_recon blocks -> 1x1 to 3 x 64 (gain
    recon_gain, bias 0.5) -> pixel shuffle 8 = x_hat.  Weights and inputs as in build_mlvc_decoder_standin.
    The 96- and 192-channel blocks take the kernels' general paths (separate
    expand conv, stand-alone or fused depthwise, ReGLU GEMM + 1x1)."""
    rng = np.random.default_rng(seed)
    h8, w8 = -(-height // 8), -(-width // 8)
    h16, w16 = -(-height // 16), -(-width // 16)
    hz, wz = -(-height // 64), -(-width // 64)
    if h8 != 2 * h16 or w8 != 2 * w16 or height != 8 * h8 or width != 8 * w8:
        raise ValueError("stand-in needs H and W multiples of 16")
    gb = GraphBuilder()
    z = gb.input("z_raw", [1, hyper, hz, wz])
    y0 = gb.input("y_raw_0", [1, latent // 2, h16, w16])
    y1 = gb.input("y_raw_1", [1, latent // 2, h16, w16])
    ref = gb.input("ref_feature", [1, feature, h8, w8])
    q = gb.input("q_index_shifted", [1], "int32")

    def conv1x1(x, cin, cout, name, gain=1.0):
        w = gb.weight(name + ".weight", kaiming_normal(rng, (cout, cin, 1, 1), gain))
        return gb.conv(x, w, gb.weight(name + ".bias", small_bias(rng, cout)))

    # mini hyperprior decoder: 1/64 -> 1/16 (x4), cropped to the y plane
    t = gb.leaky_relu(conv1x1(z, hyper, hidden, "hyper.in", np.sqrt(2.0)), 0.01)
    for i in range(hyper_blocks):
        t = _depth_conv_block(gb, rng, t, hidden, f"hyper.block{i}.", 0.25)
    for i in range(2):
        t = gb.depth_to_space(conv1x1(t, hidden, 4 * hidden, f"hyper.up{i}"), 2)
    t = gb.slice(gb.slice(t, 2, 0, h16), 3, 0, w16)
    means = gb.slice(t, 1, 0, latent)
    context = gb.slice(t, 1, latent, hidden)
    table = gb.weight("qscale", rng.uniform(0.5, 2.0, (qp_num, latent, 1, 1)).astype(np.float16))
    y = gb.add(gb.mul(gb.concat([y0, y1], 1), gb.gather(table, q)), means)
    # contextual decoder: 1/16 -> 1/8, joined with the reference feature
    t = conv1x1(gb.concat([y, context], 1), hidden, hidden, "ctx.in")
    for i in range(blocks_y):
        t = _depth_conv_block(gb, rng, t, hidden, f"ctx.block{i}.", 0.25)
    t = gb.depth_to_space(conv1x1(t, hidden, 4 * feature, "ctx.up"), 2)
    t = conv1x1(gb.concat([t, ref], 1), 2 * feature, feature, "feat.in")
    for i in range(blocks_feature):
        t = _depth_conv_block(gb, rng, t, feature, f"feat.block{i}.", 0.25)
    new_feature = t
    # reconstruction: 1/8 -> full resolution
    r = conv1x1(t, feature, recon, "recon.in")
    for i in range(blocks_recon):
        r = _depth_conv_block(gb, rng, r, recon, f"recon.block{i}.", 0.25)
    x_hat = _recon_out(gb, rng, r, recon, "recon.out", recon_gain)
    gb.output(x_hat, "x_hat")
    gb.output(new_feature, "feature")
    inputs = [np.rint(rng.standard_normal((1, hyper, hz, wz)) * 4).astype(np.float16),
              np.rint(rng.standard_normal((1, latent // 2, h16, w16)) * 3).astype(np.float16),
              np.rint(rng.standard_normal((1, latent // 2, h16, w16)) * 3).astype(np.float16),
              _fp16(rng.standard_normal((1, feature, h8, w8), dtype=np.float32)),
              np.array([q_index], np.int32)]
    return gb, inputs
