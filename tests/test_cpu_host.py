"""Host-side logic without a GPU: the graph wire format (builder <-> protobuf
schema <-> the product's C++ decoder), graph validation errors, the C ABI
surface, the planner's kernel routing and fusion decisions (planning-only
backend), and the multi-replica throughput reduction over gloo ranks."""

import os
import re
import socket
from pathlib import Path

import numpy as np
import pytest

import mlvc_b200
from mlvc_b200 import Backend
from mlvc_b200.graph import GraphBuilder, build_block_stack, build_conv3x3, build_mlvc_decoder_standin
from oracle.graph_oracle import GraphOracle
from oracle.wire_schema import parse_graph

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
B200 = (148, 232448)  # SMs, opt-in shared memory per block


def plan(graph, weights, target=B200):
    be = Backend(plan_only_for=target)
    be.load_memory(graph, weights)
    return be


# ------------------------------------------------------------- C ABI
def test_c_abi_exports_every_declared_symbol():
    header = (ROOT / "include" / "mlvc_b200.h").read_text()
    names = set(re.findall(r"\b(mlvc_b200_[a-z0-9_]+)\s*\(", header))
    assert len(names) >= 30
    lib = mlvc_b200.lib()
    for n in sorted(names):
        assert hasattr(lib, n), n
    assert lib.mlvc_b200_abi_version() == 1


def test_library_has_no_link_time_driver_dependency():
    import subprocess
    out = subprocess.run(["ldd", str(mlvc_b200.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcuda" not in out and "libcudart" not in out


@pytest.mark.skipif(os.path.exists("/dev/nvidiactl"), reason="a GPU driver is present")
def test_create_without_driver_fails_loudly():
    with pytest.raises(RuntimeError, match="cuInit"):
        Backend(0)


def test_planning_only_backend_refuses_execution():
    gb, inputs = build_conv3x3(0, 64, 16, 24)
    be = plan(*gb.finish())
    with pytest.raises(RuntimeError, match="planning-only"):
        be.run(inputs)


# ------------------------------------------------------- wire format
def test_builder_graph_parses_with_protobuf_schema():
    gb, _ = build_block_stack(seed=0, channels=32, height=8, width=12, blocks=2)
    graph, weights = gb.finish()
    g = parse_graph(graph)
    assert g.schema_version == 3 and len(g.checkpoint_sha256) == 32 and len(g.weights_sha256) == 32
    assert g.arena_alignment == 256 and g.weights_bytes == len(weights)
    ops = [n.op for n in g.nodes]
    assert ops[0] == 14 and ops[-1] == 7 and ops.count(6) == 10
    # every runtime value is born at its producing node
    by_id = {t.id: t for t in g.tensors}
    for i, n in enumerate(g.nodes):
        assert by_id[n.outputs[0]].arena.birth == i


@pytest.mark.parametrize("case", ["example_q", "block_stack_tiny", "spatial_convs"])
def test_decoder_accepts_reference_compiled_graphs(case):
    """Graphs emitted by the reference's own AOT compiler decode, validate and plan."""
    d = GOLDEN / case / "aot" / "model"
    be = plan((d / "graph.pb").read_bytes(), (d / "weights.bin").read_bytes())
    o = GraphOracle.from_dir(GOLDEN / case, "model")
    assert [n for n, _, _ in be.inputs] == o.input_names()
    assert [n for n, _, _ in be.outputs] == o.output_names()
    assert be.steps()


def _corrupt(graph, mutate):
    g = parse_graph(graph)
    mutate(g)
    return g.SerializeToString()


BAD = {
    "schema": lambda g: setattr(g, "schema_version", 2),
    "provenance": lambda g: setattr(g, "weights_sha256", b"short"),
    "arena alignment": lambda g: setattr(g, "arena_alignment", 128),
    "tensor rank": lambda g: g.tensors[0].shape.extend([1, 1, 1, 1]),
    "dilation": lambda g: [n.conv.dilations.__setitem__(0, 2) for n in g.nodes if n.op == 6][:1],
    "asymmetric pad": lambda g: [n.conv.pads.__setitem__(0, 0) for n in g.nodes if n.op == 6][:1],
    "unknown op": lambda g: setattr(g.nodes[0], "op", 15),
    "birth": lambda g: setattr(g.tensors[[t.WhichOneof("storage") for t in g.tensors].index("arena")].arena,
                               "birth", 7),
    "empty outputs": lambda g: g.ClearField("outputs"),
}


@pytest.mark.parametrize("what", sorted(BAD))
def test_decoder_rejects_malformed_graphs(what):
    gb, _ = build_conv3x3(0, 64, 8, 8)
    graph, weights = gb.finish()
    bad = _corrupt(graph, BAD[what])
    with pytest.raises(RuntimeError, match="invalid AOT graph"):
        plan(bad, weights)


def test_decoder_rejects_truncation_and_weight_size():
    gb, _ = build_conv3x3(0, 64, 8, 8)
    graph, weights = gb.finish()
    with pytest.raises(RuntimeError, match="invalid AOT graph"):
        plan(graph[: len(graph) // 2], weights)
    with pytest.raises(RuntimeError, match="weights size"):
        plan(graph, weights[:-2])


def test_state_binding_validation():
    gb = GraphBuilder()
    x = gb.input("x", [1, 8, 4, 4])
    r = gb.input("ref", [1, 8, 4, 4])
    gb.output(gb.add(x, r), "y")
    graph, weights = gb.finish()
    be = Backend(plan_only_for=B200)
    with pytest.raises(RuntimeError, match="state binding"):
        be.load_memory(graph, weights, [(5, 0)])


# ----------------------------------------------------------- planner
def _kernels(be):
    return [s["kernel"] for s in be.steps()]


def test_plan_block_stack_fuses_like_the_reference(monkeypatch):
    """Conv+LeakyReLU, Conv+Add and Conv+Slice+Slice+Clip+Mul collapse into the
    tensor-core conv epilogue (fusion_registry.cpp:711-1036); with FFN fusion
    the ReGLU conv and the conv after it (+ residual Add) become one step, and
    the expand conv, depthwise conv and projection conv (+ Add) another."""
    gb, _ = build_block_stack(seed=0)
    be = plan(*gb.finish())
    k = _kernels(be)
    assert k.count("mlvc_mbconv_tc") == 8 and k.count("mlvc_ffn_tc") == 8 and len(k) == 18, k
    assert "mlvc_conv1x1_tc" not in k and "mlvc_dwconv_tc" not in k and "mlvc_depthwise3x3_f16" not in k
    assert "mlvc_unary_f16" not in k and "mlvc_binary_same_f16" not in k and "mlvc_reglu_f16" not in k
    nodes = [s["nodes"] for s in be.steps() if s["kernel"] == "mlvc_ffn_tc"]
    assert "6-12" in nodes  # conv + slice + slice + clip + mul + conv + add
    nodes = [s["nodes"] for s in be.steps() if s["kernel"] == "mlvc_mbconv_tc"]
    assert "1-5" in nodes  # conv + leaky + depthwise conv + conv + add
    flops = sum(s["flops"] for s in be.steps())
    assert abs(flops - 39.13e9) / 39.13e9 < 0.01  # config-2 algorithmic FLOPs
    assert all(s["smem"] > 233472 // 2 for s in be.steps() if s["kernel"] in ("mlvc_ffn_tc", "mlvc_mbconv_tc"))

    monkeypatch.setenv("MLVC_B200_MB_FUSION", "0")
    k = _kernels(plan(*gb.finish()))
    assert k.count("mlvc_conv1x1_tc") == 8 and k.count("mlvc_ffn_tc") == 8 and k.count("mlvc_dwconv_tc") == 8
    assert "mlvc_mbconv_tc" not in k and len(k) == 26
    nodes = [s["nodes"] for s in plan(*gb.finish()).steps() if s["kernel"] == "mlvc_dwconv_tc"]
    assert "3-5" in nodes  # depthwise conv + 1x1 conv + add

    monkeypatch.setenv("MLVC_B200_FFN_FUSION", "0")
    monkeypatch.setenv("MLVC_B200_DW_FUSION", "0")
    split = _kernels(plan(*gb.finish()))
    assert split.count("mlvc_conv1x1_tc") == 32 and split.count("mlvc_depthwise3x3_f16") == 8
    assert "mlvc_ffn_tc" not in split and "mlvc_dwconv_tc" not in split
    nodes = [s["nodes"] for s in plan(*gb.finish()).steps() if s["kernel"] == "mlvc_conv1x1_tc"]
    assert "6-10" in nodes  # conv + slice + slice + clip + mul


@pytest.mark.parametrize("c1,c2,oc,other_reader,absorbed", [
    (128, 128, 256, False, True), (64, 192, 64, False, True),
    (96, 128, 64, False, False),   # first operand not a multiple of 64 channels
    (128, 128, 256, True, False),  # the concat has another reader
])
def test_plan_concat_read_in_place_by_1x1(c1, c2, oc, other_reader, absorbed):
    """A channel concat whose only reader is the 1x1 conv right after it is
    not materialised: the conv reads its K panels from both tensors."""
    gb = GraphBuilder()
    a = gb.input("a", [1, c1, 6, 20])
    b = gb.input("b", [1, c2, 6, 20])
    cat = gb.concat([a, b], 1)
    gb.output(gb.conv(cat, gb.weight("w", np.zeros((oc, c1 + c2, 1, 1), np.float16))), "y")
    if other_reader:
        gb.output(gb.leaky_relu(cat, 0.1), "z")
    k = _kernels(plan(*gb.finish()))
    copies = sum(1 for x in k if x.startswith("mlvc_strided_copy"))
    assert (copies == 0) == absorbed, k
    assert "mlvc_conv1x1_tc" in k


@pytest.mark.parametrize("start,end,other_reader,absorbed", [
    (128, 256, False, True), (64, 128, False, True),
    (4, 68, False, False),     # slice start not 16-byte aligned (4 channels)
    (128, 256, True, False),   # the slice has another reader: materialised, then read in place
])
def test_plan_concat_of_channel_slice_read_in_place(start, end, other_reader, absorbed):
    """A concat operand that is a channel slice of a wider tensor, read only
    by the concat, is read in place by the 1x1 conv (no copy at all)."""
    gb = GraphBuilder()
    t = gb.leaky_relu(gb.input("t", [1, 256, 6, 20]), 0.1)
    b = gb.input("b", [1, 128, 6, 20])
    sl = gb.slice(t, 1, start, end)
    cat = gb.concat([b, sl], 1)
    gb.output(gb.conv(cat, gb.weight("w", np.zeros((64, 128 + end - start, 1, 1), np.float16))), "y")
    if other_reader:
        gb.output(gb.leaky_relu(sl, 0.2), "z")
    k = _kernels(plan(*gb.finish()))
    copies = sum(1 for x in k if x.startswith("mlvc_strided_copy"))
    assert (copies == 0) == absorbed, k
    assert "mlvc_conv1x1_tc" in k


@pytest.mark.parametrize("state_read_last", [False, True])
def test_plan_state_output_aliases_state_buffer(state_read_last):
    """A state-bound output is written in place into the state buffer when
    every read of the state input precedes its first write; when a later step
    still reads the state, the output is copied after the frame."""
    gb = GraphBuilder()
    x = gb.input("x", [1, 64, 6, 10])
    ref = gb.input("ref", [1, 64, 6, 10])
    w = gb.weight("w", np.zeros((64, 64, 1, 1), np.float16))
    y = gb.leaky_relu(gb.add(gb.conv(x, w), ref), 0.1)
    feat = gb.conv(y, w)
    if state_read_last:
        gb.output(gb.add(feat, ref), "y")  # reads the state after the output is written
    else:
        gb.output(y, "y")
    gb.output(feat, "feature")
    graph, weights = gb.finish()
    be = Backend(plan_only_for=B200)
    be.load_memory(graph, weights, [(1, 1)])
    assert ("state-copy" in _kernels(be)) == state_read_last


def test_plan_mlvc_decoder_standin():
    """The MLVC-shaped stand-in plans on the tensor-core path: every 1x1 conv
    (256-channel blocks, up-sampling convs) on tcgen05, LeakyReLU / residual /
    ReGLU in the conv epilogues, each 512-channel depthwise fused with the
    projection after it (+ residual); graph I/O as documented for the decoder."""
    gb, inputs = build_mlvc_decoder_standin(width=640, height=368)
    graph, weights = gb.finish()
    be = plan(graph, weights)
    k = _kernels(be)
    assert k.count("mlvc_conv1x1_tc") == 29 and k.count("mlvc_dwconv_tc") == 7, k
    # the hyperprior's row crop and full-width slice are views, the context
    # channel slice is read in place by the 1x1 conv after its concat; the
    # means slice and the latent concat are copies
    assert k.count("mlvc_strided_copy_v8_f16") == 3, k
    # the four x2 up-sampling pixel shuffles are folded into the 1x1 convs before them
    assert "mlvc_depth_to_space_r2_v8_f16" not in k and "mlvc_depth_to_space_f16" not in k, k
    assert "mlvc_depthwise3x3_f16" not in k
    assert "mlvc_conv_direct_f16" not in k and "mlvc_unary_f16" not in k and "mlvc_reglu_f16" not in k
    assert [tuple(s) for _, _, s in be.inputs] == [(1, 128, 3, 5), (1, 64, 23, 40), (1, 64, 23, 40),
                                                     (1, 256, 46, 80), (1,)]
    assert [tuple(s) for _, _, s in be.outputs] == [(1, 3, 368, 640), (1, 256, 46, 80)]


def test_plan_mlvcs_decoder_standin():
    """The MLVC-S-shaped stand-in (96 / 192-channel blocks, 48-channel
    latents) plans on the general paths: every 1x1 conv on tcgen05 (output
    channels not a multiple of 64 included), the 384-channel depthwise fused
    with its 192-channel projection, the 192-channel depthwise of the
    96-channel blocks stand-alone (a 96-column output is no whole 64-column
    panel), no scalar fallback; documented I/O shapes."""
    from mlvc_b200.graph import build_mlvcs_decoder_standin
    gb, inputs = build_mlvcs_decoder_standin(width=640, height=368)
    be = plan(*gb.finish())
    k = _kernels(be)
    assert k.count("mlvc_conv1x1_tc") == 34 and k.count("mlvc_dwconv_tc") == 6, k
    assert k.count("mlvc_depthwise3x3_f16") == 2, k
    assert "mlvc_conv_direct_f16" not in k and "mlvc_unary_f16" not in k and "mlvc_reglu_f16" not in k
    assert [tuple(s) for _, _, s in be.inputs] == [(1, 48, 6, 10), (1, 24, 23, 40), (1, 24, 23, 40),
                                                     (1, 96, 46, 80), (1,)]
    assert [tuple(s) for _, _, s in be.outputs] == [(1, 3, 368, 640), (1, 96, 46, 80)]


@pytest.mark.parametrize("c,e,c_out,leaky,fused", [
    (128, 256, 128, True, True), (64, 64, 64, False, True), (64, 192, 128, True, True), (128, 128, 64, True, True),
    (192, 256, 128, True, False),  # input channels above two 64-channel halo slices
    (48, 128, 64, True, False),    # input channels not a multiple of 64
    (128, 320, 128, True, False),  # expanded channels above the kernel's bias capacity
    (128, 256, 192, True, False),  # a W2 slice (C_out x 64) larger than one ring slot
    (128, 96, 64, True, False),    # expanded channels not a multiple of 64
])
def test_plan_mbconv_fusion_predicates(c, e, c_out, leaky, fused):
    gb = GraphBuilder()
    x = gb.input("x", [1, c, 11, 37])
    t = gb.conv(x, gb.weight("w1", np.zeros((e, c, 1, 1), np.float16)), gb.weight("b1", np.zeros(e, np.float16)))
    if leaky:
        t = gb.leaky_relu(t, 0.01)
    d = gb.conv(t, gb.weight("dw", np.zeros((e, 1, 3, 3), np.float16)), gb.weight("db", np.zeros(e, np.float16)),
                (1, 1), (1, 1), groups=e)
    gb.output(gb.conv(d, gb.weight("w2", np.zeros((c_out, e, 1, 1), np.float16))), "y")
    k = _kernels(plan(*gb.finish()))
    assert ("mlvc_mbconv_tc" in k) == fused, k
    if fused:
        assert k == ["mlvc_boundary_f16", "mlvc_mbconv_tc", "mlvc_boundary_f16"], k


def test_plan_mbconv_needs_single_consumers():
    """The expanded tensor and the depthwise result must have no other reader."""
    gb = GraphBuilder()
    x = gb.input("x", [1, 64, 8, 16])
    t = gb.leaky_relu(gb.conv(x, gb.weight("w1", np.zeros((128, 64, 1, 1), np.float16))), 0.01)
    d = gb.conv(t, gb.weight("dw", np.zeros((128, 1, 3, 3), np.float16)), None, (1, 1), (1, 1), groups=128)
    gb.output(gb.conv(d, gb.weight("w2", np.zeros((64, 128, 1, 1), np.float16))), "y")
    gb.output(t, "expanded")
    k = _kernels(plan(*gb.finish()))
    assert "mlvc_mbconv_tc" not in k and "mlvc_dwconv_tc" in k, k


@pytest.mark.parametrize("c,c_out,h,w,fused", [
    (256, 128, 92, 160, True), (64, 64, 13, 20, True), (128, 128, 9, 300, True), (64, 256, 8, 8, True),
    (64, 64, 13, 17, True),     # ragged 16 x 8 tiles
    (64, 64, 4, 2000, True),    # wide image (2-D tiles: any width)
    (48, 64, 8, 8, False),      # channels not a multiple of 64
    (64, 96, 8, 8, False),      # output channels not a multiple of 64
    (512, 256, 8, 8, True),     # taps in two 256-channel TMA boxes
    (320, 128, 8, 8, True),     # taps in a 256- and a 64-channel box
    (576, 128, 8, 8, False),    # more channels than the kernel takes (C > 512)
])
def test_plan_depthwise_fusion_predicates(c, c_out, h, w, fused):
    gb = GraphBuilder()
    x = gb.input("x", [1, c, h, w])
    d = gb.conv(x, gb.weight("dw", np.zeros((c, 1, 3, 3), np.float16)), gb.weight("db", np.zeros(c, np.float16)),
                (1, 1), (1, 1), groups=c)
    gb.output(gb.conv(d, gb.weight("w", np.zeros((c_out, c, 1, 1), np.float16))), "y")
    k = _kernels(plan(*gb.finish()))
    assert ("mlvc_dwconv_tc" in k) == fused, k


@pytest.mark.parametrize("c,hidden,c_out,fused", [
    (128, 256, 128, True), (64, 64, 64, True), (256, 128, 128, True), (64, 192, 64, True),
    (48, 64, 64, False),     # C not a multiple of 64
    (128, 512, 128, False),  # hidden above the kernel's bias capacity
    (128, 256, 96, False),   # C_out not a multiple of 64 (64-column output panels)
    (128, 256, 256, False),  # output tile larger than the two hidden panels it is staged in
])
def test_plan_ffn_fusion_predicates(c, hidden, c_out, fused):
    gb = GraphBuilder()
    x = gb.input("x", [1, c, 9, 21])
    t = gb.conv(x, gb.weight("w1", np.zeros((2 * hidden, c, 1, 1), np.float16)))
    gate, lin = gb.slice(t, 1, 0, hidden), gb.slice(t, 1, hidden, 2 * hidden)
    y = gb.conv(gb.mul(gb.clip(gate, 0.0, 1.0), lin), gb.weight("w2", np.zeros((c_out, hidden, 1, 1), np.float16)))
    gb.output(y, "y")
    k = _kernels(plan(*gb.finish()))
    assert ("mlvc_ffn_tc" in k) == fused, k


def test_plan_conv3x3_uses_halo_kernel():
    gb, _ = build_conv3x3(0)
    be = plan(*gb.finish())
    steps = [s for s in be.steps() if s["kernel"] == "mlvc_convkxk_tc"]
    assert len(steps) == 1 and steps[0]["flops"] == 4341104640.0
    assert steps[0]["smem"] <= 232448


@pytest.mark.parametrize("ic,oc,k,stride,expect", [
    (64, 64, 3, 1, "mlvc_convkxk_tc"), (128, 256, 2, 2, "mlvc_convkxk_tc"), (64, 128, 3, 2, "mlvc_convkxk_tc"),
    (24, 24, 3, 1, "mlvc_conv_direct_f16"), (3, 32, 3, 2, "mlvc_conv_direct_f16"),
    (24, 136, 1, 1, "mlvc_conv1x1_tc"), (8, 8, 1, 1, "mlvc_conv1x1_tc"),
])
def test_plan_conv_routing(ic, oc, k, stride, expect):
    gb = GraphBuilder()
    x = gb.input("x", [1, ic, 13, 17])
    w = gb.weight("w", np.zeros((oc, ic, k, k), np.float16))
    gb.output(gb.conv(x, w, None, (stride, stride), ((k - 1) // 2 if stride == 1 else (1 if k == 3 else 0),) * 2), "y")
    assert expect in _kernels(plan(*gb.finish()))


def test_plan_smaller_smem_target_still_plans():
    gb, _ = build_block_stack(seed=0, channels=128, height=23, width=40, blocks=1)
    be = plan(*gb.finish(), target=(20, 100 * 1024))
    assert all(s["smem"] <= 100 * 1024 for s in be.steps())


# ------------------------------------------------- replicas over gloo
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _replica_rank(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    # each rank is an independent replica: plan its own copy of the graph
    gb, _ = build_block_stack(seed=0, channels=32, height=8, width=12, blocks=1)
    be = plan(*gb.finish())
    assert be.steps()
    value, ms_max = bench.replica_throughput(10.0 * (rank + 1), 50, world)
    q.put((rank, value, ms_max))
    dist.destroy_process_group()


def test_replica_throughput_gloo_two_ranks():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_replica_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(2))
    for _, value, ms_max in res:
        assert ms_max == 20.0  # max over ranks
        assert value == pytest.approx(2 * 50 / 0.020)


@pytest.mark.parametrize("decoder", [False, True])
def test_plan_feature_update_fusion(decoder, monkeypatch):
    """The recurrent-feature update (3 slices, 2 sigmoids, 6 binary operators,
    concat) becomes one step, as in the reference's matchers
    (fusion_registry.cpp:405-709); in the decoder form the separately consumed
    halves are materialised as well."""
    from feature_graphs import feature_update_graph
    gb, _ = feature_update_graph(16, 6, 10, decoder)
    k = _kernels(plan(*gb.finish()))
    assert "mlvc_feature_update_f16" in k, k
    # no sigmoid or binary operator left (the decoder graph's own LeakyReLU stays)
    assert k.count("mlvc_unary_f16") == (1 if decoder else 0) and "mlvc_binary_same_f16" not in k, k
    monkeypatch.setenv("MLVC_B200_TAIL_FUSION", "0")
    split = _kernels(plan(*gb.finish()))
    assert "mlvc_feature_update_f16" not in split
    assert split.count("mlvc_unary_f16") == (3 if decoder else 2), split


def test_plan_quantisation_tails_fused(monkeypatch):
    """The y0 (19 operators) and y1 (15 operators) quantisation tails become
    one step each, as in the reference's matchers (fusion_registry.cpp:14-404)."""
    from quant_graphs import quant_tails_graph
    gb, _ = quant_tails_graph(16, 5, 7)
    steps = plan(*gb.finish()).steps()
    k = [s["kernel"] for s in steps]
    assert k.count("mlvc_y0_tail_f16") == 1 and k.count("mlvc_y1_tail_f16") == 1, k
    assert "mlvc_unary_f16" not in k and "mlvc_binary_same_f16" not in k, k
    assert [s["nodes"] for s in steps if s["kernel"] == "mlvc_y0_tail_f16"] == ["0-18"]
    assert [s["nodes"] for s in steps if s["kernel"] == "mlvc_y1_tail_f16"] == ["19-33"]
    monkeypatch.setenv("MLVC_B200_TAIL_FUSION", "0")
    split = _kernels(plan(*gb.finish()))
    assert "mlvc_y0_tail_f16" not in split and split.count("mlvc_unary_f16") == 4  # clip, reciprocal, 2 rounds


# ------------------------------------------------- entropy-coder inputs
def test_scale_shape_and_validation():
    """mlvc_b200_scale_shape follows the reference plane sizes
    (core/src/model.cpp:94-126) and rejects the channel mappings that
    extract_scales rejects or would read outside its base table with."""
    import ctypes
    lib = mlvc_b200.lib()

    def shape(*fields):
        zc, sc = ctypes.c_size_t(), ctypes.c_size_t()
        rc = lib.mlvc_b200_scale_shape(ctypes.byref(mlvc_b200.ScaleConfig(*fields)), ctypes.byref(zc),
                                       ctypes.byref(sc))
        if rc:
            raise RuntimeError(lib.mlvc_b200_last_error().decode())
        return zc.value, sc.value

    assert shape(128, 1920, 1080, 128, 16, 8, 2, 127) == (128 * 9 * 15, 64 * 68 * 120)
    assert shape(128, 640, 368, 128, 16, 8, 2, 127) == (128 * 3 * 5, 64 * 23 * 40)
    with pytest.raises(RuntimeError, match="channel mapping is invalid"):
        shape(32, 640, 368, 128, 16, 8, 2, 127)   # base channels 64 > hyper 32
    with pytest.raises(RuntimeError, match="channel mapping is invalid"):
        shape(8, 640, 368, 5, 16, 8, 3, 127)      # (3 + 2) // 3 would leave the base table
    with pytest.raises(RuntimeError, match="positive"):
        shape(128, 640, 368, 128, 16, 0, 2, 127)


def test_planning_only_backend_refuses_entropy_inputs():
    be = Backend(plan_only_for=B200)
    with pytest.raises(RuntimeError, match="planning-only"):
        be.integer_values(np.zeros(4, np.float16))
    with pytest.raises(RuntimeError, match="planning-only"):
        be.extract_scales(np.zeros((1, 128, 3, 5), np.float16), 640, 368, 128)


@pytest.mark.parametrize("shape,axis,start,end,aliased", [
    ([1, 64, 16, 16], 2, 0, 8, True),    # leading rows of an NHWC tensor
    ([1, 64, 16, 16], 2, 4, 12, True),   # a row range at a 256-byte aligned offset
    ([1, 64, 16, 16], 3, 0, 16, True),   # full-width slice: the whole tensor
    ([1, 64, 16, 16], 3, 0, 8, False),   # part of every row: strided
    ([1, 64, 16, 16], 1, 0, 32, False),  # channel slice: strided
    ([1, 8, 6, 5], 2, 1, 4, False),      # contiguous, but the offset (80 bytes) is not 256-byte aligned
])
def test_plan_contiguous_slice_is_a_view(shape, axis, start, end, aliased):
    """A Slice whose result is one contiguous, aligned byte range of its
    source becomes a view into the source's buffer instead of a copy."""
    c = shape[1]
    gb = GraphBuilder()
    x = gb.input("x", shape)
    t = gb.conv(x, gb.weight("w1", np.zeros((c, c, 1, 1), np.float16)))
    s = gb.slice(t, axis, start, end)
    cs = gb.shape(s)[1]
    gb.output(gb.conv(s, gb.weight("w2", np.zeros((c, cs, 1, 1), np.float16))), "y")
    k = _kernels(plan(*gb.finish()))
    copies = [n for n in k if n.startswith("mlvc_strided_copy")]
    assert (not copies) == aliased, k


@pytest.mark.parametrize("case,copies", [("input_rows", 1), ("view_of_view", 0), ("input_channels_concat", 0)])
def test_plan_slice_views_of_inputs_and_chains(case, copies):
    """A row slice of a graph input is copied (only values the schedule
    produces become views); a contiguous slice of a contiguous slice is a
    view of the first source; a channel slice of an input is still read in
    place by the 1x1 conv after its concat."""
    gb = GraphBuilder()
    w = lambda cin: gb.weight("w", np.zeros((64, cin, 1, 1), np.float16))  # noqa: E731
    if case == "input_rows":
        x = gb.input("x", [1, 64, 16, 16])
        gb.output(gb.conv(gb.slice(x, 2, 0, 8), w(64)), "y")
    elif case == "view_of_view":
        t = gb.leaky_relu(gb.input("x", [1, 64, 16, 16]), 0.1)
        gb.output(gb.conv(gb.slice(gb.slice(t, 2, 0, 12), 2, 4, 12), w(64)), "y")
    else:
        x = gb.input("x", [1, 128, 16, 16])
        b = gb.input("b", [1, 64, 16, 16])
        gb.output(gb.conv(gb.concat([b, gb.slice(x, 1, 64, 128)], 1), w(128)), "y")
    k = _kernels(plan(*gb.finish()))
    assert sum(1 for n in k if n.startswith("mlvc_strided_copy")) == copies, k


def _bad_shape_graph(what):
    gb = GraphBuilder()
    a = gb.input("a", [1, 64, 8, 16])
    b = gb.input("b", [1, 64, 16, 16])
    if what == "concat":      # operands disagree outside the concat axis
        y = gb.concat([a, b], 1)
    elif what == "slice":     # declared output runs past the input
        y = gb.slice(b, 2, 4, 16)
        gb.tensors[y].shape[2] = 16
    elif what == "binary":    # operand neither 1 nor the output's extent
        y = gb.add(a, a)
        gb.tensors[y].shape[2] = 16
    elif what == "unary":     # elementwise output larger than its input
        y = gb.leaky_relu(a, 0.2)
        gb.tensors[y].shape[2] = 16
    elif what == "shuffle":   # pixel shuffle output that does not follow from its input
        y = gb.depth_to_space(b, 2)
        gb.tensors[y].shape[1] = 32
    elif what == "gather":    # declared output larger than one table row
        table = gb.weight("table", np.zeros((4, 64, 1, 1), np.float16))
        y = gb.mul(a, gb.gather(table, gb.input("q", [1], "int32")))
        gb.tensors[gb.nodes[-2].output].shape[0] = 2
    else:                     # conv output larger than stride / padding allow
        y = gb.conv(b, gb.weight("w", np.zeros((64, 64, 3, 3), np.float16)), None, (2, 2), (1, 1))
        gb.tensors[y].shape[2] = 16
    gb.output(gb.leaky_relu(y, 0.1), "y")
    return gb.finish()


@pytest.mark.parametrize("what,message", [("concat", "Concat operand shapes"), ("slice", "exceeds its input"),
                                          ("binary", "does not broadcast"), ("unary", "changes the tensor shape"),
                                          ("shuffle", "pixel .un.shuffle output shape"),
                                          ("conv", "Conv shapes do not match"),
                                          ("gather", "Gather takes one index")])
def test_plan_rejects_inconsistent_operand_extents(what, message):
    """Copy and elementwise kernels index their operands by the output's
    extents; a graph whose declared shapes disagree is rejected at load
    instead of reading or writing past a buffer."""
    with pytest.raises(RuntimeError, match=message):
        plan(*_bad_shape_graph(what))


def test_plan_rejects_conv_that_is_not_rank_4():
    gb = GraphBuilder()
    x = gb.input("x", [1, 64, 16, 16])
    y = gb.conv(x, gb.weight("w", np.zeros((64, 64, 1, 1), np.float16)))
    gb.tensors[x].shape = [64, 16, 16]  # rank-3 input
    gb.output(y, "y")
    with pytest.raises(RuntimeError, match="Conv input, weights and output must be rank 4"):
        plan(*gb.finish())


def _slice_from(start, dim=8):
    """Slice of rows [start, start + 4) of a [1, 16, dim, 12] input, with the
    start literal written as given (the builder would normalise it)."""
    gb = GraphBuilder()
    x = gb.input("x", [1, 16, dim, 12])
    y = gb.slice(x, 2, 0, 4)
    gb.tensors[gb.nodes[-1].inputs[1]].data = np.array([start], np.int64)
    gb.output(gb.leaky_relu(y, 0.5), "y")
    return gb.finish()


def test_plan_clamps_slice_start_like_the_reference(tmp_path):
    """A start below -dim wraps to a negative value, which the reference CPU
    plan clamps to 0 (backends/cpu/src/execution_plan.cpp:596-599): the graph
    loads and slices from row 0, like the reference CPU backend."""
    from oracle.ref_backend import LIB_PATH, RefCpuBackend
    graph, weights = _slice_from(-9)
    plan(graph, weights)  # accepted
    x = np.random.default_rng(0).standard_normal((1, 16, 8, 12)).astype(np.float16)
    want = GraphOracle(graph, weights).run([x])[0]
    assert np.array_equal(want, GraphOracle(*_slice_from(0)).run([x])[0])
    if LIB_PATH.exists():
        part = tmp_path / "aot" / "m"
        part.mkdir(parents=True)
        (part / "graph.pb").write_bytes(graph)
        (part / "weights.bin").write_bytes(weights)
        (ref,) = RefCpuBackend(tmp_path, "m", 1).run([x])
        assert np.array_equal(ref.view(np.uint16), want.view(np.uint16))
    with pytest.raises(RuntimeError, match="exceeds its input"):
        plan(*_slice_from(6))  # rows 6..9 of 8


@pytest.mark.parametrize("fold", [True, False])
def test_plan_pixel_shuffle_folded_into_1x1(fold, monkeypatch):
    """A 2x pixel shuffle that is the only consumer of a 1x1 conv (+ LeakyReLU)
    with channels in multiples of 256 joins the conv's step; not when the conv
    output has another reader, a residual epilogue, or the switch is off."""
    if not fold:
        monkeypatch.setenv("MLVC_B200_D2S_FUSION", "0")
    rng = np.random.default_rng(0)

    def graph(extra_reader=False, oc=512):
        gb = GraphBuilder()
        x = gb.input("x", [1, 64, 6, 10])
        y = gb.leaky_relu(gb.conv(x, gb.weight("w", (rng.standard_normal((oc, 64, 1, 1)) * 0.1).astype(np.float16))),
                          0.01)
        one = gb.weight("one", np.ones((1, 1, 1, 1), np.float16))
        gb.output(gb.mul(gb.depth_to_space(y, 2), one), "y")  # (a shuffle straight into an output joins the boundary)
        if extra_reader:
            gb.output(y, "pre")
        return gb.finish()

    k = _kernels(plan(*graph()))
    assert ("mlvc_depth_to_space_r2_v8_f16" in k) == (not fold), k
    assert "mlvc_depth_to_space_r2_v8_f16" in _kernels(plan(*graph(extra_reader=True)))
    assert "mlvc_depth_to_space_r2_v8_f16" in _kernels(plan(*graph(oc=384)))  # 96 channels: not a multiple of 64
