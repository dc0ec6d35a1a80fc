"""Codec I/O on the B200 slot path (reference: BufferedCodecBackend's
configure_codec_io / encoder_input_yuv / decoder_output_yuv,
runtime/include/mlvc/runtime/backend.hpp:69-96, with the conversions of
core/src/yuv.cpp).  A YUV420 frame goes into the pinned slot buffer, the GPU
converts it into the model input tensor, the schedule runs, and the GPU
converts the output tensor back into a YUV420 frame; the bytes must equal the
oracle's conversions around the oracle's graph, exactly (the conversions are
bit-exact by construction and the graph below is elementwise)."""

import numpy as np
import pytest

from mlvc_b200 import Backend
from mlvc_b200.graph import GraphBuilder
from oracle import yuv_oracle
from oracle.graph_oracle import GraphOracle

pytestmark = pytest.mark.gpu


def _graph(mw, mh):
    gb = GraphBuilder()
    x = gb.input("x", [1, 3, mh, mw])
    aux = gb.input("aux", [1, 3, mh, mw])
    c = gb.weight("c", np.array([0.3], np.float16).reshape(1, 1, 1, 1))
    y = gb.leaky_relu(gb.sub(gb.add(x, aux), c), 0.1)
    gb.output(y, "x_hat")
    return gb.finish()


@pytest.mark.parametrize("w,h,mw,mh,pr", [(64, 48, 64, 48, 1.0), (58, 40, 64, 48, 1.0), (40, 62, 64, 48, 1.0),
                                          (320, 184, 320, 192, 1.0)])
def test_codec_io_yuv_round_trip(w, h, mw, mh, pr):
    graph, weights = _graph(mw, mh)
    be = Backend(0)
    be.load_memory(graph, weights)
    be.reset_state()
    be.configure_codec_io(w, h, mw, mh, pr, slots=2, input_index=0, output_index=0)
    oracle = GraphOracle(graph, weights)
    rng = np.random.default_rng(w + 7 * h)
    frames = [rng.integers(0, 256, w * h * 3 // 2, dtype=np.uint8) for _ in range(4)]
    auxes = [(rng.standard_normal((1, 3, mh, mw)) * 0.2).astype(np.float16) for _ in range(4)]
    want = []
    for f, a in zip(frames, auxes):
        t, _ = yuv_oracle.yuv_to_tensor(f, w, h, mw, mh, pr)
        (xh,) = oracle.run([t, a])
        want.append(yuv_oracle.tensor_to_yuv(xh, w, h, pr))
    got = [None] * len(frames)
    for i, (f, a) in enumerate(zip(frames, auxes)):
        slot = i % 2
        if i >= 2:
            be.wait_slot(slot)
            got[i - 2] = np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(slot)])
        y, u, v = be.slot_input_yuv(slot)
        planes = yuv_oracle.split_planes(f, w, h)
        y[...], u[...], v[...] = planes
        be.slot_input(slot, 1)[...] = a
        be.submit(slot)
    for i in range(len(frames) - 2, len(frames)):
        be.wait_slot(i % 2)
        got[i] = np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(i % 2)])
    for g, wnt in zip(got, want):
        assert np.array_equal(g, wnt), np.flatnonzero(g != wnt)[:10]


def test_codec_io_output_only_and_errors():
    mw, mh = 64, 48
    graph, weights = _graph(mw, mh)
    be = Backend(0)
    be.load_memory(graph, weights)
    be.reset_state()
    with pytest.raises(RuntimeError, match="larger than the model"):
        be.configure_codec_io(80, 80, mw, mh)
    with pytest.raises(RuntimeError, match="even"):
        be.configure_codec_io(63, 48, mw, mh)
    be.configure_codec_io(60, 44, mw, mh, slots=1, input_index=None, output_index=0)
    with pytest.raises(RuntimeError, match="no codec input"):
        be.slot_input_yuv(0)
    rng = np.random.default_rng(5)
    x = (rng.random((1, 3, mh, mw)) * 1.2).astype(np.float16)
    a = np.zeros((1, 3, mh, mw), np.float16)
    be.slot_input(0, 0)[...] = x
    be.slot_input(0, 1)[...] = a
    be.submit(0)
    be.wait_slot(0)
    (xh,) = GraphOracle(graph, weights).run([x, a])
    got = np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(0)])
    assert np.array_equal(got, yuv_oracle.tensor_to_yuv(xh, 60, 44))


def _x8_graph(mw, mh):
    """x_hat from a 192-channel 1/8-scale tensor through the x8 pixel shuffle,
    as the MLVC decoders produce it (the output boundary folds the shuffle)."""
    gb = GraphBuilder()
    f = gb.input("f", [1, 192, mh // 8, mw // 8])
    s = gb.weight("s", (np.random.default_rng(3).random((1, 192, 1, 1)) + 0.5).astype(np.float16))
    gb.output(gb.depth_to_space(gb.mul(f, s), 8), "x_hat")
    return gb.finish()


@pytest.mark.parametrize("w,h,pr,fused", [(64, 48, 1.0, True), (64, 40, 1.0, True), (56, 48, 255.0, True),
                                          (58, 40, 1.0, False), (40, 64, 1.0, False)])
def test_codec_output_from_nhwc_x8(w, h, pr, fused, monkeypatch):
    """The slot path converts the decoded frame to YUV420 straight from the
    NHWC tensor of the x8 pixel shuffle when the frame is not rotated and its
    size is a multiple of 8 (58 x 40: width not a multiple of 8; 40 x 64:
    rotated onto the 64 x 48 canvas, both through the boundary kernel and the
    NCHW conversion).  Either way the bytes equal the oracle's conversion of
    the oracle's x_hat, and the fused path equals the unfused one."""
    mw, mh = 64, 48
    graph, weights = _x8_graph(mw, mh)
    rng = np.random.default_rng(w * 3 + h)
    frames = [(rng.random((1, 192, mh // 8, mw // 8)) * 1.1 * pr - 0.05 * pr).astype(np.float16) for _ in range(3)]
    oracle = GraphOracle(graph, weights)
    want = [yuv_oracle.tensor_to_yuv(oracle.run([f])[0], w, h, pr) for f in frames]
    outs = {}
    for mode in ("1", "0"):
        monkeypatch.setenv("MLVC_B200_YUV_FUSION", mode)
        be = Backend(0)
        be.load_memory(graph, weights)
        be.reset_state()
        be.configure_codec_io(w, h, mw, mh, pr, slots=1, input_index=None, output_index=0)
        assert be.codec_output_fused() == (fused and mode == "1")
        got = []
        for f in frames:
            be.slot_input(0, 0)[...] = f
            be.submit(0)
            be.wait_slot(0)
            got.append(np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(0)]).copy())
        outs[mode] = got
        be.close()
    for g1, g0, wnt in zip(outs["1"], outs["0"], want):
        assert np.array_equal(g1, wnt), np.flatnonzero(g1 != wnt)[:10]
        assert np.array_equal(g0, wnt)
