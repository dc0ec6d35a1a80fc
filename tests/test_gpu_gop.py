"""BASELINE config 4 on the MLVC-shaped decoder stand-in: a 32-frame GOP (an
I-frame from a zeroed reference feature, then 31 P-frames that each consume
the previous frame's feature) at q_index 0, 21 and 51, through the slot path
with the codec's YUV420 output conversion, against the reference CPU backend
(compiled from its sources) run frame by frame with its own carried state.

The recurrent state is bound as the codec pipeline binds it for the decoder
(input 3 <- output 1, codec/src/pipeline.cpp:161-176) and is reset only at the
I-frame.  q reaches the graph through submit(slot, shifted_q), the
reference's submit_decoder(slot, shifted_q).  Per frame the decoded YUV420
frame must satisfy the reference's own reconstruction rules
(docs/codec-compatibility.md, "Reconstruction and tensor rules": maximum YUV
sample error at most 1 and PSNR at least 60 dB against the reference's
reconstruction) and the PSNR against the source content must be within
0.01 dB of the reference's.  The source content is the seeded synthetic
YUV420 motion sequence of the benchmark configurations; the latents are
seeded integer-valued symbols (the upstream encoder network is absent).
"""

import numpy as np
import pytest

from mlvc_b200 import Backend
from mlvc_b200.graph import build_mlvc_decoder_standin, synthetic_yuv420
from oracle.ref_backend import RefCpuBackend, ref_tensor_to_yuv

pytestmark = pytest.mark.gpu

WIDTH, HEIGHT, MODEL_W, MODEL_H = 640, 360, 640, 368
FRAMES = 32
PART = "MLVCDecoder"


def psnr(a, b):
    mse = float(np.mean((a.astype(np.float64) - b.astype(np.float64)) ** 2))
    return 999.9 if mse == 0 else 10.0 * np.log10(255.0 ** 2 / mse)


@pytest.fixture(scope="module")
def standin(tmp_path_factory):
    gb, inputs = build_mlvc_decoder_standin(seed=7, width=MODEL_W, height=MODEL_H)
    graph, weights = gb.finish()
    root = tmp_path_factory.mktemp("gop")
    part = root / "aot" / PART
    part.mkdir(parents=True)
    (part / "graph.pb").write_bytes(graph)
    (part / "weights.bin").write_bytes(weights)
    return root, inputs


def frame_latents(shapes, frame):
    rng = np.random.default_rng(1000 + frame)
    return [np.rint(rng.standard_normal(s) * scale).astype(np.float16) for s, scale in zip(shapes, (4, 3, 3))]


@pytest.mark.parametrize("q", [0, 21, 51])
def test_decoder_gop_matches_reference(q, standin):
    root, inputs = standin
    shapes = [inputs[k].shape for k in range(3)]
    be = Backend(0)
    be.load(root, PART, [(3, 1)])
    be.reset_state()
    be.configure_codec_io(WIDTH, HEIGHT, MODEL_W, MODEL_H, 1.0, slots=2, output_index=0)
    ref = RefCpuBackend(root, PART, 0, state_bindings=[(3, 1, list(inputs[3].shape))])
    qv = np.array([q], np.int32)
    in_flight = {}
    report = []

    def check(slot):
        frame, want = in_flight.pop(slot)
        got = np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(slot)])
        src = np.concatenate([p.reshape(-1) for p in synthetic_yuv420(frame, WIDTH, HEIGHT)])
        err = int(np.abs(got.astype(np.int32) - want.astype(np.int32)).max())
        p_ref, p_gpu, p_pair = psnr(src, want), psnr(src, got), psnr(got, want)
        report.append((frame, err, p_pair, p_gpu - p_ref))
        assert err <= 1, f"q {q} frame {frame}: max YUV error {err}"
        assert p_pair >= 60.0, f"q {q} frame {frame}: PSNR against the reference {p_pair:.2f} dB"
        assert abs(p_gpu - p_ref) <= 0.01, f"q {q} frame {frame}: PSNR {p_gpu:.4f} vs reference {p_ref:.4f} dB"

    for frame in range(FRAMES):
        slot = frame % 2
        if slot in in_flight:
            be.wait_slot(slot)
            check(slot)
        lat = frame_latents(shapes, frame)
        for k, a in enumerate(lat):
            be.slot_input(slot, k)[...] = a
        be.submit(slot, shifted_q=q)
        (x_ref,) = ref.run(lat + [qv])
        in_flight[slot] = (frame, ref_tensor_to_yuv(x_ref, WIDTH, HEIGHT))
    for slot in sorted(in_flight, key=lambda s: in_flight[s][0]):
        be.wait_slot(slot)
        check(slot)
    assert len(report) == FRAMES
    # a new GOP: the I-frame after reset_state reproduces the first frame
    first = report[0]
    be.reset_state()
    be.slot_input(0, 0)[...], be.slot_input(0, 1)[...], be.slot_input(0, 2)[...] = frame_latents(shapes, 0)
    be.submit(0, shifted_q=q)
    be.wait_slot(0)
    ref.reset_state()
    (x_ref,) = ref.run(frame_latents(shapes, 0) + [qv])
    again = np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(0)])
    assert int(np.abs(again.astype(np.int32) - ref_tensor_to_yuv(x_ref, WIDTH, HEIGHT).astype(np.int32)).max()) <= 1
    print(f"q {q}: worst frame error {max(r[1] for r in report)}, min PSNR vs reference "
          f"{min(r[2] for r in report):.2f} dB, max |dPSNR| {max(abs(r[3]) for r in report):.4f} dB; first {first}")
    be.close()
    ref.close()


def test_submit_with_q_matches_run(standin):
    """submit(slot, shifted_q) (the reference's submit_decoder(slot, shifted_q),
    set_q_index at backends/driver_cubin/src/cuda_graph_executor.cpp:66-82)
    gives the same decoded tensor as run() with that q input, for q 0, 21, 51,
    and the q value changes the result (it selects the dequantisation row)."""
    root, inputs = standin
    lat = [inputs[0], inputs[1], inputs[2]]
    be = Backend(0)
    be.load(root, PART, [(3, 1)])
    be.configure_slots(2)
    outs = {}
    for q in (0, 21, 51):
        be.reset_state()
        x_run, = be.run(lat + [np.array([q], np.int32)])
        be.reset_state()
        for k, a in enumerate(lat):
            be.slot_input(1, k)[...] = a
        be.slot_input(1, 3)[...] = -7  # overwritten by submit(slot, shifted_q)
        be.submit(1, shifted_q=q)
        be.wait_slot(1)
        x_slot = be.slot_output(1, 0)
        assert np.array_equal(x_slot.view(np.uint16), x_run.view(np.uint16)), q
        outs[q] = x_run
    assert not np.array_equal(outs[0], outs[51])
    with pytest.raises(RuntimeError, match="q_index_shifted"):
        from mlvc_b200.graph import build_conv3x3
        gb, _ = build_conv3x3(0, channels=16, height=8, width=8)
        g, w = gb.finish()
        other = Backend(0)
        other.load_memory(g, w)
        other.configure_slots(1)
        other.submit(0, shifted_q=3)
    be.close()
