"""The reference-side adapter (include/mlvc_b200_adapter.hpp) on the GPU,
created through the reference's own backend registry by the name "b200" and
driven through the decoder calls of the codec's buffered path
(codec/src/pipeline.cpp decode_buffered: configure_codec_io, decoder_inputs,
submit_decoder(slot, shifted_q), wait_codec_slot, decoder_output_yuv).  It
must be recognised as a BufferedCodecBackend and decode the same frames,
bit for bit, as the product's own slot API, with q reaching the graph."""

import numpy as np
import pytest

from adapter_probe import PROBE, AdapterProbe
from mlvc_b200 import Backend
from mlvc_b200.graph import build_mlvc_decoder_standin

pytestmark = pytest.mark.gpu


def test_adapter_decodes_like_the_slot_api(tmp_path):
    if not PROBE.exists():
        pytest.fail(f"adapter probe missing: {PROBE} (make -C oracle adapter REF=<reference tree>)")
    gb, inputs = build_mlvc_decoder_standin(seed=9, width=256, height=128)
    gb.save(tmp_path, "MLVCDecoder")
    probe = AdapterProbe(tmp_path, 0)
    assert probe.buffered and probe.name == "b200"
    probe.load("MLVCDecoder", [(3, 1)])
    probe.reset_state()
    probe.configure(256, 120, 256, 128, slots=2)
    views = probe.decoder_inputs(0)
    assert [n for n, _ in views] == ["z_raw", "y_raw_0", "y_raw_1"]  # q_index_shifted is set by submit

    be = Backend(0)
    be.load(tmp_path, "MLVCDecoder", [(3, 1)])
    be.reset_state()
    be.configure_codec_io(256, 120, 256, 128, 1.0, slots=2, output_index=0)
    rng = np.random.default_rng(4)
    frames = []
    for f, q in enumerate((0, 21, 51, 21)):
        slot = f % 2
        lat = [np.rint(rng.standard_normal(inputs[k].shape) * s).astype(np.float16)
               for k, s in zip(range(3), (4, 3, 3))]
        for (name, view), a in zip(probe.decoder_inputs(slot), lat):
            view[...] = a.view(np.uint8).reshape(-1)
            be.slot_input(slot, ["z_raw", "y_raw_0", "y_raw_1"].index(name))[...] = a
        probe.submit_decoder(slot, q)
        be.submit(slot, shifted_q=q)
        probe.wait(slot)
        be.wait_slot(slot)
        got = probe.decoder_output(slot)
        want = np.concatenate([p.reshape(-1) for p in be.slot_output_yuv(slot)])
        assert np.array_equal(got, want), (f, q)
        frames.append(got)
    assert not np.array_equal(frames[0], frames[1])  # q and the carried state change the frame
    probe.close()
    be.close()
