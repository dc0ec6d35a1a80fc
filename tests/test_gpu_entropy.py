"""Entropy-coder inputs on the B200, through the C ABI: scale extraction
(reference extract_scales, core/src/scales.cpp:25-105) and the FP16 ->
int32 symbol conversion (integer_values, core/src/entropy.cpp:201-226).
Both are integer work, so the results must equal the oracle bit for bit; the
oracle itself is pinned against the reference's compiled scales.cpp on the
CPU (tests/test_cpu_oracle.py)."""

import numpy as np
import pytest

from mlvc_b200 import Backend
from oracle import scales_oracle

pytestmark = pytest.mark.gpu

SCALE_CASES = [  # model_width, model_height, latent, hyper, repeat, downsample_hyperprior
    (640, 368, 128, 128, 2, 8),
    (1920, 1088, 128, 128, 2, 8),
    (1920, 1080, 128, 128, 2, 8),
    (640, 368, 48, 48, 4, 8),
    (96, 80, 64, 32, 2, 4),
    (200, 120, 96, 64, 3, 2),
    (16, 16, 2, 1, 2, 8),     # one latent pixel, one output channel
]


@pytest.fixture(scope="module")
def be():
    return Backend(0)


@pytest.mark.parametrize("mw,mh,latent,hyper,repeat,ds", SCALE_CASES)
def test_extract_scales_bit_exact(be, mw, mh, latent, hyper, repeat, ds):
    zh, zw = -(-mh // (16 * ds)), -(-mw // (16 * ds))
    yh, yw = -(-mh // 16), -(-mw // 16)
    rng = np.random.default_rng(mw * 7 + mh + latent)
    z = (rng.standard_normal((1, hyper, zh, zw)) * 60).astype(np.float16)
    edges = np.array([np.inf, -np.inf, np.nan, 65504, -0.0, 127.99, -128.0, 0.999], np.float16)
    z.flat[: min(z.size, edges.size)] = edges[: z.size]
    got0, got1 = be.extract_scales(z, mw, mh, latent, 16, ds, repeat, 127)
    want0, want1 = scales_oracle.extract_scales(z, latent, yh, yw, repeat, ds, 127)
    assert got0.shape == want0.shape == (latent // 2, yh, yw)
    assert np.array_equal(got0, want0) and np.array_equal(got1, want1)


def test_extract_scales_rejects_mismatched_z(be):
    z = np.zeros((1, 128, 3, 4), np.float16)  # 640x368 needs a 3 x 5 hyper plane
    with pytest.raises(RuntimeError, match="does not match model metadata"):
        be.extract_scales(z, 640, 368, 128)
    with pytest.raises(RuntimeError, match="channel mapping is invalid"):
        be.extract_scales(np.zeros((1, 32, 3, 5), np.float16), 640, 368, 128)


@pytest.mark.parametrize("n", [1, 7, 4096, 64 * 68 * 120 + 3])
def test_integer_values_bit_exact(be, n):
    rng = np.random.default_rng(n)
    v = np.clip(rng.standard_normal(n) * np.float32(3000), -32768, 32752).astype(np.float16)
    v[: min(n, 6)] = np.array([-1.5, 1.5, -0.0, -32768, 32752, 0.75], np.float16)[: min(n, 6)]
    got = be.integer_values(v)
    assert got.dtype == np.int32 and got.shape == v.shape
    assert np.array_equal(got, scales_oracle.integer_values(v))


def test_integer_values_all_finite_in_range_halves(be):
    """Every FP16 bit pattern inside [-32768, 32767] converts like the oracle."""
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    v = bits.view(np.float16)
    f = v.astype(np.float32)
    v = v[np.isfinite(f) & (f >= -32768) & (f <= 32767)]
    assert np.array_equal(be.integer_values(v), scales_oracle.integer_values(v))


@pytest.mark.parametrize("bad", [np.inf, -np.inf, np.nan, 32768, -32800])
def test_integer_values_out_of_range_raises(be, bad):
    v = np.zeros(1000, np.float16)
    v[517] = bad
    with pytest.raises(RuntimeError, match="entropy symbol is outside signed 16-bit range"):
        be.integer_values(v)
    # the backend stays usable after the error
    assert be.integer_values(np.array([3.5, -2.5], np.float16)).tolist() == [3, -2]


def test_integer_values_empty(be):
    assert be.integer_values(np.zeros(0, np.float16)).shape == (0,)


def test_device_forms_match_host_forms(be):
    """The device-pointer entry points (buffers from another allocator, here
    torch) give the same symbols and scales as the host-buffer calls, and
    report out-of-range values through the caller's device flag."""
    import torch
    rng = np.random.default_rng(11)
    z = (rng.standard_normal((1, 128, 3, 5)) * 50).astype(np.float16)
    y = np.rint(rng.standard_normal((1, 64, 23, 40)) * 300).astype(np.float16)
    dev = torch.device("cuda:0")
    zt, yt = torch.from_numpy(z).to(dev), torch.from_numpy(y).to(dev)
    s0 = torch.empty((64, 23, 40), dtype=torch.int32, device=dev)
    s1 = torch.empty_like(s0)
    sym = torch.empty(y.shape, dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    be.extract_scales_device(zt.data_ptr(), 128, 640, 368, 128, s0.data_ptr(), s1.data_ptr())
    be.integer_values_device(yt.data_ptr(), y.size, sym.data_ptr(), flag.data_ptr())
    torch.cuda.synchronize()
    want0, want1 = be.extract_scales(z, 640, 368, 128)
    assert np.array_equal(s0.cpu().numpy(), want0) and np.array_equal(s1.cpu().numpy(), want1)
    assert np.array_equal(sym.cpu().numpy(), be.integer_values(y)) and int(flag.item()) == 0
    yt[0, 3, 4, 5] = float("inf")
    torch.cuda.synchronize()
    be.integer_values_device(yt.data_ptr(), y.size, sym.data_ptr(), flag.data_ptr())
    torch.cuda.synchronize()
    assert int(flag.item()) != 0
