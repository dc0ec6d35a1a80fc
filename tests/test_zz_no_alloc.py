"""mlvc_b200_integer_values_noalloc: the FP16 -> int32 symbol conversion for
callers that cannot allocate device memory (a device allocation stalls the
whole GPU, which a real-time encoder loop cannot afford, and a process whose
device memory belongs to another framework's pool must not allocate behind
its back).  It works out of a fixed array inside the library, so it must give
the same symbols as the allocating entry point mlvc_b200_integer_values,
call after call, and it must start every call from a cleared out-of-range
word.  This file is collected last on purpose: a run that stops at the first
failure has run every other test before it."""

import ctypes

import numpy as np
import pytest

import mlvc_b200
from mlvc_b200 import Backend

MAX_VALUES = 1 << 21


def noalloc(values):
    v = np.ascontiguousarray(values, np.float16)
    out = np.empty(v.shape, np.int32)
    rc = mlvc_b200.lib().mlvc_b200_integer_values_noalloc(v.ctypes.data, v.size, out.ctypes.data)
    if rc != 0:
        raise RuntimeError(mlvc_b200.lib().mlvc_b200_last_error().decode())
    return out


def test_noalloc_rejects_calls_above_its_limit():
    """The size check comes before any device work (no GPU needed)."""
    lib = mlvc_b200.lib()
    rc = lib.mlvc_b200_integer_values_noalloc(ctypes.c_void_p(16), MAX_VALUES + 1, ctypes.c_void_p(16))
    assert rc != 0
    assert "at most 2097152 values" in lib.mlvc_b200_last_error().decode()


@pytest.mark.gpu
def test_noalloc_matches_allocating_entry_point():
    be = Backend(0)
    rng = np.random.default_rng(7)
    # two calls in a row with different sizes (vector body + ragged tail), then the limit itself
    first = np.rint(rng.standard_normal((1, 64, 68, 120)) * 300).astype(np.float16)
    second = np.clip(rng.standard_normal(4099) * 9000, -32768, 32752).astype(np.float16)
    for values in (first, second):
        got = noalloc(values)
        assert np.array_equal(got, be.integer_values(values))
    full = np.clip(rng.standard_normal(MAX_VALUES) * 20000, -32768, 32752).astype(np.float16)
    assert np.array_equal(noalloc(full), be.integer_values(full))


@pytest.mark.gpu
def test_noalloc_clears_its_out_of_range_word():
    """A failing call leaves the shared out-of-range word set; the next call
    must clear it before it runs."""
    be = Backend(0)
    bad = np.zeros(1000, np.float16)
    bad[517] = np.inf
    with pytest.raises(RuntimeError, match="entropy symbol is outside signed 16-bit range"):
        noalloc(bad)
    good = np.array([3.5, -2.5, 32752, -32768, 0.25], np.float16)
    assert noalloc(good).tolist() == be.integer_values(good).tolist() == [3, -2, 32752, -32768, 0]


@pytest.mark.gpu
def test_noalloc_matches_the_oracle_restatement():
    """Independently of the GPU's allocating path: the numpy restatement of the
    reference's integer_values (core/src/entropy.cpp:201-226), on every
    finite FP16 value inside [-32768, 32767] and on the same values shuffled."""
    from oracle import scales_oracle
    bits = np.arange(1 << 16, dtype=np.uint16).view(np.float16)
    f = bits.astype(np.float32)  # compared in FP32: 32767 as an FP16 scalar would round to 32768
    ok = np.isfinite(f) & (f >= -32768.0) & (f <= 32767.0)
    values = bits[ok]
    assert values.size == 61441 and 32752.0 in values and -32768.0 in values and 32768.0 not in values
    assert np.array_equal(noalloc(values), scales_oracle.integer_values(values))
    shuffled = np.random.default_rng(3).permutation(values)
    assert np.array_equal(noalloc(shuffled), scales_oracle.integer_values(shuffled))


@pytest.mark.gpu
def test_noalloc_as_the_first_device_work_of_a_process():
    """The per-device set-up runs in the first call; here that call is the
    process's first CUDA work (no backend exists yet), and a backend created
    afterwards on the same thread agrees with it."""
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    code = (
        "import sys; sys.path[:0] = [%r, %r]\n"
        "import numpy as np, mlvc_b200\n"
        "from mlvc_b200 import Backend\n"
        "v = np.rint(np.random.default_rng(5).standard_normal(70001) * 500).astype(np.float16)\n"
        "out = np.empty(v.shape, np.int32)\n"
        "assert mlvc_b200.lib().mlvc_b200_integer_values_noalloc(v.ctypes.data, v.size, out.ctypes.data) == 0\n"
        "be = Backend(0)\n"
        "assert np.array_equal(out, be.integer_values(v))\n"
        "print('ok')\n" % (str(root), str(root / "mlvc.cpp_b200")))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


@pytest.mark.gpu
def test_noalloc_on_a_second_device():
    """The set-up is per device: with device 1 current, the call uses device
    1's copy of the array.  Needs two visible GPUs."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    torch.cuda.set_device(1)  # makes device 1 current for the CUDA runtime of this thread
    try:
        v = np.rint(np.random.default_rng(6).standard_normal(9001) * 700).astype(np.float16)
        be = Backend(1)
        assert np.array_equal(noalloc(v), be.integer_values(v))
    finally:
        torch.cuda.set_device(0)
