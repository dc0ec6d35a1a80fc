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
