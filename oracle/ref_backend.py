"""ctypes driver for the reference's own CPU backend (oracle/_ref/libmlvc_ref_cpu.so).

TEST INFRASTRUCTURE ONLY: the checker in tests/ and the timed reference arm
and CPU baseline of bench.py.  The library is the reference's backends/cpu
sources compiled unchanged (oracle/Makefile) plus ref_shim/, driven through
the reference InferenceBackend contract (runtime/include/mlvc/runtime/
backend.hpp:48-63): create -> load -> reset_state -> run.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_ref" / "libmlvc_ref_cpu.so"
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"reference CPU backend not built: {LIB_PATH} (make -C oracle ref)")
        L = ctypes.CDLL(str(LIB_PATH))
        vp, cp, sz = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t
        L.mlvc_ref_create.restype = vp
        L.mlvc_ref_create.argtypes = [cp, ctypes.c_int, cp, sz]
        L.mlvc_ref_load.argtypes = [vp, cp, ctypes.c_int, vp, vp, vp, cp, sz]
        L.mlvc_ref_reset_state.argtypes = [vp, cp, sz]
        L.mlvc_ref_run.argtypes = [vp, ctypes.c_int, vp, vp, vp, vp, cp, sz]
        L.mlvc_ref_output_count.argtypes = [vp]
        L.mlvc_ref_output_info.restype = ctypes.c_int64
        L.mlvc_ref_output_info.argtypes = [vp, ctypes.c_int, vp, vp, vp]
        L.mlvc_ref_output_copy.argtypes = [vp, ctypes.c_int, vp, sz]
        L.mlvc_ref_destroy.argtypes = [vp]
        L.mlvc_ref_yuv_to_tensor.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_float, vp, vp, cp, sz]
        L.mlvc_ref_tensor_to_yuv.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_float, vp, cp, sz]
        L.mlvc_ref_extract_scales.argtypes = [vp] + [ctypes.c_int] * 8 + [vp, vp, cp, sz]
        _lib = L
    return _lib


class RefCpuBackend:
    def __init__(self, model_dir, part, threads=0, state_bindings=()):
        L = lib()
        err = ctypes.create_string_buffer(1024)
        self._h = L.mlvc_ref_create(str(model_dir).encode(), int(threads), err, 1024)
        if not self._h:
            raise RuntimeError(err.value.decode())
        n = len(state_bindings)
        si = (ctypes.c_uint64 * max(1, n))(*[b[0] for b in state_bindings])
        so = (ctypes.c_uint64 * max(1, n))(*[b[1] for b in state_bindings])
        shapes = (ctypes.c_int64 * max(4, 4 * n))(*[d for b in state_bindings for d in b[2]])
        if L.mlvc_ref_load(self._h, part.encode(), n, si, so, shapes, err, 1024) != 0:
            raise RuntimeError(err.value.decode())
        if n and L.mlvc_ref_reset_state(self._h, err, 1024) != 0:
            raise RuntimeError(err.value.decode())

    def run(self, inputs):
        L = lib()
        arrs = [np.ascontiguousarray(a) for a in inputs]
        n = len(arrs)
        data = (ctypes.c_void_p * max(1, n))(*[a.ctypes.data for a in arrs])
        dts = (ctypes.c_int * max(1, n))(*[0 if a.dtype == np.float16 else 1 for a in arrs])
        ranks = (ctypes.c_int * max(1, n))(*[a.ndim for a in arrs])
        flat = [d for a in arrs for d in a.shape]
        shapes = (ctypes.c_int64 * max(1, len(flat)))(*flat)
        err = ctypes.create_string_buffer(1024)
        if L.mlvc_ref_run(self._h, n, data, dts, ranks, shapes, err, 1024) != 0:
            raise RuntimeError(err.value.decode())
        outs = []
        for i in range(L.mlvc_ref_output_count(self._h)):
            dt, rk, s4 = ctypes.c_int(), ctypes.c_int(), (ctypes.c_int64 * 4)()
            nb = L.mlvc_ref_output_info(self._h, i, ctypes.byref(dt), ctypes.byref(rk), s4)
            o = np.empty(tuple(s4[:rk.value]), np.float16 if dt.value == 0 else np.int32)
            L.mlvc_ref_output_copy(self._h, i, o.ctypes.data, nb)
            outs.append(o)
        return outs

    def reset_state(self):
        """InferenceBackend::reset_state(): zeroes every bound state (a new GOP)."""
        err = ctypes.create_string_buffer(1024)
        if lib().mlvc_ref_reset_state(self._h, err, 1024) != 0:
            raise RuntimeError(err.value.decode())

    def close(self):
        if self._h:
            lib().mlvc_ref_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_yuv_to_tensor(yuv, width, height, model_width, model_height, pixel_range=1.0):
    """The reference's prepare_model_input (core/src/yuv.cpp:339-400) on a
    planar YUV420 byte frame: returns ([1, 3, mh, mw] float16, rotated)."""
    import numpy as np
    yuv = np.ascontiguousarray(yuv, np.uint8)
    out = np.empty((1, 3, model_height, model_width), np.float16)
    rot = ctypes.c_int(0)
    err = ctypes.create_string_buffer(512)
    if lib().mlvc_ref_yuv_to_tensor(yuv.ctypes.data, width, height, model_width, model_height, pixel_range,
                                    out.ctypes.data, ctypes.byref(rot), err, 512):
        raise RuntimeError(err.value.decode())
    return out, bool(rot.value)


def ref_tensor_to_yuv(tensor, width, height, pixel_range=1.0):
    """The reference's prepare_model_output_into (core/src/yuv.cpp:410-525):
    [1, 3, mh, mw] float16 -> planar YUV420 bytes of a width x height frame."""
    import numpy as np
    t = np.ascontiguousarray(tensor, np.float16)
    mh, mw = t.shape[2], t.shape[3]
    out = np.empty(width * height * 3 // 2, np.uint8)
    err = ctypes.create_string_buffer(512)
    if lib().mlvc_ref_tensor_to_yuv(t.ctypes.data, mw, mh, width, height, pixel_range, out.ctypes.data, err, 512):
        raise RuntimeError(err.value.decode())
    return out


def ref_extract_scales(z_raw, model_width, model_height, latent_channels, downsample_latent=16,
                       downsample_hyperprior=8, y_scale_repeat=2, scale_max_index=127):
    """The reference's extract_scales (core/src/scales.cpp:25-105) on a
    [1, hyper, zh, zw] float16 z_raw: returns (scales_0, scales_1), int32
    [latent / 2, yh, yw] each."""
    import numpy as np
    z = np.ascontiguousarray(z_raw, np.float16)
    yh = -(-model_height // downsample_latent)
    yw = -(-model_width // downsample_latent)
    s0 = np.empty((latent_channels // 2, yh, yw), np.int32)
    s1 = np.empty_like(s0)
    err = ctypes.create_string_buffer(512)
    if lib().mlvc_ref_extract_scales(z.ctypes.data, z.shape[1], model_width, model_height, latent_channels,
                                     downsample_latent, downsample_hyperprior, y_scale_repeat, scale_max_index,
                                     s0.ctypes.data, s1.ctypes.data, err, 512):
        raise RuntimeError(err.value.decode())
    return s0, s1
