"""Python host mirror of the reference backend interface over libmlvc_b200.so.

`Backend` follows mlvc::InferenceBackend (runtime/include/mlvc/runtime/
backend.hpp:48-63): load(model_name, state bindings) -> run(inputs) ->
reset_state(), plus the slot path of BufferedCodecBackend (backend.hpp:79-96)
in tensor form.  Tensors are NCHW numpy arrays (float16 or int32), the same
contract as mlvc::Tensor.  Every call goes through the C ABI declared in
include/mlvc_b200.h; failures raise RuntimeError with the library's message.

There is no fallback: if the native library is missing or the device is not
an sm_100 GPU, construction fails.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = _PKG_ROOT / "lib" / "libmlvc_b200.so"
_lib = None


class Tensor(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("rank", ctypes.c_int32), ("shape", ctypes.c_int64 * 4),
                ("data", ctypes.c_void_p), ("bytes", ctypes.c_size_t)]


class StateBinding(ctypes.Structure):
    _fields_ = [("input_index", ctypes.c_size_t), ("output_index", ctypes.c_size_t)]


class ScaleConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "hyperprior_channels", "model_width", "model_height", "latent_channels", "downsample_latent",
        "downsample_hyperprior", "y_scale_repeat", "scale_max_index")]


EXPORTS = {
    "mlvc_b200_abi_version": ([], ctypes.c_int),
    "mlvc_b200_last_error": ([], ctypes.c_char_p),
    "mlvc_b200_create": ([ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mlvc_b200_create_offline": ([ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)], ctypes.c_int),
    "mlvc_b200_destroy": ([ctypes.c_void_p], None),
    "mlvc_b200_name": ([ctypes.c_void_p], ctypes.c_char_p),
    "mlvc_b200_load": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(StateBinding),
                        ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_load_memory": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                               ctypes.POINTER(StateBinding), ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_input_count": ([ctypes.c_void_p], ctypes.c_size_t),
    "mlvc_b200_output_count": ([ctypes.c_void_p], ctypes.c_size_t),
    "mlvc_b200_input_info": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(Tensor),
                              ctypes.POINTER(ctypes.c_char_p)], ctypes.c_int),
    "mlvc_b200_output_info": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(Tensor),
                               ctypes.POINTER(ctypes.c_char_p)], ctypes.c_int),
    "mlvc_b200_run": ([ctypes.c_void_p, ctypes.POINTER(Tensor), ctypes.c_size_t, ctypes.POINTER(Tensor),
                       ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_reset_state": ([ctypes.c_void_p], ctypes.c_int),
    "mlvc_b200_scale_shape": ([ctypes.POINTER(ScaleConfig), ctypes.POINTER(ctypes.c_size_t),
                               ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "mlvc_b200_extract_scales": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ScaleConfig),
                                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_integer_values": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p],
                                 ctypes.c_int),
    "mlvc_b200_extract_scales_device": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.POINTER(ScaleConfig),
                                         ctypes.c_uint64, ctypes.c_uint64], ctypes.c_int),
    "mlvc_b200_integer_values_device": ([ctypes.c_void_p, ctypes.c_uint64, ctypes.c_size_t, ctypes.c_uint64,
                                         ctypes.c_uint64], ctypes.c_int),
    "mlvc_b200_integer_values_noalloc": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p], ctypes.c_int),
    "mlvc_b200_configure_slots": ([ctypes.c_void_p, ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_slot_count": ([ctypes.c_void_p], ctypes.c_size_t),
    "mlvc_b200_slot_input": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t], ctypes.c_void_p),
    "mlvc_b200_slot_output": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t], ctypes.c_void_p),
    "mlvc_b200_configure_codec_io": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_float, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t],
                                     ctypes.c_int),
    "mlvc_b200_codec_output_fused": ([ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
    "mlvc_b200_slot_input_yuv": ([ctypes.c_void_p, ctypes.c_size_t] + [ctypes.POINTER(ctypes.c_void_p)] * 3,
                                 ctypes.c_int),
    "mlvc_b200_slot_output_yuv": ([ctypes.c_void_p, ctypes.c_size_t] + [ctypes.POINTER(ctypes.c_void_p)] * 3,
                                  ctypes.c_int),
    "mlvc_b200_submit": ([ctypes.c_void_p, ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_submit_q": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32], ctypes.c_int),
    "mlvc_b200_wait_slot": ([ctypes.c_void_p, ctypes.c_size_t], ctypes.c_int),
    "mlvc_b200_enqueue": ([ctypes.c_void_p], ctypes.c_int),
    "mlvc_b200_synchronize": ([ctypes.c_void_p], ctypes.c_int),
    "mlvc_b200_stream": ([ctypes.c_void_p], ctypes.c_void_p),
    "mlvc_b200_step_count": ([ctypes.c_void_p], ctypes.c_size_t),
    "mlvc_b200_step_info": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_char_p),
                             ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(ctypes.c_double),
                             ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint32),
                             ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "mlvc_b200_time_steps": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(ctypes.c_float)],
                             ctypes.c_int),
    "mlvc_b200_trace_spans": ([ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(ctypes.c_float)],
                              ctypes.c_int),
    "mlvc_b200_kernel_launches": ([ctypes.c_void_p], ctypes.c_int),
    "mlvc_b200_device_bytes": ([ctypes.c_void_p], ctypes.c_size_t),
    "mlvc_b200_trace_step": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), ctypes.c_size_t,
                              ctypes.POINTER(ctypes.c_size_t)], ctypes.c_int),
    "mlvc_b200_test_wait_expiry": ([ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint64,
                                    ctypes.POINTER(ctypes.c_uint32)], ctypes.c_int),
    "mlvc_b200_set_debug_tensors": ([ctypes.c_void_p, ctypes.c_int], ctypes.c_int),
    "mlvc_b200_read_tensor": ([ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_size_t,
                               ctypes.POINTER(ctypes.c_int)], ctypes.c_int),
}


def lib():
    """Loads the in-tree native library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"mlvc-b200 native library not built: {LIB_PATH} (run python mlvc.cpp_b200/build.py)")
        l = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in EXPORTS.items():
            f = getattr(l, name)
            f.argtypes = args
            f.restype = res
        _lib = l
    return _lib


def _check(rc):
    if rc != 0:
        raise RuntimeError(lib().mlvc_b200_last_error().decode())


def _np_dtype(code):
    return np.float16 if code == 0 else np.int32


class Backend:
    """One B200 backend instance bound to one device (BackendOptions::device_id)."""

    def __init__(self, device_id: int = 0, plan_only_for=None, debug_tensors=False):
        """plan_only_for=(sm_count, smem_optin_bytes) creates a planning-only
        instance that never touches a GPU (mlvc_b200_create_offline).
        debug_tensors keeps every intermediate readable with read_tensor()."""
        self._h = ctypes.c_void_p()
        if plan_only_for is None:
            _check(lib().mlvc_b200_create(device_id, ctypes.byref(self._h)))
        else:
            _check(lib().mlvc_b200_create_offline(int(plan_only_for[0]), int(plan_only_for[1]), ctypes.byref(self._h)))
        if debug_tensors:
            _check(lib().mlvc_b200_set_debug_tensors(self._h, 1))
        self._in, self._out = [], []

    def close(self):
        if self._h:
            lib().mlvc_b200_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def name(self):
        return lib().mlvc_b200_name(self._h).decode()

    # ------------------------------------------------------------ load
    def load(self, model_dir, model_name, state_bindings=()):
        b = (StateBinding * max(1, len(state_bindings)))(*[StateBinding(i, o) for i, o in state_bindings])
        _check(lib().mlvc_b200_load(self._h, str(model_dir).encode(), model_name.encode(), b, len(state_bindings)))
        self._describe()

    def load_memory(self, graph_pb: bytes, weights: bytes, state_bindings=()):
        b = (StateBinding * max(1, len(state_bindings)))(*[StateBinding(i, o) for i, o in state_bindings])
        g = ctypes.create_string_buffer(graph_pb, len(graph_pb))
        w = ctypes.create_string_buffer(weights, max(1, len(weights)))
        _check(lib().mlvc_b200_load_memory(self._h, g, len(graph_pb), w, len(weights), b, len(state_bindings)))
        self._describe()

    def _describe(self):
        L = lib()
        self._in, self._out = [], []
        for count, info, dst in ((L.mlvc_b200_input_count, L.mlvc_b200_input_info, self._in),
                                 (L.mlvc_b200_output_count, L.mlvc_b200_output_info, self._out)):
            for i in range(count(self._h)):
                t, name = Tensor(), ctypes.c_char_p()
                _check(info(self._h, i, ctypes.byref(t), ctypes.byref(name)))
                dst.append((name.value.decode(), _np_dtype(t.dtype), tuple(t.shape[:t.rank])))

    @property
    def inputs(self):
        return list(self._in)

    @property
    def outputs(self):
        return list(self._out)

    # ------------------------------------------------------------- run
    def run(self, inputs):
        if len(inputs) != len(self._in):
            raise RuntimeError("mlvc-b200: graph input count mismatch")
        keep = []
        tin = (Tensor * max(1, len(inputs)))()
        for k, (arr, (_, dt, shape)) in enumerate(zip(inputs, self._in)):
            a = np.ascontiguousarray(arr)
            keep.append(a)
            tin[k].dtype = 0 if a.dtype == np.float16 else 1 if a.dtype == np.int32 else -1
            tin[k].rank = a.ndim
            for r in range(a.ndim):
                tin[k].shape[r] = a.shape[r]
            tin[k].data = a.ctypes.data
            tin[k].bytes = a.nbytes
        outs = [np.empty(shape, dt) for _, dt, shape in self._out]
        tout = (Tensor * max(1, len(outs)))()
        for k, o in enumerate(outs):
            tout[k].data = o.ctypes.data
            tout[k].bytes = o.nbytes
        _check(lib().mlvc_b200_run(self._h, tin, len(inputs), tout, len(outs)))
        return outs

    def reset_state(self):
        _check(lib().mlvc_b200_reset_state(self._h))

    # --------------------------------------------- entropy-coder inputs
    def extract_scales(self, z_raw, model_width, model_height, latent_channels, downsample_latent=16,
                       downsample_hyperprior=8, y_scale_repeat=2, scale_max_index=127):
        """mlvc::extract_scales (core/src/scales.cpp:25-105) on the GPU:
        z_raw float16 [1, hyper, zh, zw] -> (scales_0, scales_1) int32
        [latent / 2, yh, yw].  Needs no loaded graph."""
        z = np.ascontiguousarray(z_raw, np.float16)
        cfg = ScaleConfig(int(z.shape[1]) if z.ndim == 4 else 0, model_width, model_height, latent_channels,
                          downsample_latent, downsample_hyperprior, y_scale_repeat, scale_max_index)
        zc, sc = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib().mlvc_b200_scale_shape(ctypes.byref(cfg), ctypes.byref(zc), ctypes.byref(sc)))
        yh = -(-model_height // downsample_latent)
        yw = -(-model_width // downsample_latent)
        s0 = np.empty((latent_channels // 2, yh, yw), np.int32)
        s1 = np.empty_like(s0)
        _check(lib().mlvc_b200_extract_scales(self._h, z.ctypes.data, z.size, ctypes.byref(cfg), s0.ctypes.data,
                                              s1.ctypes.data, s0.size))
        return s0, s1

    def integer_values(self, values):
        """mlvc::integer_values (core/src/entropy.cpp:201-226) on the GPU:
        float16 values -> int32 symbols by truncation (same shape); raises
        RuntimeError when a value is not finite or outside [-32768, 32767]."""
        v = np.ascontiguousarray(values, np.float16)
        out = np.empty(v.shape, np.int32)
        _check(lib().mlvc_b200_integer_values(self._h, v.ctypes.data, v.size, out.ctypes.data))
        return out

    def extract_scales_device(self, z_ptr, hyperprior_channels, model_width, model_height, latent_channels,
                              scales_0_ptr, scales_1_ptr, downsample_latent=16, downsample_hyperprior=8,
                              y_scale_repeat=2, scale_max_index=127):
        """Device-pointer form of extract_scales (enqueued on self.stream, no
        wait): z_ptr -> FP16 [hyper, zh, zw], scales_*_ptr -> int32 planes."""
        cfg = ScaleConfig(hyperprior_channels, model_width, model_height, latent_channels, downsample_latent,
                          downsample_hyperprior, y_scale_repeat, scale_max_index)
        _check(lib().mlvc_b200_extract_scales_device(self._h, z_ptr, ctypes.byref(cfg), scales_0_ptr, scales_1_ptr))

    def integer_values_device(self, values_ptr, count, symbols_ptr, out_of_range_ptr):
        """Device-pointer form of integer_values (enqueued on self.stream, no
        wait); the device uint32 at out_of_range_ptr, zeroed by the caller,
        becomes non-zero when a value is out of range."""
        _check(lib().mlvc_b200_integer_values_device(self._h, values_ptr, count, symbols_ptr, out_of_range_ptr))

    # ----------------------------------------------------------- slots
    def configure_slots(self, n):
        _check(lib().mlvc_b200_configure_slots(self._h, n))

    def slot_input(self, slot, i):
        """numpy view of the pinned host buffer of input i in `slot`."""
        ptr = lib().mlvc_b200_slot_input(self._h, slot, i)
        if not ptr:
            raise RuntimeError(lib().mlvc_b200_last_error().decode())
        _, dt, shape = self._in[i]
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        return np.frombuffer((ctypes.c_char * n).from_address(ptr), dt).reshape(shape)

    def slot_output(self, slot, i):
        ptr = lib().mlvc_b200_slot_output(self._h, slot, i)
        if not ptr:
            raise RuntimeError(lib().mlvc_b200_last_error().decode())
        _, dt, shape = self._out[i]
        n = int(np.prod(shape)) * np.dtype(dt).itemsize
        return np.frombuffer((ctypes.c_char * n).from_address(ptr), dt).reshape(shape)

    NO_CODEC_TENSOR = ctypes.c_size_t(-1).value

    def configure_codec_io(self, width, height, model_width, model_height, pixel_range=1.0, slots=2,
                           input_index=None, output_index=None):
        """BufferedCodecBackend::configure_codec_io: graph input `input_index`
        takes a YUV420 frame per slot, output `output_index` returns one (None:
        that side stays a tensor)."""
        none = self.NO_CODEC_TENSOR
        _check(lib().mlvc_b200_configure_codec_io(
            self._h, width, height, model_width, model_height, pixel_range, slots,
            none if input_index is None else input_index, none if output_index is None else output_index))
        self._yuv = (width, height)

    def _planes(self, fn, slot):
        ptrs = [ctypes.c_void_p() for _ in range(3)]
        _check(fn(self._h, slot, *[ctypes.byref(q) for q in ptrs]))
        w, h = self._yuv
        sizes = (w * h, w * h // 4, w * h // 4)
        shapes = ((h, w), (h // 2, w // 2), (h // 2, w // 2))
        return tuple(np.frombuffer((ctypes.c_char * n).from_address(q.value), np.uint8).reshape(s)
                     for q, n, s in zip(ptrs, sizes, shapes))

    def codec_output_fused(self):
        """True when the slot graphs convert the decoded frame to YUV420 straight
        from the NHWC tensor of the x8 output pixel shuffle."""
        v = ctypes.c_int()
        _check(lib().mlvc_b200_codec_output_fused(self._h, ctypes.byref(v)))
        return bool(v.value)

    def slot_input_yuv(self, slot):
        """(Y, U, V) numpy views of the slot's pinned YUV420 input frame."""
        return self._planes(lib().mlvc_b200_slot_input_yuv, slot)

    def slot_output_yuv(self, slot):
        """(Y, U, V) numpy views of the slot's decoded YUV420 frame."""
        return self._planes(lib().mlvc_b200_slot_output_yuv, slot)

    def submit(self, slot, shifted_q=None):
        """submit(slot), or with shifted_q the reference's submit_encoder /
        submit_decoder(slot, shifted_q): the q_index_shifted input of the slot
        is set to shifted_q first."""
        if shifted_q is None:
            _check(lib().mlvc_b200_submit(self._h, slot))
        else:
            _check(lib().mlvc_b200_submit_q(self._h, slot, int(shifted_q)))

    def wait_slot(self, slot):
        _check(lib().mlvc_b200_wait_slot(self._h, slot))

    # ----------------------------------------------------- measurement
    def enqueue(self):
        _check(lib().mlvc_b200_enqueue(self._h))

    def synchronize(self):
        _check(lib().mlvc_b200_synchronize(self._h))

    @property
    def stream(self):
        return lib().mlvc_b200_stream(self._h)

    def steps(self):
        L = lib()
        out = []
        for i in range(L.mlvc_b200_step_count(self._h)):
            k, n = ctypes.c_char_p(), ctypes.c_char_p()
            fl, by = ctypes.c_double(), ctypes.c_double()
            g, b, s = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_uint32()
            _check(L.mlvc_b200_step_info(self._h, i, ctypes.byref(k), ctypes.byref(n), ctypes.byref(fl),
                                         ctypes.byref(by), ctypes.byref(g), ctypes.byref(b), ctypes.byref(s)))
            out.append(dict(kernel=k.value.decode(), nodes=n.value.decode(), flops=fl.value, bytes=by.value,
                            grid=g.value, block=b.value, smem=s.value))
        return out

    def time_steps(self, iterations=10, flush_bytes=0):
        """Mean ms per step, each step launched alone between CUDA events on the
        backend's stream; flush_bytes > 0 flushes L2 before every step."""
        n = lib().mlvc_b200_step_count(self._h)
        buf = (ctypes.c_float * max(1, n))()
        _check(lib().mlvc_b200_time_steps(self._h, iterations, flush_bytes, buf))
        return list(buf[:n])

    def trace_spans(self, iterations=10, flush_bytes=0):
        """Per-step device span (ms) of the tensor-core steps inside a replayed
        frame, from the kernels' own %globaltimer stamps (0 for other steps);
        see include/mlvc_b200.h."""
        n = lib().mlvc_b200_step_count(self._h)
        buf = (ctypes.c_float * max(1, n))()
        _check(lib().mlvc_b200_trace_spans(self._h, iterations, flush_bytes, buf))
        return list(buf[:n])

    def trace_step(self, index):
        """[CTAs, 64] %globaltimer stamps of one tensor-core conv or fused FFN
        step (see include/mlvc_b200.h); requires a previous run()."""
        n = ctypes.c_size_t()
        _check(lib().mlvc_b200_trace_step(self._h, index, None, 0, ctypes.byref(n)))
        buf = (ctypes.c_uint64 * n.value)()
        _check(lib().mlvc_b200_trace_step(self._h, index, buf, n.value, ctypes.byref(n)))
        return np.frombuffer(buf, np.uint64).reshape(-1, 64).copy()

    def test_wait_expiry(self, step_index, limit_ns):
        """Failure-detection test: relaunch a mlvc_conv1x1_tc step with its
        bounded waits limited to limit_ns and one activation panel withheld;
        returns the device status word the aborted launch left (see
        include/mlvc_b200.h)."""
        status = ctypes.c_uint32()
        _check(lib().mlvc_b200_test_wait_expiry(self._h, step_index, int(limit_ns), ctypes.byref(status)))
        return status.value

    @property
    def kernel_launches(self):
        return lib().mlvc_b200_kernel_launches(self._h)

    def read_tensor(self, name, shape, dtype=np.float16):
        """NCHW copy of a tensor the last run materialised, or None when it only
        exists inside a fused step."""
        out = np.empty(shape, dtype)
        found = ctypes.c_int(0)
        _check(lib().mlvc_b200_read_tensor(self._h, name.encode(), out.ctypes.data, out.nbytes, ctypes.byref(found)))
        return out if found.value else None

    @property
    def device_bytes(self):
        return lib().mlvc_b200_device_bytes(self._h)
