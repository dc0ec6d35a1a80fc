"""ctypes driver of oracle/_ref/libmlvc_b200_adapter_probe.so: the product's
reference-side adapter (include/mlvc_b200_adapter.hpp) created through the
reference's own backend registry and driven through its decoder slot calls
(see oracle/ref_shim/adapter_probe.cpp)."""

import ctypes
from pathlib import Path

import numpy as np

PROBE = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libmlvc_b200_adapter_probe.so"
_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(PROBE))
        vp, cp, sz, i = ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_int
        L.probe_create.restype = vp
        L.probe_create.argtypes = [cp, i, ctypes.POINTER(i), cp, sz]
        L.probe_destroy.argtypes = [vp]
        L.probe_name.argtypes = [vp, cp, sz]
        L.probe_load.argtypes = [vp, cp, i, vp, vp, cp, sz]
        L.probe_reset_state.argtypes = [vp, cp, sz]
        L.probe_configure.argtypes = [vp, i, i, i, i, i, cp, sz]
        L.probe_decoder_input.argtypes = [vp, sz, sz, cp, sz, ctypes.POINTER(vp), ctypes.POINTER(sz), cp, sz]
        L.probe_decoder_input_count.argtypes = [vp, sz, ctypes.POINTER(sz), cp, sz]
        L.probe_submit_decoder.argtypes = [vp, sz, i, cp, sz]
        L.probe_wait.argtypes = [vp, sz, cp, sz]
        L.probe_decoder_output.argtypes = [vp, sz, vp, sz, cp, sz]
        _lib = L
    return _lib


class AdapterProbe:
    def __init__(self, model_dir, device=0):
        self._err = ctypes.create_string_buffer(1024)
        buffered = ctypes.c_int(0)
        self._h = lib().probe_create(str(model_dir).encode(), device, ctypes.byref(buffered), self._err, 1024)
        if not self._h:
            raise RuntimeError(self._err.value.decode())
        self.buffered = bool(buffered.value)

    def _ok(self, rc):
        if rc != 0:
            raise RuntimeError(self._err.value.decode())

    @property
    def name(self):
        out = ctypes.create_string_buffer(64)
        lib().probe_name(self._h, out, 64)
        return out.value.decode()

    def load(self, model, bindings=()):
        n = len(bindings)
        si = (ctypes.c_uint64 * max(1, n))(*[b[0] for b in bindings])
        so = (ctypes.c_uint64 * max(1, n))(*[b[1] for b in bindings])
        self._ok(lib().probe_load(self._h, model.encode(), n, si, so, self._err, 1024))

    def reset_state(self):
        self._ok(lib().probe_reset_state(self._h, self._err, 1024))

    def configure(self, width, height, model_width, model_height, slots=2):
        self._ok(lib().probe_configure(self._h, width, height, model_width, model_height, slots, self._err, 1024))
        self._wh = (width, height)

    def decoder_inputs(self, slot):
        """[(name, uint8 view of the slot buffer)] in the order decoder_inputs(slot) returns them."""
        count = ctypes.c_size_t()
        self._ok(lib().probe_decoder_input_count(self._h, slot, ctypes.byref(count), self._err, 1024))
        out = []
        for k in range(count.value):
            name = ctypes.create_string_buffer(256)
            data, nbytes = ctypes.c_void_p(), ctypes.c_size_t()
            self._ok(lib().probe_decoder_input(self._h, slot, k, name, 256, ctypes.byref(data), ctypes.byref(nbytes),
                                               self._err, 1024))
            buf = (ctypes.c_char * nbytes.value).from_address(data.value)
            out.append((name.value.decode(), np.frombuffer(buf, np.uint8)))
        return out

    def submit_decoder(self, slot, shifted_q):
        self._ok(lib().probe_submit_decoder(self._h, slot, shifted_q, self._err, 1024))

    def wait(self, slot):
        self._ok(lib().probe_wait(self._h, slot, self._err, 1024))

    def decoder_output(self, slot):
        w, h = self._wh
        out = np.empty(w * h * 3 // 2, np.uint8)
        self._ok(lib().probe_decoder_output(self._h, slot, out.ctypes.data, out.size, self._err, 1024))
        return out

    def close(self):
        if self._h:
            lib().probe_destroy(self._h)
            self._h = None
