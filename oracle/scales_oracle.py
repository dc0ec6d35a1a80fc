"""Test infrastructure only (the checker, never the product): numpy
restatements of the two integer steps between the decoder graph and the
entropy coder.

* extract_scales (core/src/scales.cpp:25-105): base scale of hyper-latent
  channel b < latent / y_scale_repeat at z position (zy, zx) =
  clamp(trunc(|z|), 0, scale_max_index) for finite z.  For a non-finite z the
  reference's int cast is undefined; its compiled code (gcc -O3, x86) yields
  INT_MIN there (the truncating conversion gives INT_MIN and the compiler
  drops the lower clamp of a cast |x|), which is what this restatement and the
  GPU kernel reproduce.  Output channel c < latent / 2 at
  latent pixel (y, x) takes base channels c / y_scale_repeat ("first") and
  (c + latent / 2) / y_scale_repeat ("second") at (min(y / s, zh - 1),
  min(x / s, zw - 1)), s = downsample_hyperprior; scales_0 = first where
  (x + y) is even, else second; scales_1 the other one.
* integer_values (core/src/entropy.cpp:201-226): FP16 latents -> int32
  entropy symbols by truncation; a non-finite value or one outside
  [-32768, 32767] is an error ("entropy symbol is outside signed 16-bit
  range").  The reference function cannot be compiled here (entropy.cpp needs
  the absent msrtc_rans coder), so this restatement is pinned by the
  reference's stated semantics and the tests' edge cases.

extract_scales is pinned against the reference's own compiled code in
tests/test_cpu_oracle.py.
"""

import numpy as np

INT_MIN = np.int32(-2147483648)


def extract_scales(z_raw, latent_channels, y_height, y_width, y_scale_repeat=2, spatial_repeat=8,
                   scale_max_index=127):
    z = np.asarray(z_raw, np.float16)[0]  # [hyper, zh, zw]
    hyper, zh, zw = z.shape
    base_channels = latent_channels // y_scale_repeat
    if base_channels > hyper:
        raise ValueError("scale decoder channel mapping is invalid")
    a = np.abs(z[:base_channels].astype(np.float32))
    finite = np.isfinite(a)
    base = np.full(a.shape, INT_MIN, np.int32)
    base[finite] = np.clip(np.trunc(a[finite]), 0, scale_max_index).astype(np.int32)
    half = latent_channels // 2
    c = np.arange(half)[:, None, None]
    y = np.arange(y_height)[None, :, None]
    x = np.arange(y_width)[None, None, :]
    zy = np.minimum(y // spatial_repeat, zh - 1)
    zx = np.minimum(x // spatial_repeat, zw - 1)
    first = base[c // y_scale_repeat, zy, zx]
    second = base[(c + half) // y_scale_repeat, zy, zx]
    even = ((x + y) & 1) == 0
    s0 = np.where(even, first, second).astype(np.int32)
    s1 = np.where(even, second, first).astype(np.int32)
    return s0, s1


def integer_values(values):
    v = np.asarray(values, np.float16).astype(np.float32).reshape(-1)
    if not (np.isfinite(v) & (v >= -32768.0) & (v <= 32767.0)).all():
        raise ValueError("entropy symbol is outside signed 16-bit range")
    return np.trunc(v).astype(np.int32)
