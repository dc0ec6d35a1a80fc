"""Test infrastructure only (the checker, never the product): a numpy
restatement of the reference's YUV420 <-> model-tensor conversions of the
codec I/O path, core/src/yuv.cpp.

* frame_padding (yuv.cpp:324-337): the frame sits at the top-left of the
  model canvas; when it does not fit natively but fits transposed, it is
  stored transposed (rotated).
* prepare_model_input (yuv.cpp:339-400, with convert_luma_plane_input /
  convert_chroma_plane_input at :161-221): tensor[c, y, x] =
  lut[plane sample], lut[s] = fp16((s / 255) * pixel_range) in FP32; chroma
  is nearest (x / 2, y / 2); the last frame row / column is replicated into
  the padding (clamped coordinates).
* prepare_model_output_into (yuv.cpp:410-525): byte = round_half_even(
  clamp(v / pixel_range, 0, 1) * 255) in FP32, chroma from
  (((s00 + s01) + s10) + s11) * 0.25 of the values already divided by
  pixel_range.

Pinned against the reference's own compiled code in tests/test_cpu_oracle.py.
"""

import numpy as np


def frame_padding(width, height, model_width, model_height):
    for w, h in ((width, height), (model_width, model_height)):
        if w <= 0 or h <= 0 or w % 2 or h % 2:
            raise ValueError("YUV420 dimensions must be positive and even")
    native = width <= model_width and height <= model_height
    rotated = height <= model_width and width <= model_height
    if not native and not rotated:
        raise ValueError("input frame is larger than the model dimensions")
    return not native


def split_planes(yuv, width, height):
    ys = width * height
    y = yuv[:ys].reshape(height, width)
    u = yuv[ys:ys + ys // 4].reshape(height // 2, width // 2)
    v = yuv[ys + ys // 4:].reshape(height // 2, width // 2)
    return y, u, v


def yuv_to_tensor(yuv, width, height, model_width, model_height, pixel_range=1.0):
    rotated = frame_padding(width, height, model_width, model_height)
    y, u, v = split_planes(np.asarray(yuv, np.uint8), width, height)
    lut = ((np.arange(256, dtype=np.float32) / np.float32(255.0)) * np.float32(pixel_range)).astype(np.float16)
    active_w, active_h = (height, width) if rotated else (width, height)
    my = np.minimum(np.arange(model_height), active_h - 1)[:, None]
    mx = np.minimum(np.arange(model_width), active_w - 1)[None, :]
    sy, sx = (mx, my) if rotated else (my, mx)
    sy, sx = np.broadcast_arrays(sy, sx)
    out = np.empty((1, 3, model_height, model_width), np.float16)
    out[0, 0] = lut[y[sy, sx]]
    out[0, 1] = lut[u[sy // 2, sx // 2]]
    out[0, 2] = lut[v[sy // 2, sx // 2]]
    return out, rotated


def _quantize(v):
    v = np.clip(v, np.float32(0.0), np.float32(1.0)).astype(np.float32)
    return np.rint(v * np.float32(255.0)).astype(np.uint8)


def tensor_to_yuv(tensor, width, height, pixel_range=1.0):
    t = np.asarray(tensor, np.float16)
    model_height, model_width = t.shape[2], t.shape[3]
    rotated = frame_padding(width, height, model_width, model_height)
    f = t[0].astype(np.float32) / np.float32(pixel_range)  # [3, mh, mw], FP32 division
    if rotated:
        f = f.transpose(0, 2, 1)  # sample(c, y, x) = tensor[c, x, y]
    f = f[:, :height, :width]
    y = _quantize(f[0])
    out = [y.reshape(-1)]
    for c in (1, 2):
        p = f[c]
        s = ((p[0::2, 0::2] + p[0::2, 1::2]) + p[1::2, 0::2]) + p[1::2, 1::2]
        out.append(_quantize(s * np.float32(0.25)).reshape(-1))
    return np.concatenate(out)
