"""Helpers around the public C ABI (include/depth_anything_v2.h)."""
import ctypes

import numpy as np

from dav2_b200 import capi


def create(lib, path, encoder="vits", flags=0, device=0):
    opts = capi.CreateOptions(ctypes.sizeof(capi.CreateOptions), capi.ABI_VERSION, capi.ENCODERS[encoder], device,
                              flags, None)
    ctx = ctypes.c_void_p()
    rc = lib.dav2_create(str(path).encode(), ctypes.byref(opts), ctypes.byref(ctx))
    return rc, ctx


def infer_tensor(lib, ctx, image):
    image = np.ascontiguousarray(image, np.float32)
    c, h, w = image.shape
    out = np.zeros((h, w), np.float32)
    rc = lib.dav2_infer_tensor_f32(ctx, image.ctypes.data, w, h, out.ctypes.data, out.size)
    assert rc == 0, lib.dav2_last_error()
    return out


def infer_tensor_batch(lib, ctx, images):
    images = np.ascontiguousarray(images, np.float32)
    b, c, h, w = images.shape
    out = np.zeros((b, h, w), np.float32)
    rc = lib.dav2_infer_tensor_f32_batch(ctx, images.ctypes.data, b, w, h, out.ctypes.data, out.size)
    assert rc == 0, lib.dav2_last_error()
    return out


def infer_bgr8(lib, ctx, bgr, input_size=518):
    bgr = np.ascontiguousarray(bgr, np.uint8)
    h, w = bgr.shape[:2]
    out = np.zeros((h, w), np.float32)
    rc = lib.dav2_infer_bgr8(ctx, bgr.ctypes.data, w, h, w * 3, input_size, out.ctypes.data, out.size)
    assert rc == 0, lib.dav2_last_error()
    return out
