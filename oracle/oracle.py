"""CPU oracle for the Depth Anything V2 tensor-operator hot path.

TEST INFRASTRUCTURE ONLY. This module wraps ``liboracle.so`` (a plain-C
restatement of the reference runtime's Vulkan shaders, see dav2_oracle.c) and
composes its operators into the reference graph (encoder: src/encoder.cpp:322-597,
DPT head: src/dpt.cpp:628-863, executor tail: src/vulkan_executor.cpp:572-636).
Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference
arm import it, as the checker. The product (libdav2_b200.so) never calls it.

Pinning: tests/test_oracle_golden.py checks every operator against the
reference's own known-answer cases (tests/vulkan_smoke.cpp, image_tests.cpp)
and against fixtures produced by the reference's Python model
(tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t
_i = ctypes.c_int
_f = ctypes.c_float

_SIGS = {
    "dav2o_crc32": (ctypes.c_uint32, [ctypes.c_void_p, _sz]),
    "dav2o_network_shape": (_i, [_i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "dav2o_preprocess_bgr8": (_i, [_u8p, _i, _i, ctypes.c_ssize_t, _i, _i, _f32p]),
    "dav2o_preprocess_inferbridge_bgra8": (_i, [_u8p, _i, _i, ctypes.c_ssize_t, _i, _i, _f32p]),
    "dav2o_preprocess_u32_bicubic": (None, [_u32p, _i, _i, _i, _i, _i, _i, _f32p]),
    "dav2o_preprocess_bgr8_bilinear": (None, [_u8p, _i, _i, ctypes.c_ssize_t, _i, _i, _f32p]),
    "dav2o_layer_norm": (None, [_f32p, _f32p, _f32p, _f32p, _sz, _i, _f]),
    "dav2o_gelu": (None, [_f32p, _f32p, _sz]),
    "dav2o_softmax_rows": (None, [_f32p, _f32p, _sz, _i, _f]),
    "dav2o_add_scaled": (None, [_f32p, _f32p, _f32p, _f32p, _sz, _i]),
    "dav2o_relu": (None, [_f32p, _f32p, _sz]),
    "dav2o_add": (None, [_f32p, _f32p, _f32p, _sz]),
    "dav2o_sigmoid_scale": (None, [_f32p, _f32p, _sz, _f]),
    "dav2o_bilinear_align_true": (None, [_f32p, _i, _i, _i, _i, _i, _f32p]),
    "dav2o_bilinear_half_pixel": (None, [_f32p, _i, _i, _i, _i, _i, _f32p]),
    "dav2o_reduce_minmax": (None, [_f32p, _sz, _f32p]),
    "dav2o_normalize_relative": (None, [_f32p, _sz, _f32p]),
    "dav2o_normalize_metric": (None, [_f32p, _sz, _f32p, _f]),
    "dav2o_quantize_rows_s8": (None, [_f32p, _sz, _i, _sz, _u32p, _f32p]),
    "dav2o_im2col_quantize_s8": (None, [_f32p, _i, _i, _i, _i, _i, _i, _i, _i, _u32p, _f32p]),
    "dav2o_linear_s8": (None, [_u32p, _u32p, _f32p, _f32p, ctypes.c_void_p, _sz, _i, _i, _sz, _sz, _i, _i, _f32p]),
    "dav2o_conv_transpose_s8": (None, [_u32p, _u32p, _f32p, _f32p, _f32p, _i, _i, _i, _i, _i, _f32p]),
    "dav2o_pack_weight_s8": (None, [_f32p, _sz, _i, _i, _i, _i, _u32p, _f32p]),
    "dav2o_linear_f32": (None, [_f32p, _f32p, ctypes.c_void_p, _sz, _i, _i, _f32p]),
    "dav2o_conv2d_f32": (None, [_f32p, _f32p, ctypes.c_void_p, _i, _i, _i, _i, _i, _i, _i, _f32p]),
    "dav2o_conv_transpose_f32": (None, [_f32p, _f32p, _f32p, _i, _i, _i, _i, _i, _f32p]),
    "dav2o_project_tokens_f32": (None, [_f32p, _f32p, _f32p, _i, _i, _i, _i, _f32p]),
    "dav2o_patch_embed_f32": (None, [_f32p, _f32p, _f32p, _f32p, _i, _i, _i, _f32p]),
    "dav2o_position_bicubic": (None, [_f32p, _i, _i, _i, _f32p]),
    "dav2o_add_position": (None, [_f32p, _f32p, _f32p, _i, _i, _i]),
    "dav2o_attention_head64": (None, [_f32p, _i, _i, _f32p]),
    "dav2o_threads": (_i, []),
    "dav2o_set_threads": (None, [_i]),
}


def build() -> Path:
    """Compile liboracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _HERE / "liboracle.so"


def lib():
    global _LIB
    if _LIB is None:
        path = _HERE / "liboracle.so"
        if not path.exists():
            build()
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGS.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------- operators
def crc32(data: bytes) -> int:
    buf = ctypes.create_string_buffer(data, len(data))
    return lib().dav2o_crc32(ctypes.cast(buf, ctypes.c_void_p), len(data))


def network_shape(width, height, input_size):
    ow, oh = _i(), _i()
    rc = lib().dav2o_network_shape(width, height, input_size, ctypes.byref(ow), ctypes.byref(oh))
    if rc != 0:
        raise ValueError("image dimensions and input_size must be positive")
    return ow.value, oh.value


def preprocess_bgr8(bgr, dst_w, dst_h):
    bgr = _c(bgr, np.uint8)
    h, w = bgr.shape[:2]
    out = np.empty((3, dst_h, dst_w), np.float32)
    rc = lib().dav2o_preprocess_bgr8(bgr, w, h, w * 3, dst_w, dst_h, out)
    if rc != 0:
        raise ValueError("invalid source image")
    return out


def preprocess_inferbridge_bgra8(bgra, dst_w, dst_h):
    bgra = _c(bgra, np.uint8)
    h, w = bgra.shape[:2]
    out = np.empty((3, dst_h, dst_w), np.float32)
    rc = lib().dav2o_preprocess_inferbridge_bgra8(bgra, w, h, w * 4, dst_w, dst_h, out)
    if rc != 0:
        raise ValueError("invalid source image")
    return out


def preprocess_u32_bicubic(pixels, dst_w, dst_h, rgba=False):
    pixels = _c(pixels, np.uint32)
    h, w = pixels.shape
    out = np.empty((3, dst_h, dst_w), np.float32)
    lib().dav2o_preprocess_u32_bicubic(pixels, w, h, w, int(rgba), dst_w, dst_h, out)
    return out


def preprocess_bgr8_bilinear(bgr, dst_w, dst_h):
    bgr = _c(bgr, np.uint8)
    h, w = bgr.shape[:2]
    out = np.empty((3, dst_h, dst_w), np.float32)
    lib().dav2o_preprocess_bgr8_bilinear(bgr, w, h, w * 3, dst_w, dst_h, out)
    return out


def layer_norm(x, w, b, eps=1e-6):
    x = _c(x)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().dav2o_layer_norm(x, _c(w), _c(b), out, x.size // cols, cols, eps)
    return out


def gelu(x):
    x = _c(x)
    out = np.empty_like(x)
    lib().dav2o_gelu(x, out, x.size)
    return out


def softmax_rows(x, scale=1.0):
    x = _c(x)
    cols = x.shape[-1]
    out = np.empty_like(x)
    lib().dav2o_softmax_rows(x, out, x.size // cols, cols, scale)
    return out


def add_scaled(residual, addend, scale):
    residual, addend, scale = _c(residual), _c(addend), _c(scale)
    out = np.empty_like(residual)
    lib().dav2o_add_scaled(residual, addend, scale, out, residual.size, scale.size)
    return out


def relu(x):
    x = _c(x)
    out = np.empty_like(x)
    lib().dav2o_relu(x, out, x.size)
    return out


def add(a, b):
    a, b = _c(a), _c(b)
    out = np.empty_like(a)
    lib().dav2o_add(a, b, out, a.size)
    return out


def sigmoid_scale(x, scale):
    x = _c(x)
    out = np.empty_like(x)
    lib().dav2o_sigmoid_scale(x, out, x.size, scale)
    return out


def bilinear_align_true(x, out_w, out_h):
    x = _c(x)
    c, h, w = x.shape
    out = np.empty((c, out_h, out_w), np.float32)
    lib().dav2o_bilinear_align_true(x, w, h, out_w, out_h, c, out)
    return out


def bilinear_half_pixel(x, out_w, out_h):
    x = _c(x)
    c, h, w = x.shape
    out = np.empty((c, out_h, out_w), np.float32)
    lib().dav2o_bilinear_half_pixel(x, w, h, out_w, out_h, c, out)
    return out


def reduce_minmax(x):
    x = _c(x)
    rng = np.empty(2, np.float32)
    lib().dav2o_reduce_minmax(x, x.size, rng)
    return rng


def normalize_relative(depth, rng):
    d = _c(depth).copy()
    lib().dav2o_normalize_relative(d, d.size, _c(rng))
    return d


def normalize_metric(depth, rng, maximum_depth):
    d = _c(depth).copy()
    lib().dav2o_normalize_metric(d, d.size, _c(rng), maximum_depth)
    return d


def quantize_rows_s8(x, rows, cols, input_offset=0):
    x = _c(x).reshape(-1)
    packed = np.empty((rows, cols // 4), np.uint32)
    scales = np.empty(rows, np.float32)
    lib().dav2o_quantize_rows_s8(x, rows, cols, input_offset, packed, scales)
    return packed, scales


def im2col_quantize_s8(x, kernel, stride, padding):
    x = _c(x)
    c, h, w = x.shape
    ow = (w + 2 * padding - kernel) // stride + 1
    oh = (h + 2 * padding - kernel) // stride + 1
    words = (c * kernel * kernel + 3) // 4
    packed = np.empty((oh * ow, words), np.uint32)
    scales = np.empty(oh * ow, np.float32)
    lib().dav2o_im2col_quantize_s8(x, w, h, c, ow, oh, kernel, stride, padding, packed, scales)
    return packed, scales


def linear_s8(packed_in, packed_w, s_in, s_w, bias, rows, in_cols, out_cols,
              row_offset=0, row_stride=None, transposed=False, out=None):
    row_stride = rows if row_stride is None else row_stride
    if out is None:
        size = out_cols * row_stride if transposed else (rows + row_offset) * out_cols
        out = np.zeros(size, np.float32)
    b = None if bias is None else _c(bias)
    lib().dav2o_linear_s8(_c(packed_in, np.uint32), _c(packed_w, np.uint32), _c(s_in), _c(s_w),
                          _ptr(b), rows, in_cols, out_cols, row_offset, row_stride,
                          int(transposed), int(b is not None), out)
    return out


def conv_transpose_s8(packed_in, packed_w, s_in, s_w, bias, in_w, in_h, in_c, out_c, k):
    out = np.empty((out_c, in_h * k, in_w * k), np.float32)
    lib().dav2o_conv_transpose_s8(_c(packed_in, np.uint32), _c(packed_w, np.uint32), _c(s_in),
                                  _c(s_w), _c(bias), in_w, in_h, in_c, out_c, k, out)
    return out


def pack_weight_s8(weight, transposed_conv=False):
    """Per-output-row symmetric int8 codes (src/gpu_model.cpp:207-284)."""
    weight = _c(weight)
    if transposed_conv:
        cin, cout, k, _ = weight.shape
        rows, cols = k * k * cout, cin
    else:
        rows, cols = weight.shape[0], weight.size // weight.shape[0]
        cout, k = 0, 0
    packed = np.empty((rows, cols // 4), np.uint32)
    scales = np.empty(rows, np.float32)
    lib().dav2o_pack_weight_s8(weight, rows, cols, int(transposed_conv), cout, k, packed, scales)
    return packed, scales


def linear_f32(x, w, b):
    x, w = _c(x), _c(w)
    rows = x.size // x.shape[-1]
    out = np.empty((rows, w.shape[0]), np.float32)
    bb = None if b is None else _c(b)
    lib().dav2o_linear_f32(x, w, _ptr(bb), rows, x.shape[-1], w.shape[0], out)
    return out


def conv2d_f32(x, w, b, stride=1, padding=0):
    x, w = _c(x), _c(w)
    c, h, wd = x.shape
    co, _, k, _ = w.shape
    ow = (wd + 2 * padding - k) // stride + 1
    oh = (h + 2 * padding - k) // stride + 1
    out = np.empty((co, oh, ow), np.float32)
    bb = None if b is None else _c(b)
    lib().dav2o_conv2d_f32(x, w, _ptr(bb), wd, h, c, co, k, stride, padding, out)
    return out


def conv_transpose_f32(x, w, b):
    x, w = _c(x), _c(w)
    c, h, wd = x.shape
    _, co, k, _ = w.shape
    out = np.empty((co, h * k, wd * k), np.float32)
    lib().dav2o_conv_transpose_f32(x, w, _c(b), wd, h, c, co, k, out)
    return out


def project_tokens_f32(tokens, w, b, pw, ph):
    tokens = _c(tokens)
    co, emb = w.shape[0], w.size // w.shape[0]
    out = np.empty((co, ph, pw), np.float32)
    lib().dav2o_project_tokens_f32(tokens, _c(w).reshape(co, emb), _c(b), pw, ph, emb, co, out)
    return out


def patch_embed_f32(image, w, b, cls):
    image = _c(image)
    _, h, wd = image.shape
    emb = w.shape[0]
    out = np.empty(((h // 14) * (wd // 14) + 1, emb), np.float32)
    lib().dav2o_patch_embed_f32(image, _c(w), _c(b), _c(cls).reshape(-1), wd, h, emb, out)
    return out


def position_bicubic(pos_embed, pw, ph):
    pos = _c(pos_embed).reshape(1370, -1)
    emb = pos.shape[1]
    out = np.empty((emb, ph, pw), np.float32)
    lib().dav2o_position_bicubic(pos, emb, pw, ph, out)
    return out


def add_position(tokens, planar, pos_embed, pw, ph):
    t = _c(tokens).copy()
    pos = _c(pos_embed).reshape(1370, -1)
    lib().dav2o_add_position(t, _c(planar), pos, pw, ph, pos.shape[1])
    return t


def attention_head64(qkv, tokens, heads):
    out = np.empty((tokens, heads * 64), np.float32)
    lib().dav2o_attention_head64(_c(qkv), tokens, heads, out)
    return out


def threads() -> int:
    return lib().dav2o_threads()


def set_threads(n: int) -> None:
    lib().dav2o_set_threads(n)


# ------------------------------------------------------------------ the graph
ENCODERS = {
    # name: (embedding, heads, blocks, taps, features, out_channels)
    "vits": (384, 6, 12, (2, 5, 8, 11), 64, (48, 96, 192, 384)),
    "vitb": (768, 12, 12, (2, 5, 8, 11), 128, (96, 192, 384, 768)),
    "vitl": (1024, 16, 24, (4, 11, 17, 23), 256, (256, 512, 1024, 1024)),
}


class _Int8Weights:
    """Lazily packed per-output-row int8 weight codes (src/gpu_model.cpp:207-284)."""

    def __init__(self, sd):
        self.sd = sd
        self.cache = {}

    def get(self, name, transposed_conv=False):
        if name not in self.cache:
            self.cache[name] = pack_weight_s8(self.sd[name], transposed_conv)
        return self.cache[name]


def _linear(sd, q8, x, name, precision):
    w, b = sd[name + ".weight"], sd[name + ".bias"]
    if precision == "int8":
        rows, cols = x.shape
        px, sx = quantize_rows_s8(x, rows, cols)
        pw, sw = q8.get(name + ".weight")
        return linear_s8(px, pw, sx, sw, b, rows, cols, w.shape[0]).reshape(rows, w.shape[0])
    return linear_f32(x, w, b)


def ln1_codes(sd, x, block):
    """Block `block`'s first LayerNorm (f32) and, at int8 precision, the
    per-row codes and scales its QKV GEMM reads (quantize_rows_int8_fused:
    x / scale): returns (normalized f32, packed codes u32, scales)."""
    p = f"pretrained.blocks.{block}"
    n = layer_norm(x, sd[p + ".norm1.weight"], sd[p + ".norm1.bias"])
    rows, cols = n.shape
    px, sx = quantize_rows_s8(n, rows, cols)
    return n, px, sx


def encoder_block(sd, x, block, encoder, precision="fp32", q8=None, tokens=None):
    """One DINOv2 block of src/encoder.cpp:426-591 on residual rows x
    ([images*tokens, D], images stacked; tokens = rows of one image).

    precision "int8" restates the reference's INT8 routing: every linear on
    per-row int8 activations (src/operators.cpp:770-845) with f32 outputs,
    attention at its fp16 operand precision — Q, K and V rounded to f16 as
    bmm_score_fp16.glsl / bmm_value_fp16.glsl read them
    (src/encoder.cpp:389-396) — with f32 scores, softmax and accumulation, and
    the f32 attention output and GELU hidden quantized by the next linear."""
    emb, heads, _, _, _, _ = ENCODERS[encoder]
    q8 = q8 if q8 is not None else _Int8Weights(sd)
    tokens = tokens or x.shape[0]
    p = f"pretrained.blocks.{block}"
    n = layer_norm(x, sd[p + ".norm1.weight"], sd[p + ".norm1.bias"])
    qkv = _linear(sd, q8, n, p + ".attn.qkv", precision)
    if precision == "int8":
        qkv = qkv.astype(np.float16).astype(np.float32)
    att = np.concatenate([attention_head64(qkv[i:i + tokens], tokens, heads)
                          for i in range(0, x.shape[0], tokens)]).reshape(x.shape[0], emb)
    y = _linear(sd, q8, att, p + ".attn.proj", precision)
    x = add_scaled(x, y, sd[p + ".ls1.gamma"])
    n = layer_norm(x, sd[p + ".norm2.weight"], sd[p + ".norm2.bias"])
    hdn = gelu(_linear(sd, q8, n, p + ".mlp.fc1", precision))
    y = _linear(sd, q8, hdn, p + ".mlp.fc2", precision)
    return add_scaled(x, y, sd[p + ".ls2.gamma"])


def embed(sd, image, encoder, precision="fp32"):
    """Patch embedding + cls + positional embedding (src/operators.cpp:1211-1406)
    of one planar [3,H,W] image: the residual rows entering block 0."""
    emb = ENCODERS[encoder][0]
    _, h, w = image.shape
    pw, ph = w // 14, h // 14
    if precision == "int8":
        q8 = _Int8Weights(sd)
        packed, scales = im2col_quantize_s8(image, 14, 14, 0)
        pwt, swt = q8.get("pretrained.patch_embed.proj.weight")
        tokens = np.zeros(((pw * ph + 1), emb), np.float32)
        tokens[0] = sd["pretrained.cls_token"].reshape(-1)
        tokens = linear_s8(packed, pwt, scales, swt, sd["pretrained.patch_embed.proj.bias"],
                           pw * ph, 3 * 14 * 14, emb, row_offset=1, row_stride=pw * ph + 1,
                           out=tokens.reshape(-1)).reshape(-1, emb)
    else:
        tokens = patch_embed_f32(image, sd["pretrained.patch_embed.proj.weight"],
                                 sd["pretrained.patch_embed.proj.bias"], sd["pretrained.cls_token"])
    planar = position_bicubic(sd["pretrained.pos_embed"], pw, ph)
    return add_position(tokens, planar, sd["pretrained.pos_embed"], pw, ph)


def encoder_forward(sd, image, encoder, precision="fp32"):
    """DINOv2 forward of src/encoder.cpp:322-597 on one planar [3,H,W] image.

    precision "fp32" restates the FP32 executor; "int8" the INT8 routing
    (encoder_block) with the int8 patch embedding of src/operators.cpp:1270-1308.
    Returns the four tapped, normalized token matrices [1+hw, D] and (pw, ph).
    """
    _, _, blocks, taps, _, _ = ENCODERS[encoder]
    _, h, w = image.shape
    pw, ph = w // 14, h // 14
    q8 = _Int8Weights(sd)
    x = embed(sd, image, encoder, precision)
    feats = []
    for i in range(blocks):
        x = encoder_block(sd, x, i, encoder, precision, q8)
        if i in taps:
            feats.append(layer_norm(x, sd["pretrained.norm.weight"], sd["pretrained.norm.bias"]))
    return feats, pw, ph


def _conv(sd, x, name, stride, padding, bias=True, q8=None):
    w = sd[name + ".weight"]
    b = sd.get(name + ".bias") if bias else None
    if q8 is not None:
        c, h, wd = x.shape
        k = w.shape[2]
        packed, scales = im2col_quantize_s8(x, k, stride, padding)
        pwt, swt = q8.get(name + ".weight")
        ow = (wd + 2 * padding - k) // stride + 1
        oh = (h + 2 * padding - k) // stride + 1
        out = linear_s8(packed, pwt, scales, swt, b, ow * oh, c * k * k, w.shape[0], transposed=True)
        return out.reshape(w.shape[0], oh, ow)
    return conv2d_f32(x, w, b, stride, padding)


def _rcu(sd, x, prefix):
    out = relu(x)
    out = _conv(sd, out, prefix + ".conv1", 1, 1)
    out = relu(out)
    out = _conv(sd, out, prefix + ".conv2", 1, 1)
    return add(out, x)


def _fusion(sd, path, skip, prefix, out_w, out_h):
    if skip is not None:
        path = add(path, _rcu(sd, skip, prefix + ".resConfUnit1"))
    path = _rcu(sd, path, prefix + ".resConfUnit2")
    path = bilinear_align_true(path, out_w, out_h)
    return _conv(sd, path, prefix + ".out_conv", 1, 0)


def dpt_forward(sd, feats, pw, ph, encoder, precision="fp32", metric_max_depth=0.0):
    """DPT head of src/dpt.cpp:628-863: returns depth [14*ph, 14*pw].

    In "int8" the projections and resize layers use int8 (src/dpt.cpp:504-506)
    and the refinement convolutions stay fp32 (the reference keeps them at
    its fp16/fp32 refinement precision)."""
    _, _, _, _, features, out_ch = ENCODERS[encoder]
    q8 = _Int8Weights(sd) if precision == "int8" else None
    layers = []
    for i in range(4):
        name = f"depth_head.projects.{i}"
        if q8 is not None:
            rows, emb = pw * ph, feats[i].shape[1]
            px, sx = quantize_rows_s8(feats[i], rows, emb, input_offset=emb)
            pwt, swt = q8.get(name + ".weight")
            proj = linear_s8(px, pwt, sx, swt, sd[name + ".bias"], rows, emb, out_ch[i],
                             transposed=True).reshape(out_ch[i], ph, pw)
        else:
            proj = project_tokens_f32(feats[i], sd[name + ".weight"], sd[name + ".bias"], pw, ph)
        r = f"depth_head.resize_layers.{i}"
        if i < 2:
            if q8 is not None:
                k = 4 if i == 0 else 2
                packed, scales = im2col_quantize_s8(proj, 1, 1, 0)
                pwt, swt = q8.get(r + ".weight", transposed_conv=True)
                layers.append(conv_transpose_s8(packed, pwt, scales, swt, sd[r + ".bias"],
                                                pw, ph, out_ch[i], out_ch[i], k))
            else:
                layers.append(conv_transpose_f32(proj, sd[r + ".weight"], sd[r + ".bias"]))
        elif i == 2:
            layers.append(proj)
        else:
            layers.append(_conv(sd, proj, r, 2, 1, q8=q8))
    rn = [_conv(sd, layers[i], f"depth_head.scratch.layer{i + 1}_rn", 1, 1, bias=False) for i in range(4)]
    s = "depth_head.scratch"
    path = _fusion(sd, rn[3], None, s + ".refinenet4", rn[2].shape[2], rn[2].shape[1])
    path = _fusion(sd, path, rn[2], s + ".refinenet3", rn[1].shape[2], rn[1].shape[1])
    path = _fusion(sd, path, rn[1], s + ".refinenet2", rn[0].shape[2], rn[0].shape[1])
    path = _fusion(sd, path, rn[0], s + ".refinenet1", rn[0].shape[2] * 2, rn[0].shape[1] * 2)
    out = _conv(sd, path, s + ".output_conv1", 1, 1)
    out = bilinear_align_true(out, pw * 14, ph * 14)
    out = _conv(sd, out, s + ".output_conv2.0", 1, 1)
    out = relu(out)
    out = _conv(sd, out, s + ".output_conv2.2", 1, 0)
    if metric_max_depth > 0:
        out = sigmoid_scale(out, metric_max_depth)
    else:
        out = relu(out)
    return out.reshape(ph * 14, pw * 14)


def infer_tensor(sd, image, encoder, precision="fp32", out_w=None, out_h=None, metric_max_depth=0.0):
    """dav2_infer_tensor_f32 / Executor::infer_resized on one planar image
    (src/vulkan_executor.cpp:572-636): graph, then align-corners bilinear to
    the requested output size when it differs. metric_max_depth > 0 selects
    the metric head (a model file with is_metric set)."""
    feats, pw, ph = encoder_forward(sd, image, encoder, precision)
    depth = dpt_forward(sd, feats, pw, ph, encoder, precision, metric_max_depth)
    h, w = depth.shape
    if out_w is not None and (out_w != w or out_h != h):
        depth = bilinear_align_true(depth[None], out_w, out_h)[0]
    return depth


def inferbridge_bgra8(sd, bgra, encoder, input_size=518, precision="fp32", metric_max_depth=0.0):
    """dav2_inferbridge_bgra8_f32 (src/dav2.cpp:754-803): nearest resize to
    the transposed network shape, graph, then host min/max normalization
    (span max - min, or 25 - min for a metric model; all zeros when the span
    is not positive)."""
    h, w = bgra.shape[:2]
    nw, nh = network_shape(w, h, input_size)
    image = preprocess_inferbridge_bgra8(bgra, nh, nw)
    depth = infer_tensor(sd, image, encoder, precision, metric_max_depth=metric_max_depth)
    lo = np.float32(depth.min())
    span = np.float32(25.0) - lo if metric_max_depth > 0 else np.float32(depth.max()) - lo
    if not span > 0:
        return np.zeros_like(depth)
    return ((depth - lo) / span).astype(np.float32)


def infer_bgr8(sd, bgr, encoder, input_size=518, precision="fp32"):
    """dav2_infer_bgr8 (src/dav2.cpp:630-668)."""
    h, w = bgr.shape[:2]
    nw, nh = network_shape(w, h, input_size)
    image = preprocess_bgr8(bgr, nw, nh)
    return infer_tensor(sd, image, encoder, precision, w, h)


if os.environ.get("DAV2_ORACLE_BUILD_ON_IMPORT") == "1":
    build()
