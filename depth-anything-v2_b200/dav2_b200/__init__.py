"""Python access to libdav2_b200.so (the B200 executor and its operator C ABI).

The library is the product: the public C ABI of include/depth_anything_v2.h
(dav2_create / dav2_infer_bgr8 / dav2_infer_tensor_f32 ...) and the
operator-layer C ABI of include/dav2cuda.h. This module only declares the
ctypes signatures. It never falls back to a CPU implementation: loading fails
loudly when the shared library is missing.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
LIB_PATH = PKG / "lib" / "libdav2_b200.so"
INCLUDE = PKG.parent / "include"

_lib = None

u32, i32, u64, f32 = ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint64, ctypes.c_float
vp = ctypes.c_void_p
szt = ctypes.c_size_t

# name: (restype, argtypes) for include/dav2cuda.h
DAV2CUDA = {
    "dav2cuda_last_error": (ctypes.c_char_p, []),
    "dav2cuda_build_info": (ctypes.c_char_p, []),
    "dav2cuda_device_error": (ctypes.c_int, []),
    "dav2cuda_launch_count": (u64, [ctypes.c_int]),
    "dav2cuda_wait_probe": (ctypes.c_int, [u64, u32, vp]),
    "dav2cuda_layer_norm": (ctypes.c_int, [vp, vp, vp, vp, u32, u32, f32, vp]),
    "dav2cuda_gelu": (ctypes.c_int, [vp, vp, u64, vp]),
    "dav2cuda_softmax_rows": (ctypes.c_int, [vp, vp, u64, u32, f32, vp]),
    "dav2cuda_add_scaled": (ctypes.c_int, [vp, vp, vp, vp, u64, u32, vp]),
    "dav2cuda_relu": (ctypes.c_int, [vp, vp, u64, vp]),
    "dav2cuda_add": (ctypes.c_int, [vp, vp, vp, u64, vp]),
    "dav2cuda_sigmoid_scale": (ctypes.c_int, [vp, vp, u64, f32, vp]),
    "dav2cuda_bilinear_align_true": (ctypes.c_int, [vp, vp, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_bilinear_align_nhwc_16": (ctypes.c_int, [vp, vp, u32, u32, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_reduce_minmax": (ctypes.c_int, [vp, vp, u64, vp]),
    "dav2cuda_normalize_relative": (ctypes.c_int, [vp, vp, u64, vp]),
    "dav2cuda_normalize_metric": (ctypes.c_int, [vp, vp, u64, f32, vp]),
    "dav2cuda_preprocess_u32": (ctypes.c_int, [vp, vp, u32, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_preprocess_bgr8": (ctypes.c_int, [vp, vp, u32, u32, u32, u64, u64, u32, u32, vp]),
    "dav2cuda_preprocess_bgr8_bilinear": (ctypes.c_int, [vp, vp, u32, u32, u32, u64, u64, u32, u32, vp]),
    "dav2cuda_quantize_rows_s8": (ctypes.c_int, [vp, vp, vp, u32, u32, u64, vp]),
    "dav2cuda_pack_weight_s8": (ctypes.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_im2col_quantize_s8": (ctypes.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, i32, vp]),
    "dav2cuda_linear_s8_packed": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_linear_int8_workspace_size": (u64, [u32, u32, u32]),
    "dav2cuda_conv2d_int8_workspace_size": (u64, [u32, u32, u32, u32, u32, u32, u32]),
    "dav2cuda_conv_transpose_int8_workspace_size": (u64, [u32, u32, u32, u32, u32]),
    "dav2cuda_linear_int8": (ctypes.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_linear_int8_residual": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_im2col_quantize_nhwc": (ctypes.c_int, [vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_linear_int8_noalloc_scratch_limit": (u64, []),
    "dav2cuda_linear_int8_noalloc": (ctypes.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, vp]),
    "dav2cuda_conv2d_int8": (ctypes.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_conv_transpose_int8": (ctypes.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_conv3x3_int8_up2_workspace_size": (u64, [u32, u32, u32, u32, u32]),
    "dav2cuda_conv3x3_int8_up2": (ctypes.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_conv3x3_head_16": (ctypes.c_int, [vp, vp, vp, vp, vp, f32, f32, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_conv3x3_c128_16": (ctypes.c_int, [vp, vp, vp, vp, u32, u32, u32, u32, u32, vp]),
    "dav2cuda_prepare_tokens_workspace_size": (u64, [u32, u32, u32]),
    "dav2cuda_prepare_tokens_half": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_prepare_tokens_int8": (ctypes.c_int, [vp, vp, vp, vp, vp, vp, vp, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_project_tokens_workspace_size": (u64, [u32, u32, u32, u32]),
    "dav2cuda_project_tokens_half": (ctypes.c_int, [vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_project_tokens_int8": (ctypes.c_int, [vp, vp, vp, vp, vp, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_conv_transpose_half_workspace_size": (u64, [u32, u32, u32, u32, u32]),
    "dav2cuda_conv_transpose_half": (ctypes.c_int, [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_attention_head64": (ctypes.c_int, [vp, vp, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_attention_head64_workspace_size": (u64, [u32, u32, u32]),
    "dav2cuda_linear_half_workspace_size": (u64, [u32, u32, u32]),
    "dav2cuda_linear_half": (ctypes.c_int, [vp, vp, vp, vp, u32, u32, u32, u32, u32, vp, u64, vp]),
    "dav2cuda_conv2d_half_workspace_size": (u64, [u32, u32, u32, u32, u32, u32, u32]),
    "dav2cuda_conv2d_half": (ctypes.c_int, [vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, u32, vp, u64, vp]),
}


def lib_path() -> Path:
    return LIB_PATH


def load(path: Path | None = None):
    """Load libdav2_b200.so and declare the C signatures (raises if absent)."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(path or LIB_PATH)
    if not path.exists():
        raise FileNotFoundError(f"{path} is missing: run __graft_entry__.build() first")
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in DAV2CUDA.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    from . import capi

    capi.declare(lib)
    _lib = lib
    return lib


class Dav2CudaError(RuntimeError):
    pass


def check(rc: int) -> None:
    if rc != 0:
        msg = _lib.dav2cuda_last_error().decode() if _lib is not None else ""
        raise Dav2CudaError(f"dav2cuda status {rc}: {msg}")
