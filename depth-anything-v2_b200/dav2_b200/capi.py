"""ctypes declarations of the public C ABI (include/depth_anything_v2.h)."""
from __future__ import annotations

import ctypes

u32, i32, u64, f32 = ctypes.c_uint32, ctypes.c_int32, ctypes.c_uint64, ctypes.c_float
vp = ctypes.c_void_p


class CreateOptions(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("abi_version", u32), ("encoder", ctypes.c_int),
                ("vulkan_device_index", i32), ("flags", u32), ("cache_path_utf8", ctypes.c_char_p)]


class ModelInfo(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("abi_version", u32), ("encoder", ctypes.c_int), ("is_metric", u32),
                ("metric_max_depth", f32), ("reserved", u32 * 3)]


class ImageShape(ctypes.Structure):
    _fields_ = [("width", i32), ("height", i32)]


class GpuCapabilities(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("abi_version", u32), ("flags", u64), ("adapter_luid", u64),
                ("maximum_in_flight_jobs", u32), ("reserved", u32)]


class TransferCounters(ctypes.Structure):
    _fields_ = [("struct_size", u32), ("reserved", u32), ("tensor_upload_bytes", u64),
                ("tensor_download_bytes", u64)]


ABI_VERSION = 1
ENCODERS = {"vits": 0, "vitb": 1, "vitl": 2}
FLAGS = {"fp32": 1 << 0, "fp32_weights": 1 << 1, "fp32_attention": 1 << 2, "fp16": 1 << 3, "int8": 1 << 4,
         "metal": 1 << 5, "vulkan": 1 << 6, "bf16": 1 << 7}
STATUS = {0: "ok", 1: "invalid argument", 2: "model I/O error", 3: "invalid model format",
          4: "Vulkan unavailable", 5: "out of memory", 6: "inference failed", 7: "buffer too small",
          8: "unsupported", 9: "internal error", 10: "invalid state", 11: "cancelled"}

PUBLIC = {
    "dav2_abi_version": (u32, []),
    "dav2_version_string": (ctypes.c_char_p, []),
    "dav2_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "dav2_last_error": (ctypes.c_char_p, []),
    "dav2_get_network_shape": (ctypes.c_int, [i32, i32, i32, ctypes.POINTER(ImageShape)]),
    "dav2_get_inferbridge_shape": (ctypes.c_int, [i32, i32, i32, ctypes.POINTER(ImageShape)]),
    "dav2_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(CreateOptions), ctypes.POINTER(vp)]),
    "dav2_get_model_info": (ctypes.c_int, [vp, ctypes.POINTER(ModelInfo)]),
    "dav2_prepare": (ctypes.c_int, [vp, i32, i32, i32]),
    "dav2_destroy": (None, [vp]),
    "dav2_probe_gpu_capabilities": (ctypes.c_int, [i32, ctypes.POINTER(GpuCapabilities)]),
    "dav2_get_gpu_capabilities": (ctypes.c_int, [vp, ctypes.POINTER(GpuCapabilities)]),
    "dav2_get_transfer_counters": (ctypes.c_int, [vp, ctypes.POINTER(TransferCounters)]),
    "dav2_submit_d3d12": (ctypes.c_int, [vp, vp, ctypes.POINTER(vp)]),
    "dav2_submit_d3d12_texture": (ctypes.c_int, [vp, vp, ctypes.POINTER(vp)]),
    "dav2_submit_d3d12_texture_binding": (ctypes.c_int, [vp, vp, ctypes.POINTER(vp)]),
    "dav2_submit_metal_texture_binding": (ctypes.c_int, [vp, vp, ctypes.POINTER(vp)]),
    "dav2_gpu_job_poll": (ctypes.c_int, [vp, vp]),
    "dav2_gpu_job_cancel": (ctypes.c_int, [vp]),
    "dav2_gpu_job_release": (None, [vp]),
    "dav2_gpu_output_acquire": (ctypes.c_int, [vp, u32, vp, ctypes.POINTER(vp)]),
    "dav2_gpu_texture_output_acquire": (ctypes.c_int, [vp, u32, vp, ctypes.POINTER(vp)]),
    "dav2_gpu_output_release": (None, [vp]),
    "dav2_infer_bgr8": (ctypes.c_int, [vp, vp, i32, i32, ctypes.c_ssize_t, i32, vp, ctypes.c_size_t]),
    "dav2_inferbridge_bgra8_f32": (ctypes.c_int, [vp, vp, i32, i32, ctypes.c_ssize_t, i32, vp, ctypes.c_size_t]),
    "dav2_infer_tensor_f32": (ctypes.c_int, [vp, vp, i32, i32, vp, ctypes.c_size_t]),
    # extensions (no reference counterpart): batched entry points
    "dav2_infer_tensor_f32_batch": (ctypes.c_int, [vp, vp, u32, i32, i32, vp, ctypes.c_size_t]),
    "dav2_infer_bgr8_batch": (ctypes.c_int, [vp, vp, u32, i32, i32, ctypes.c_ssize_t, ctypes.c_ssize_t, i32, vp,
                                             ctypes.c_size_t]),
    "dav2_infer_device_bgr8_batch": (ctypes.c_int, [vp, vp, u32, i32, i32, ctypes.c_ssize_t, ctypes.c_ssize_t, i32,
                                                    vp, vp]),
    "dav2_synchronize": (ctypes.c_int, [vp]),
    "dav2_infer_device_frames_bgr8": (ctypes.c_int, [vp, vp, u32, i32, i32, ctypes.c_ssize_t, ctypes.c_ssize_t, i32,
                                                     vp, vp]),
    "dav2_submit_device_pixels": (ctypes.c_int, [vp, vp, u32, i32, i32, ctypes.c_ssize_t, ctypes.c_ssize_t,
                                                 ctypes.c_int, i32, vp, vp]),
    "dav2_probe_encoder_block": (ctypes.c_int, [vp, u32, i32, i32, u32, vp, vp, vp, vp]),
    "dav2_probe_head": (ctypes.c_int, [vp, u32, i32, i32, vp, vp]),
    "dav2_get_kernel_launch_count": (ctypes.c_int, [vp, ctypes.POINTER(u64)]),
    "dav2_profile_operations": (ctypes.c_int, [vp, u32, i32, i32, ctypes.c_char_p, ctypes.c_size_t]),
}


def declare(lib) -> None:
    for name, (res, args) in PUBLIC.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
