/*
 * Depth Anything V2 native inference ABI, served by the B200 CUDA executor.
 *
 * Drop-in for the reference runtime's public header (include/depth_anything_v2.h
 * of laurentdupin/Depth-Anything-V2): every type, constant, struct layout and
 * function signature below is the one that header defines (ABI version 1), so
 * existing callers (C, ctypes as in tools/compare_assets.py:116-137) link
 * unchanged. The executor behind it is CUDA (sm_100a); Vulkan/Metal-specific
 * names keep their meaning for source compatibility:
 *   - dav2_create_options.vulkan_device_index selects the CUDA device ordinal;
 *   - DAV2_CREATE_FORCE_METAL / _VULKAN are accepted and select no other
 *     backend (there is none in this library);
 *   - the D3D12 / Metal texture submission functions return
 *     DAV2_STATUS_UNSUPPORTED (graphics-API interop is not part of this
 *     library; the headless device-buffer path is dav2_infer_device_bgr8_batch).
 * Functions marked EXTENSION have no counterpart in the reference.
 */
#ifndef DEPTH_ANYTHING_V2_H
#define DEPTH_ANYTHING_V2_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define DAV2_API __declspec(dllexport)
#define DAV2_CALL __cdecl
#else
#define DAV2_API __attribute__((visibility("default")))
#define DAV2_CALL
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DAV2_ABI_VERSION 1u

typedef struct dav2_context dav2_context;
typedef struct dav2_gpu_job dav2_gpu_job;
typedef struct dav2_gpu_output_lease dav2_gpu_output_lease;

typedef enum dav2_status {
    DAV2_STATUS_OK = 0,
    DAV2_STATUS_INVALID_ARGUMENT = 1,
    DAV2_STATUS_MODEL_IO = 2,
    DAV2_STATUS_MODEL_FORMAT = 3,
    DAV2_STATUS_VULKAN_UNAVAILABLE = 4, /* here: no usable CUDA device */
    DAV2_STATUS_OUT_OF_MEMORY = 5,
    DAV2_STATUS_INFERENCE_FAILED = 6,
    DAV2_STATUS_BUFFER_TOO_SMALL = 7,
    DAV2_STATUS_UNSUPPORTED = 8,
    DAV2_STATUS_INTERNAL_ERROR = 9,
    DAV2_STATUS_INVALID_STATE = 10,
    DAV2_STATUS_CANCELLED = 11
} dav2_status;

typedef enum dav2_encoder {
    DAV2_ENCODER_VITS = 0,
    DAV2_ENCODER_VITB = 1,
    DAV2_ENCODER_VITL = 2
} dav2_encoder;

typedef struct dav2_create_options {
    uint32_t struct_size;
    uint32_t abi_version;
    dav2_encoder encoder;
    int32_t vulkan_device_index;
    uint32_t flags;
    const char* cache_path_utf8; /* optional tail; unused by the CUDA executor */
} dav2_create_options;

enum {
    DAV2_CREATE_FORCE_FP32 = 1u << 0u,
    DAV2_CREATE_FORCE_FP32_WEIGHTS = 1u << 1u,
    DAV2_CREATE_FORCE_FP32_ATTENTION = 1u << 2u,
    DAV2_CREATE_FORCE_FP16 = 1u << 3u,
    DAV2_CREATE_FORCE_INT8 = 1u << 4u,
    DAV2_CREATE_FORCE_METAL = 1u << 5u,
    DAV2_CREATE_FORCE_VULKAN = 1u << 6u,
    /* EXTENSION (no reference counterpart; the reference has fp16, not bf16):
     * every GEMM, convolution and attention with bf16 operands and f32
     * accumulation, bf16 activations between them. */
    DAV2_CREATE_FORCE_BF16 = 1u << 7u
};

typedef struct dav2_model_info {
    uint32_t struct_size;
    uint32_t abi_version;
    dav2_encoder encoder;
    uint32_t is_metric;
    float metric_max_depth;
    uint32_t reserved[3];
} dav2_model_info;

typedef struct dav2_image_shape {
    int32_t width;
    int32_t height;
} dav2_image_shape;

enum {
    DAV2_GPU_CAP_D3D12_SHARED_INPUT = 1ull << 0u,
    DAV2_GPU_CAP_D3D12_FENCE_WAIT = 1ull << 1u,
    DAV2_GPU_CAP_D3D12_SHARED_OUTPUT = 1ull << 2u,
    DAV2_GPU_CAP_D3D12_FENCE_SIGNAL = 1ull << 3u,
    DAV2_GPU_CAP_ASYNC_SUBMIT = 1ull << 4u,
    DAV2_GPU_CAP_CANCELLATION = 1ull << 5u,
    DAV2_GPU_CAP_NO_HOST_PIXEL_STAGING = 1ull << 6u,
    DAV2_GPU_CAP_NO_HOST_DEPTH_STAGING = 1ull << 7u,
    DAV2_GPU_CAP_D3D12_SHARED_TEXTURE_INPUT = 1ull << 8u,
    DAV2_GPU_CAP_D3D12_SHARED_TEXTURE_OUTPUT = 1ull << 9u,
    DAV2_GPU_CAP_METAL_TEXTURE_INPUT = 1ull << 10u,
    DAV2_GPU_CAP_METAL_SHARED_EVENT_WAIT = 1ull << 11u,
    DAV2_GPU_CAP_METAL_TEXTURE_OUTPUT = 1ull << 12u,
    DAV2_GPU_CAP_METAL_SHARED_EVENT_SIGNAL = 1ull << 13u
};

typedef enum dav2_gpu_pixel_format {
    DAV2_GPU_PIXEL_BGRA8 = 1,
    DAV2_GPU_PIXEL_RGBA8 = 2,
    DAV2_GPU_PIXEL_DEPTH_FLOAT32 = 3
} dav2_gpu_pixel_format;

typedef enum dav2_gpu_job_state {
    DAV2_GPU_JOB_QUEUED = 0,
    DAV2_GPU_JOB_RUNNING = 1,
    DAV2_GPU_JOB_COMPLETE = 2,
    DAV2_GPU_JOB_FAILED = 3,
    DAV2_GPU_JOB_CANCELLED = 4
} dav2_gpu_job_state;

typedef struct dav2_gpu_capabilities {
    uint32_t struct_size;
    uint32_t abi_version;
    uint64_t flags;
    uint64_t adapter_luid;
    uint32_t maximum_in_flight_jobs;
    uint32_t reserved;
} dav2_gpu_capabilities;

typedef struct dav2_d3d12_submit_request {
    uint32_t struct_size;
    uint32_t abi_version;
    uint64_t shared_resource_handle;
    uint64_t resource_byte_size;
    uint32_t width;
    uint32_t height;
    uint32_t row_stride_bytes;
    uint32_t pixel_format;
    int32_t input_size;
    uint32_t reserved;
    uint64_t wait_fence_handle;
    uint64_t wait_fence_value;
    uint64_t source_frame_id;
    uint64_t timestamp_ns;
} dav2_d3d12_submit_request;

typedef struct dav2_d3d12_texture_submit_request {
    uint32_t struct_size;
    uint32_t abi_version;
    uint64_t shared_texture_handle;
    uint32_t width;
    uint32_t height;
    uint32_t pixel_format;
    int32_t input_size;
    uint64_t wait_fence_handle;
    uint64_t wait_fence_value;
    uint64_t source_frame_id;
    uint64_t timestamp_ns;
} dav2_d3d12_texture_submit_request;

typedef struct dav2_d3d12_texture_binding_request {
    uint32_t struct_size;
    uint32_t abi_version;
    uint64_t input_texture_handle;
    uint32_t input_width;
    uint32_t input_height;
    uint32_t input_pixel_format;
    int32_t input_size;
    uint64_t wait_fence_handle;
    uint64_t wait_fence_value;
    uint64_t output_texture_handle;
    uint32_t output_width;
    uint32_t output_height;
    uint64_t signal_fence_handle;
    uint64_t signal_fence_value;
    uint64_t source_frame_id;
    uint64_t timestamp_ns;
    uint64_t input_texture_identity;
    uint64_t output_texture_identity;
} dav2_d3d12_texture_binding_request;

typedef struct dav2_metal_texture_binding_request {
    uint32_t struct_size;
    uint32_t abi_version;
    uint64_t input_texture;
    uint32_t input_width;
    uint32_t input_height;
    uint32_t input_pixel_format;
    int32_t input_size;
    uint64_t wait_shared_event;
    uint64_t wait_value;
    uint64_t output_texture;
    uint32_t output_width;
    uint32_t output_height;
    uint64_t signal_shared_event;
    uint64_t signal_value;
    uint64_t source_frame_id;
    uint64_t timestamp_ns;
} dav2_metal_texture_binding_request;

typedef struct dav2_gpu_job_status {
    uint32_t struct_size;
    uint32_t state;
    uint32_t output_count;
    uint32_t reserved;
    uint64_t source_frame_id;
} dav2_gpu_job_status;

typedef struct dav2_d3d12_output_descriptor {
    uint32_t struct_size;
    uint32_t abi_version;
    uint32_t pixel_format;
    uint32_t reserved;
    uint32_t width;
    uint32_t height;
    uint32_t row_stride_bytes;
    uint32_t reserved2;
    uint64_t byte_size;
    uint64_t shared_resource_handle;
    uint64_t ready_fence_handle;
    uint64_t ready_fence_value;
    uint64_t source_frame_id;
    uint64_t timestamp_ns;
} dav2_d3d12_output_descriptor;

typedef struct dav2_d3d12_texture_output_descriptor {
    uint32_t struct_size;
    uint32_t abi_version;
    uint32_t pixel_format;
    uint32_t reserved;
    uint32_t width;
    uint32_t height;
    uint32_t reserved2;
    uint32_t reserved3;
    uint64_t shared_texture_handle;
    uint64_t ready_fence_handle;
    uint64_t ready_fence_value;
    uint64_t source_frame_id;
    uint64_t timestamp_ns;
} dav2_d3d12_texture_output_descriptor;

typedef struct dav2_transfer_counters {
    uint32_t struct_size;
    uint32_t reserved;
    uint64_t tensor_upload_bytes;
    uint64_t tensor_download_bytes;
} dav2_transfer_counters;

/* src/dav2.cpp:96-124 */
DAV2_API uint32_t DAV2_CALL dav2_abi_version(void);
DAV2_API const char* DAV2_CALL dav2_version_string(void);
DAV2_API const char* DAV2_CALL dav2_status_string(dav2_status status);
DAV2_API const char* DAV2_CALL dav2_last_error(void);

/* src/dav2.cpp:126-156 (network_shape rule: src/image.cpp:138-161) */
DAV2_API dav2_status DAV2_CALL dav2_get_network_shape(int32_t image_width, int32_t image_height,
                                                      int32_t input_size, dav2_image_shape* network_shape);
DAV2_API dav2_status DAV2_CALL dav2_get_inferbridge_shape(int32_t image_width, int32_t image_height,
                                                          int32_t input_size, dav2_image_shape* output_shape);

/* src/dav2.cpp:158-213: validates options, creates the executor (here the
 * CUDA executor of src/executor_factory.cpp's slot). */
DAV2_API dav2_status DAV2_CALL dav2_create(const char* model_path_utf8, const dav2_create_options* options,
                                           dav2_context** context);
DAV2_API dav2_status DAV2_CALL dav2_get_model_info(const dav2_context* context, dav2_model_info* info);
DAV2_API dav2_status DAV2_CALL dav2_prepare(dav2_context* context, int32_t image_width, int32_t image_height,
                                            int32_t input_size);
DAV2_API void DAV2_CALL dav2_destroy(dav2_context* context);

DAV2_API dav2_status DAV2_CALL dav2_probe_gpu_capabilities(int32_t vulkan_device_index,
                                                           dav2_gpu_capabilities* capabilities);
DAV2_API dav2_status DAV2_CALL dav2_get_gpu_capabilities(const dav2_context* context,
                                                         dav2_gpu_capabilities* capabilities);
DAV2_API dav2_status DAV2_CALL dav2_get_transfer_counters(const dav2_context* context,
                                                          dav2_transfer_counters* counters);

/* Graphics-API interop (D3D12 / Metal): DAV2_STATUS_UNSUPPORTED here. */
DAV2_API dav2_status DAV2_CALL dav2_submit_d3d12(dav2_context* context, const dav2_d3d12_submit_request* request,
                                                 dav2_gpu_job** job);
DAV2_API dav2_status DAV2_CALL dav2_submit_d3d12_texture(dav2_context* context,
                                                         const dav2_d3d12_texture_submit_request* request,
                                                         dav2_gpu_job** job);
DAV2_API dav2_status DAV2_CALL dav2_submit_d3d12_texture_binding(dav2_context* context,
                                                                 const dav2_d3d12_texture_binding_request* request,
                                                                 dav2_gpu_job** job);
DAV2_API dav2_status DAV2_CALL dav2_submit_metal_texture_binding(dav2_context* context,
                                                                 const dav2_metal_texture_binding_request* request,
                                                                 dav2_gpu_job** job);
DAV2_API dav2_status DAV2_CALL dav2_gpu_job_poll(const dav2_gpu_job* job, dav2_gpu_job_status* status);
DAV2_API dav2_status DAV2_CALL dav2_gpu_job_cancel(dav2_gpu_job* job);
DAV2_API void DAV2_CALL dav2_gpu_job_release(dav2_gpu_job* job);
DAV2_API dav2_status DAV2_CALL dav2_gpu_output_acquire(dav2_gpu_job* job, uint32_t output_index,
                                                       dav2_d3d12_output_descriptor* descriptor,
                                                       dav2_gpu_output_lease** lease);
DAV2_API dav2_status DAV2_CALL dav2_gpu_texture_output_acquire(dav2_gpu_job* job, uint32_t output_index,
                                                               dav2_d3d12_texture_output_descriptor* descriptor,
                                                               dav2_gpu_output_lease** lease);
DAV2_API void DAV2_CALL dav2_gpu_output_release(dav2_gpu_output_lease* lease);

/* src/dav2.cpp:630-668: BGR8 (cv2.imread layout) -> depth per source pixel.
 * Preprocessing (bicubic + ImageNet normalization) runs on the device. */
DAV2_API dav2_status DAV2_CALL dav2_infer_bgr8(dav2_context* context, const uint8_t* bgr, int32_t image_width,
                                               int32_t image_height, ptrdiff_t row_stride_bytes, int32_t input_size,
                                               float* output_depth, size_t output_count);

/* src/dav2.cpp:754-804: InferBridge BGRA contract (nearest resize, min/max
 * normalized output at the transposed network dimensions). */
DAV2_API dav2_status DAV2_CALL dav2_inferbridge_bgra8_f32(dav2_context* context, const uint8_t* bgra,
                                                          int32_t image_width, int32_t image_height,
                                                          ptrdiff_t row_stride_bytes, int32_t input_size,
                                                          float* output_depth, size_t output_count);

/* src/dav2.cpp:603-628: normalized planar RGB f32, batch of one. */
DAV2_API dav2_status DAV2_CALL dav2_infer_tensor_f32(dav2_context* context, const float* normalized_rgb_chw,
                                                     int32_t network_width, int32_t network_height,
                                                     float* output_depth, size_t output_count);

/* EXTENSION: dav2_infer_tensor_f32 for `batch` images stored back to back
 * (host memory); output is batch * network_width * network_height floats. */
DAV2_API dav2_status DAV2_CALL dav2_infer_tensor_f32_batch(dav2_context* context, const float* normalized_rgb_chw,
                                                           uint32_t batch, int32_t network_width,
                                                           int32_t network_height, float* output_depth,
                                                           size_t output_count);

/* EXTENSION: dav2_infer_bgr8 for `batch` equally sized host images
 * (image_stride_bytes apart); output is batch * image_width * image_height
 * floats, image after image. */
DAV2_API dav2_status DAV2_CALL dav2_infer_bgr8_batch(dav2_context* context, const uint8_t* bgr, uint32_t batch,
                                                     int32_t image_width, int32_t image_height,
                                                     ptrdiff_t row_stride_bytes, ptrdiff_t image_stride_bytes,
                                                     int32_t input_size, float* output_depth, size_t output_count);

/* EXTENSION: the headless device-resident submit path (the CUDA analogue
 * of the reference's GPU submit path without graphics interop): device BGR8
 * images in, device depth out (batch * image_width * image_height floats).
 * stream NULL = the context's own stream, and the call waits for the work to
 * finish. A non-NULL cudaStream_t makes the call return as soon as the work
 * is queued on that stream; a device-side failure of that work is reported
 * by the context's next call or by dav2_synchronize. Calls of one context on
 * different streams run one after another on the device (each waits for the
 * previous call's work), because they share the context's buffers. */
DAV2_API dav2_status DAV2_CALL dav2_infer_device_bgr8_batch(dav2_context* context, const uint8_t* device_bgr,
                                                            uint32_t batch, int32_t image_width,
                                                            int32_t image_height, ptrdiff_t row_stride_bytes,
                                                            ptrdiff_t image_stride_bytes, int32_t input_size,
                                                            float* device_depth, void* stream);

/* EXTENSION: the high-resolution video path: `batch` device BGR8 frames of
 * image_width x image_height, each resized bilinearly (half-pixel centres,
 * align_corners=False) to a square network_size x network_size input
 * (network_size a multiple of 14), through the graph, and the depth resized
 * back (align-corners bilinear, as Executor::infer_resized does) to
 * image_width x image_height in device_depth. Stream semantics as
 * dav2_infer_device_bgr8_batch. */
DAV2_API dav2_status DAV2_CALL dav2_infer_device_frames_bgr8(dav2_context* context, const uint8_t* device_bgr,
                                                             uint32_t batch, int32_t image_width,
                                                             int32_t image_height, ptrdiff_t row_stride_bytes,
                                                             ptrdiff_t image_stride_bytes, int32_t network_size,
                                                             float* device_depth, void* stream);

/* EXTENSION: the headless analogue of the reference's GPU submit path
 * (src/vulkan_executor.cpp:656-812, dav2_submit_d3d12 without the D3D12
 * interop): `batch` device images of packed 8-bit pixels (pixel_format
 * DAV2_GPU_PIXEL_BGRA8 or DAV2_GPU_PIXEL_RGBA8, row_stride_bytes and
 * image_stride_bytes multiples of 4) -> GPU bicubic preprocessing to the
 * network shape (preprocess_rgba.glsl) -> graph -> per-image min/max
 * normalization at the network resolution (normalize_relative, or
 * normalize_metric with the 25 m presentation span for a metric model) ->
 * align-corners bilinear expansion to image_width x image_height in
 * device_output. Stream semantics as dav2_infer_device_bgr8_batch. */
DAV2_API dav2_status DAV2_CALL dav2_submit_device_pixels(dav2_context* context, const uint8_t* device_pixels,
                                                         uint32_t batch, int32_t image_width, int32_t image_height,
                                                         ptrdiff_t row_stride_bytes, ptrdiff_t image_stride_bytes,
                                                         dav2_gpu_pixel_format pixel_format, int32_t input_size,
                                                         float* device_output, void* stream);

/* EXTENSION: number of device kernels the context has launched so far
 * (each CUDA-graph replay counts its kernel nodes). */
DAV2_API dav2_status DAV2_CALL dav2_get_kernel_launch_count(const dav2_context* context, uint64_t* launches);

/* EXTENSION: per-operation device timing of one batch through the network
 * (the CUDA counterpart of the reference's DAV2_VULKAN_PROFILE=1 dispatch
 * timer): runs the graph once without capture, with an event after every
 * launch on its stream, and writes {"ops": [{"name", "ms"}...], "total_ms"}
 * as JSON into `json` (capacity bytes). */
DAV2_API dav2_status DAV2_CALL dav2_profile_operations(dav2_context* context, uint32_t batch, int32_t network_width,
                                                       int32_t network_height, char* json, size_t capacity);

/* EXTENSION (stage probes; the analogue of the reference's
 * tools/dav2_encoder_probe.cpp stage dumps, used by the block- and head-level
 * parity tests): run one stage of the context's (batch, network_width,
 * network_height) graph — the same kernels in the same order as the
 * captured graph — on host inputs, synchronously. tokens = 1 +
 * (network_width/14)(network_height/14).
 * dav2_probe_encoder_block: transformer block `block` on residual-stream
 *   rows x_in ([batch*tokens][embedding] f32) -> x_out (same shape). At int8
 *   precision, ln1_codes ([batch*tokens][embedding]) and ln1_scales
 *   ([batch*tokens]) may be non-NULL and receive the block's first LayerNorm
 *   as the int8 codes and f32 row scales that its QKV GEMM reads.
 * dav2_probe_head: the four tap LayerNorms and the DPT head from the tapped
 *   residual streams tap_x ([4][batch*tokens][embedding] f32) -> depth
 *   ([batch][network_height][network_width]). */
DAV2_API dav2_status DAV2_CALL dav2_probe_encoder_block(dav2_context* context, uint32_t batch, int32_t network_width,
                                                        int32_t network_height, uint32_t block, const float* x_in,
                                                        float* x_out, int8_t* ln1_codes, float* ln1_scales);
DAV2_API dav2_status DAV2_CALL dav2_probe_head(dav2_context* context, uint32_t batch, int32_t network_width,
                                               int32_t network_height, const float* tap_x, float* depth);

/* EXTENSION: waits for all work the context queued, on any stream; returns
 * DAV2_STATUS_INFERENCE_FAILED when that work hit a device-side failure (a
 * bounded pipeline wait that gave up). */
DAV2_API dav2_status DAV2_CALL dav2_synchronize(dav2_context* context);

#ifdef __cplusplus
}
#endif

#endif
