// The public C ABI (include/depth_anything_v2.h) over the CUDA executor.
// Argument checks, their order, the status mapping of exceptions and the
// thread-local last-error string follow src/dav2.cpp:71-90 and 96-668. The
// runtime throws dav2::StatusError where the public status is fixed at the
// throw site (model I/O / format, no device, device-side failure,
// unsupported precision); protect() maps the class, never the message.
#include <algorithm>
#include <cstddef>
#include <cstring>
#include <memory>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "depth_anything_v2.h"
#include "executor.h"
#include "image.h"
#include "status_error.h"

struct dav2_context {
    std::shared_ptr<dav2::Executor> executor;
    std::vector<float> image_input;
    std::vector<float> image_output;
};

namespace {

thread_local std::string last_error;

class ApiError final : public std::runtime_error {
public:
    ApiError(dav2_status status, const char* message) : std::runtime_error(message), status_(status) {}
    dav2_status status() const { return status_; }

private:
    dav2_status status_;
};

dav2_status fail(dav2_status status, const char* message) {
    last_error = message ? message : "";
    return status;
}

template <typename F>
dav2_status protect(F&& f) {
    try {
        f();
        last_error.clear();
        return DAV2_STATUS_OK;
    } catch (const ApiError& e) {
        return fail(e.status(), e.what());
    } catch (const dav2::StatusError& e) {
        return fail(e.status(), e.what());
    } catch (const std::bad_alloc&) {
        return fail(DAV2_STATUS_OUT_OF_MEMORY, "out of memory");
    } catch (const std::invalid_argument& e) {
        return fail(DAV2_STATUS_INVALID_ARGUMENT, e.what());
    } catch (const std::exception& e) {
        return fail(DAV2_STATUS_INTERNAL_ERROR, e.what());
    } catch (...) {
        return fail(DAV2_STATUS_INTERNAL_ERROR, "unknown internal error");
    }
}

bool supported_encoder(dav2_encoder e) {
    return e == DAV2_ENCODER_VITS || e == DAV2_ENCODER_VITB || e == DAV2_ENCODER_VITL;
}

}  // namespace

extern "C" {

DAV2_API uint32_t DAV2_CALL dav2_abi_version(void) { return DAV2_ABI_VERSION; }

DAV2_API const char* DAV2_CALL dav2_version_string(void) { return "0.1.0-b200"; }

DAV2_API const char* DAV2_CALL dav2_status_string(dav2_status status) {
    switch (status) {
        case DAV2_STATUS_OK: return "ok";
        case DAV2_STATUS_INVALID_ARGUMENT: return "invalid argument";
        case DAV2_STATUS_MODEL_IO: return "model I/O error";
        case DAV2_STATUS_MODEL_FORMAT: return "invalid model format";
        case DAV2_STATUS_VULKAN_UNAVAILABLE: return "Vulkan unavailable";
        case DAV2_STATUS_OUT_OF_MEMORY: return "out of memory";
        case DAV2_STATUS_INFERENCE_FAILED: return "inference failed";
        case DAV2_STATUS_BUFFER_TOO_SMALL: return "buffer too small";
        case DAV2_STATUS_UNSUPPORTED: return "unsupported";
        case DAV2_STATUS_INTERNAL_ERROR: return "internal error";
        case DAV2_STATUS_INVALID_STATE: return "invalid state";
        case DAV2_STATUS_CANCELLED: return "cancelled";
        default: return "unknown status";
    }
}

DAV2_API const char* DAV2_CALL dav2_last_error(void) { return last_error.c_str(); }

DAV2_API dav2_status DAV2_CALL dav2_get_network_shape(int32_t w, int32_t h, int32_t input_size,
                                                      dav2_image_shape* shape) {
    if (!shape) return fail(DAV2_STATUS_INVALID_ARGUMENT, "network_shape is null");
    return protect([&] {
        const dav2::ImageShape s = dav2::network_shape(w, h, input_size);
        shape->width = s.width;
        shape->height = s.height;
    });
}

DAV2_API dav2_status DAV2_CALL dav2_get_inferbridge_shape(int32_t w, int32_t h, int32_t input_size,
                                                          dav2_image_shape* shape) {
    if (!shape) return fail(DAV2_STATUS_INVALID_ARGUMENT, "output_shape is null");
    return protect([&] {
        const dav2::ImageShape s = dav2::network_shape(w, h, input_size);
        shape->width = s.height;
        shape->height = s.width;
    });
}

DAV2_API dav2_status DAV2_CALL dav2_create(const char* path, const dav2_create_options* options,
                                           dav2_context** context) {
    if (!context) return fail(DAV2_STATUS_INVALID_ARGUMENT, "context is null");
    *context = nullptr;
    if (!path || path[0] == '\0') return fail(DAV2_STATUS_INVALID_ARGUMENT, "model_path_utf8 is empty");
    constexpr size_t legacy = offsetof(dav2_create_options, cache_path_utf8);
    if (!options || options->struct_size < legacy) return fail(DAV2_STATUS_INVALID_ARGUMENT, "invalid create options");
    if (options->abi_version != DAV2_ABI_VERSION) return fail(DAV2_STATUS_INVALID_ARGUMENT, "ABI version mismatch");
    if (!supported_encoder(options->encoder)) return fail(DAV2_STATUS_INVALID_ARGUMENT, "unsupported encoder");
    constexpr uint32_t supported = DAV2_CREATE_FORCE_FP32 | DAV2_CREATE_FORCE_FP32_WEIGHTS |
                                   DAV2_CREATE_FORCE_FP32_ATTENTION | DAV2_CREATE_FORCE_FP16 |
                                   DAV2_CREATE_FORCE_INT8 | DAV2_CREATE_FORCE_METAL | DAV2_CREATE_FORCE_VULKAN |
                                   DAV2_CREATE_FORCE_BF16;
    if (options->flags & ~supported) return fail(DAV2_STATUS_INVALID_ARGUMENT, "unsupported create flags");
    const uint32_t prec = options->flags & (DAV2_CREATE_FORCE_FP32 | DAV2_CREATE_FORCE_FP16 | DAV2_CREATE_FORCE_INT8 |
                                            DAV2_CREATE_FORCE_BF16);
    if (prec && (prec & (prec - 1)))
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "multiple DAV2 execution precisions were requested");
    return protect([&] {
        auto ctx = std::make_unique<dav2_context>();
        const std::string cache = options->struct_size >= sizeof(dav2_create_options) && options->cache_path_utf8
                                      ? options->cache_path_utf8
                                      : "";
        ctx->executor = std::shared_ptr<dav2::Executor>(
            dav2::create_executor(path, options->encoder, options->vulkan_device_index, options->flags, cache));
        *context = ctx.release();
    });
}

DAV2_API dav2_status DAV2_CALL dav2_prepare(dav2_context* context, int32_t w, int32_t h, int32_t input_size) {
    if (!context || w <= 0 || h <= 0 || input_size <= 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "invalid prepare request");
    return protect([&] { context->executor->prepare(w, h, input_size); });
}

DAV2_API void DAV2_CALL dav2_destroy(dav2_context* context) { delete context; }

DAV2_API dav2_status DAV2_CALL dav2_get_model_info(const dav2_context* context, dav2_model_info* info) {
    if (!context || !info || info->struct_size < sizeof(*info))
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "invalid model info query");
    return protect([&] {
        const float depth = context->executor->metric_max_depth();
        *info = {};
        info->struct_size = sizeof(*info);
        info->abi_version = DAV2_ABI_VERSION;
        info->encoder = context->executor->encoder();
        info->is_metric = depth > 0.0f ? 1u : 0u;
        info->metric_max_depth = depth;
    });
}

DAV2_API dav2_status DAV2_CALL dav2_probe_gpu_capabilities(int32_t device, dav2_gpu_capabilities* caps) {
    if (!caps) return fail(DAV2_STATUS_INVALID_ARGUMENT, "GPU capabilities are null");
    if (caps->struct_size < sizeof(*caps) || device < 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "invalid GPU capability probe");
    return protect([&] {
        const dav2::GpuCapabilities c = dav2::probe_gpu_capabilities(device);
        *caps = {};
        caps->struct_size = sizeof(*caps);
        caps->abi_version = DAV2_ABI_VERSION;
        caps->flags = c.flags;
        caps->adapter_luid = c.adapter_luid;
        caps->maximum_in_flight_jobs = c.maximum_in_flight_jobs;
    });
}

DAV2_API dav2_status DAV2_CALL dav2_get_gpu_capabilities(const dav2_context* context, dav2_gpu_capabilities* caps) {
    if (!context || !caps) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null GPU capability argument");
    if (caps->struct_size < sizeof(*caps))
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "GPU capabilities struct is too small");
    return protect([&] {
        const dav2::GpuCapabilities c = context->executor->gpu_capabilities();
        *caps = {};
        caps->struct_size = sizeof(*caps);
        caps->abi_version = DAV2_ABI_VERSION;
        caps->flags = c.flags;
        caps->adapter_luid = c.adapter_luid;
        caps->maximum_in_flight_jobs = c.maximum_in_flight_jobs;
    });
}

DAV2_API dav2_status DAV2_CALL dav2_get_transfer_counters(const dav2_context* context,
                                                          dav2_transfer_counters* counters) {
    if (!context || !counters || counters->struct_size < sizeof(*counters))
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "invalid transfer counter query");
    return protect([&] {
        uint64_t up = 0, down = 0;
        context->executor->transfer_counters(up, down);
        *counters = {};
        counters->struct_size = sizeof(*counters);
        counters->tensor_upload_bytes = up;
        counters->tensor_download_bytes = down;
    });
}

// ---- graphics-API interop: not part of this library
#define DAV2_UNSUPPORTED_SUBMIT(fn, req_t)                                                                    \
    DAV2_API dav2_status DAV2_CALL fn(dav2_context* context, const req_t* request, dav2_gpu_job** job) {     \
        if (!context || !request || !job) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null submit argument"); \
        *job = nullptr;                                                                                       \
        return fail(DAV2_STATUS_UNSUPPORTED, "graphics-API interop is not available in the CUDA executor");   \
    }
DAV2_UNSUPPORTED_SUBMIT(dav2_submit_d3d12, dav2_d3d12_submit_request)
DAV2_UNSUPPORTED_SUBMIT(dav2_submit_d3d12_texture, dav2_d3d12_texture_submit_request)
DAV2_UNSUPPORTED_SUBMIT(dav2_submit_d3d12_texture_binding, dav2_d3d12_texture_binding_request)
DAV2_UNSUPPORTED_SUBMIT(dav2_submit_metal_texture_binding, dav2_metal_texture_binding_request)
#undef DAV2_UNSUPPORTED_SUBMIT

DAV2_API dav2_status DAV2_CALL dav2_gpu_job_poll(const dav2_gpu_job* job, dav2_gpu_job_status* status) {
    if (!job || !status) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null GPU job poll argument");
    return fail(DAV2_STATUS_UNSUPPORTED, "no GPU jobs exist in the CUDA executor");
}
DAV2_API dav2_status DAV2_CALL dav2_gpu_job_cancel(dav2_gpu_job* job) {
    if (!job) return fail(DAV2_STATUS_INVALID_ARGUMENT, "GPU job is null");
    return fail(DAV2_STATUS_UNSUPPORTED, "no GPU jobs exist in the CUDA executor");
}
DAV2_API void DAV2_CALL dav2_gpu_job_release(dav2_gpu_job*) {}
DAV2_API dav2_status DAV2_CALL dav2_gpu_output_acquire(dav2_gpu_job* job, uint32_t, dav2_d3d12_output_descriptor* d,
                                                       dav2_gpu_output_lease** lease) {
    if (!job || !d || !lease) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null GPU output acquire argument");
    *lease = nullptr;
    return fail(DAV2_STATUS_UNSUPPORTED, "no GPU jobs exist in the CUDA executor");
}
DAV2_API dav2_status DAV2_CALL dav2_gpu_texture_output_acquire(dav2_gpu_job* job, uint32_t,
                                                               dav2_d3d12_texture_output_descriptor* d,
                                                               dav2_gpu_output_lease** lease) {
    if (!job || !d || !lease) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null GPU texture output acquire argument");
    *lease = nullptr;
    return fail(DAV2_STATUS_UNSUPPORTED, "no GPU jobs exist in the CUDA executor");
}
DAV2_API void DAV2_CALL dav2_gpu_output_release(dav2_gpu_output_lease*) {}

// ---- inference
DAV2_API dav2_status DAV2_CALL dav2_infer_tensor_f32(dav2_context* context, const float* chw, int32_t w, int32_t h,
                                                     float* depth, size_t count) {
    if (!context || !chw || !depth) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    if (w <= 0 || h <= 0 || w % 14 != 0 || h % 14 != 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "network dimensions must be positive multiples of 14");
    if (count < size_t(w) * size_t(h)) return fail(DAV2_STATUS_BUFFER_TOO_SMALL, "output buffer is too small");
    return protect([&] { context->executor->infer(chw, w, h, depth); });
}

DAV2_API dav2_status DAV2_CALL dav2_infer_tensor_f32_batch(dav2_context* context, const float* chw, uint32_t batch,
                                                           int32_t w, int32_t h, float* depth, size_t count) {
    if (!context || !chw || !depth || batch == 0) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    if (w <= 0 || h <= 0 || w % 14 != 0 || h % 14 != 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "network dimensions must be positive multiples of 14");
    if (count < size_t(batch) * size_t(w) * size_t(h))
        return fail(DAV2_STATUS_BUFFER_TOO_SMALL, "output buffer is too small");
    return protect([&] { context->executor->infer_batch(chw, int(batch), w, h, depth); });
}

DAV2_API dav2_status DAV2_CALL dav2_infer_bgr8(dav2_context* context, const uint8_t* bgr, int32_t w, int32_t h,
                                               ptrdiff_t stride, int32_t input_size, float* depth, size_t count) {
    if (!context || !bgr || !depth) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    const size_t required = w > 0 && h > 0 ? size_t(w) * size_t(h) : 0;
    if (count < required) return fail(DAV2_STATUS_BUFFER_TOO_SMALL, "output buffer is too small");
    return protect([&] {
        dav2::network_shape(w, h, input_size);  // argument validation
        context->executor->infer_bgr8(bgr, 1, w, h, stride, 0, input_size, depth, false, nullptr);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_infer_bgr8_batch(dav2_context* context, const uint8_t* bgr, uint32_t batch,
                                                     int32_t w, int32_t h, ptrdiff_t stride, ptrdiff_t image_stride,
                                                     int32_t input_size, float* depth, size_t count) {
    if (!context || !bgr || !depth || batch == 0) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    const size_t required = w > 0 && h > 0 ? size_t(batch) * size_t(w) * size_t(h) : 0;
    if (count < required) return fail(DAV2_STATUS_BUFFER_TOO_SMALL, "output buffer is too small");
    return protect([&] {
        dav2::network_shape(w, h, input_size);
        context->executor->infer_bgr8(bgr, int(batch), w, h, stride, image_stride, input_size, depth, false, nullptr);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_infer_device_bgr8_batch(dav2_context* context, const uint8_t* bgr, uint32_t batch,
                                                            int32_t w, int32_t h, ptrdiff_t stride,
                                                            ptrdiff_t image_stride, int32_t input_size, float* depth,
                                                            void* stream) {
    if (!context || !bgr || !depth || batch == 0) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    return protect([&] {
        dav2::network_shape(w, h, input_size);
        context->executor->infer_bgr8(bgr, int(batch), w, h, stride, image_stride, input_size, depth, true, stream);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_infer_device_frames_bgr8(dav2_context* context, const uint8_t* bgr, uint32_t batch,
                                                             int32_t w, int32_t h, ptrdiff_t stride,
                                                             ptrdiff_t image_stride, int32_t network_size,
                                                             float* depth, void* stream) {
    if (!context || !bgr || !depth || batch == 0) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    return protect([&] {
        context->executor->infer_frames_bgr8(bgr, int(batch), w, h, stride, image_stride, network_size, depth, stream);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_submit_device_pixels(dav2_context* context, const uint8_t* pixels, uint32_t batch,
                                                         int32_t w, int32_t h, ptrdiff_t stride, ptrdiff_t image_stride,
                                                         dav2_gpu_pixel_format format, int32_t input_size,
                                                         float* output, void* stream) {
    if (!context || !pixels || !output || batch == 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "null submit argument");
    if (format != DAV2_GPU_PIXEL_BGRA8 && format != DAV2_GPU_PIXEL_RGBA8)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "unsupported pixel format");
    return protect([&] {
        dav2::network_shape(w, h, input_size);
        context->executor->submit_pixels(pixels, int(batch), w, h, stride, image_stride, format == DAV2_GPU_PIXEL_RGBA8,
                                         input_size, output, stream);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_get_kernel_launch_count(const dav2_context* context, uint64_t* launches) {
    if (!context || !launches) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null launch count argument");
    return protect([&] { *launches = context->executor->kernel_launches(); });
}

DAV2_API dav2_status DAV2_CALL dav2_profile_operations(dav2_context* context, uint32_t batch, int32_t w, int32_t h,
                                                       char* json, size_t capacity) {
    if (!context || !json || capacity == 0 || batch == 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "invalid profile request");
    return protect([&] {
        const std::string s = context->executor->profile_json(int(batch), w, h);
        if (s.size() + 1 > capacity) throw ApiError(DAV2_STATUS_BUFFER_TOO_SMALL, "profile buffer is too small");
        std::memcpy(json, s.c_str(), s.size() + 1);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_probe_encoder_block(dav2_context* context, uint32_t batch, int32_t w, int32_t h,
                                                        uint32_t block, const float* x_in, float* x_out,
                                                        int8_t* ln1_codes, float* ln1_scales) {
    if (!context || !x_in || !x_out || batch == 0) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null probe argument");
    if (w <= 0 || h <= 0 || w % 14 != 0 || h % 14 != 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "network dimensions must be positive multiples of 14");
    return protect([&] {
        context->executor->probe_block(int(batch), w, h, int(block), x_in, x_out, ln1_codes, ln1_scales);
    });
}

DAV2_API dav2_status DAV2_CALL dav2_probe_head(dav2_context* context, uint32_t batch, int32_t w, int32_t h,
                                               const float* tap_x, float* depth) {
    if (!context || !tap_x || !depth || batch == 0) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null probe argument");
    if (w <= 0 || h <= 0 || w % 14 != 0 || h % 14 != 0)
        return fail(DAV2_STATUS_INVALID_ARGUMENT, "network dimensions must be positive multiples of 14");
    return protect([&] { context->executor->probe_head(int(batch), w, h, tap_x, depth); });
}

DAV2_API dav2_status DAV2_CALL dav2_synchronize(dav2_context* context) {
    if (!context) return fail(DAV2_STATUS_INVALID_ARGUMENT, "context is null");
    return protect([&] { context->executor->synchronize(); });
}

DAV2_API dav2_status DAV2_CALL dav2_inferbridge_bgra8_f32(dav2_context* context, const uint8_t* bgra, int32_t w,
                                                          int32_t h, ptrdiff_t stride, int32_t input_size,
                                                          float* depth, size_t count) {
    if (!context || !bgra || !depth) return fail(DAV2_STATUS_INVALID_ARGUMENT, "null inference argument");
    return protect([&] {
        const dav2::ImageShape upstream = dav2::network_shape(w, h, input_size);
        const dav2::ImageShape shape{upstream.height, upstream.width};
        const size_t required = size_t(shape.width) * shape.height;
        if (count < required) throw ApiError(DAV2_STATUS_BUFFER_TOO_SMALL, "output buffer is too small");
        dav2::preprocess_inferbridge_bgra8(bgra, w, h, stride, shape, context->image_input);
        context->image_output.resize(required);
        context->executor->infer(context->image_input.data(), shape.width, shape.height,
                                 context->image_output.data());
        // min/max normalization on the host (src/dav2.cpp:787-803)
        const auto mm = std::minmax_element(context->image_output.begin(), context->image_output.end());
        const float lo = *mm.first;
        const float span = context->executor->metric_max_depth() > 0.0f ? 25.0f - lo : *mm.second - lo;
        if (!(span > 0.0f)) {
            std::fill_n(depth, required, 0.0f);
            return;
        }
        for (size_t i = 0; i < required; ++i) depth[i] = (context->image_output[i] - lo) / span;
    });
}

}  // extern "C"
