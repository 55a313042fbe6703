// The executor plugin boundary: the reference's class Executor
// (src/executor.h:87-121) with its factory (src/executor_factory.cpp:7-53),
// served by the CUDA executor. The Linux DMA-BUF capture consumer base and
// the D3D12/Metal submit methods are not part of this interface (graphics
// interop is out of scope; the C ABI reports DAV2_STATUS_UNSUPPORTED for
// them). Batched and device-resident methods are B200 extensions.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>

#include "depth_anything_v2.h"

namespace dav2 {

struct GpuCapabilities {
    std::uint64_t flags = 0;
    std::uint64_t adapter_luid = 0;
    std::uint32_t maximum_in_flight_jobs = 0;
};

class Executor {
public:
    virtual ~Executor() = default;
    virtual void prepare(int image_width, int image_height, int input_size) = 0;
    // normalized planar RGB, batch of one, host memory (src/executor.h:97-110)
    virtual void infer(const float* normalized_rgb_chw, int width, int height, float* depth) = 0;
    virtual void infer_resized(const float* normalized_rgb_chw, int width, int height, float* depth,
                               int output_width, int output_height) = 0;
    virtual GpuCapabilities gpu_capabilities() const = 0;
    virtual void transfer_counters(std::uint64_t& upload_bytes, std::uint64_t& download_bytes) const = 0;
    virtual dav2_encoder encoder() const = 0;
    virtual float metric_max_depth() const = 0;

    // ---- extensions
    virtual void infer_batch(const float* normalized_rgb_chw, int batch, int width, int height,
                             float* depth) = 0;
    // BGR8 images (host or device memory) -> depth at the source size.
    virtual void infer_bgr8(const std::uint8_t* bgr, int batch, int width, int height, std::ptrdiff_t row_stride,
                            std::ptrdiff_t image_stride, int input_size, float* depth, bool device_memory,
                            void* stream) = 0;
    // Video frames (device memory): BGR8 -> bilinear (half-pixel) to a square
    // network_size input -> graph -> depth resized to the frame size.
    virtual void infer_frames_bgr8(const std::uint8_t* bgr, int batch, int width, int height,
                                   std::ptrdiff_t row_stride, std::ptrdiff_t image_stride, int network_size,
                                   float* depth, void* stream) = 0;
    // The headless GPU submit path (src/vulkan_executor.cpp:656-812 without
    // graphics interop): packed BGRA8/RGBA8 device images -> bicubic ->
    // graph -> per-image min/max normalization -> output at the image size.
    virtual void submit_pixels(const std::uint8_t* pixels, int batch, int width, int height,
                               std::ptrdiff_t row_stride, std::ptrdiff_t image_stride, bool rgba, int input_size,
                               float* output, void* stream) = 0;
    virtual void synchronize() = 0;
    // Kernels this executor has launched (graph kernel nodes per replay included).
    virtual std::uint64_t kernel_launches() const = 0;
    // Runs the (batch, width, height) graph once without graph capture,
    // timing every launch with events on its stream; returns JSON.
    virtual std::string profile_json(int batch, int width, int height) = 0;
    // Stage probes (the analogue of the reference's tools/dav2_encoder_probe.cpp
    // stage dumps): run one stage of the (batch, width, height) graph — the
    // same launches the captured graph makes — on host inputs.
    //   probe_block: transformer block `block` on residual rows x_in
    //     ([batch*tokens][embedding] f32) -> x_out; at int8 precision
    //     ln1_codes / ln1_scales (nullable) receive the block's first
    //     LayerNorm as the int8 codes and f32 row scales its GEMM reads.
    //   probe_head: the tap LayerNorms and the DPT head from the four tapped
    //     residual streams ([4][batch*tokens][embedding]) -> depth
    //     [batch][height][width].
    virtual void probe_block(int batch, int width, int height, int block, const float* x_in, float* x_out,
                             std::int8_t* ln1_codes, float* ln1_scales) = 0;
    virtual void probe_head(int batch, int width, int height, const float* tap_x, float* depth) = 0;
};

// src/executor_factory.cpp:7-42: FORCE_METAL / FORCE_VULKAN both set is an
// invalid argument; otherwise the CUDA executor on device `device_index`.
std::unique_ptr<Executor> create_executor(const std::string& model_path, dav2_encoder encoder, int device_index,
                                          std::uint32_t flags, const std::string& cache_path);
GpuCapabilities probe_gpu_capabilities(int device_index);

}  // namespace dav2
