// CUDA executor: the DINOv2 encoder (src/encoder.cpp:322-597) and the DPT
// head (src/dpt.cpp:628-863) as a sequence of sm_100a kernels on one stream,
// captured once per input shape into a CUDA graph.
//
// Layouts in HBM (per batch of B images, T = 1 + pw*ph tokens):
//   residual stream  f32 [B*T, D]           (in-place LayerScale updates)
//   GEMM activations int8 codes [rows, K] + f32 row scales   (int8 path)
//                    f16 [rows, K]                            (fp16 path)
//   QKV / attention  f16 [B*T, 3D] / [B*T, D]
//   DPT feature maps channels-last f16 [B][h][w][Cp], Cp = channels rounded
//                    up to 64 (zero pad) so the implicit-GEMM convolutions
//                    can read 128-byte channel blocks with TMA
//   depth            f32 [B][H][W]
// Precision routing follows the reference (src/encoder.cpp:255-303,
// src/dpt.cpp:479-535): in int8 mode the transformer linears, the patch
// embedding, the DPT projections and resize layers use per-row int8
// activations x per-output-channel int8 weights; attention and the DPT
// refinement convolutions run with f16 operands (the reference's fp16
// refinement precision); every accumulation is f32 / s32.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "executor.h"
#include "image.h"
#include "launch.h"
#include "model_file.h"
#include "status_error.h"

namespace dav2 {
namespace {

using namespace dav2cuda;

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        if (e == cudaErrorMemoryAllocation) throw std::bad_alloc();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

void op(int rc, const char* what) {
    if (rc != 0) throw std::runtime_error(std::string(what) + ": " + dav2cuda_last_error());
}

constexpr uint32_t up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

// True when `p` is page-locked host memory the copy engines can read directly.
bool is_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost;
}

struct Arch {
    uint32_t d, heads, blocks, taps[4], f, oc[4];
};

Arch arch_for(dav2_encoder e) {
    switch (e) {
        case DAV2_ENCODER_VITS: return {384, 6, 12, {2, 5, 8, 11}, 64, {48, 96, 192, 384}};
        case DAV2_ENCODER_VITB: return {768, 12, 12, {2, 5, 8, 11}, 128, {96, 192, 384, 768}};
        case DAV2_ENCODER_VITL: return {1024, 16, 24, {4, 11, 17, 23}, 256, {256, 512, 1024, 1024}};
        default: throw std::invalid_argument("unsupported encoder");
    }
}

// Device memory: one cudaMalloc per region, bump-allocated, 256-byte aligned.
class Arena {
public:
    Arena() = default;
    Arena(const Arena&) = delete;
    Arena& operator=(const Arena&) = delete;
    ~Arena() {
        if (base_) cudaFree(base_);
    }
    void reserve(uint64_t bytes) {
        cuda_check(cudaMalloc(&base_, bytes), "cudaMalloc");
        cuda_check(cudaMemset(base_, 0, bytes), "cudaMemset");
        cap_ = bytes;
    }
    template <typename T>
    T* take(uint64_t bytes) {
        const uint64_t at = (used_ + 255) & ~uint64_t(255);
        if (base_ == nullptr) {  // sizing pass
            used_ = at + bytes;
            return nullptr;
        }
        if (at + bytes > cap_) throw std::runtime_error("arena overflow");
        used_ = at + bytes;
        return reinterpret_cast<T*>(static_cast<uint8_t*>(base_) + at);
    }
    uint64_t used() const { return used_; }
    // Ends a sizing pass: the next reserve() makes take() hand out memory.
    void rewind() { used_ = 0; }

private:
    void* base_ = nullptr;
    uint64_t cap_ = 0, used_ = 0;
};

struct Linear {
    void* w = nullptr;        // int8 codes [n][kp] or f16 [n][kp]
    float* s = nullptr;       // int8 row scales [n]
    const float* b = nullptr; // bias [n] (nullable)
    uint32_t n = 0, kp = 0;
};

struct Block {
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b, *ls1, *ls2;
    Linear qkv, proj, fc1, fc2;
};

struct RefineNet {
    Linear rcu[2][2];  // [unit][conv], f16 [F][9F]
    Linear out;        // f16 [F][F]
};

class CudaExecutor final : public Executor {
public:
    CudaExecutor(const std::string& path, dav2_encoder encoder, int device, uint32_t flags)
        : model_(path, encoder), encoder_(encoder), device_(device), arch_(arch_for(encoder)) {
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) throw_no_device("no CUDA device is available");
        if (device < 0 || device >= count) throw std::invalid_argument("CUDA device index out of range");
        int8_ = (flags & DAV2_CREATE_FORCE_INT8) != 0;
        bf16_ = (flags & DAV2_CREATE_FORCE_BF16) != 0;
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
        cuda_check(cudaEventCreateWithFlags(&done_, cudaEventDisableTiming), "cudaEventCreate");
        cuda_check(cudaEventCreateWithFlags(&err_event_, cudaEventDisableTiming), "cudaEventCreate");
        cuda_check(cudaMallocHost(&err_host_, sizeof(int)), "cudaMallocHost");
        *err_host_ = 0;
        model_.verify_crc();
        load_weights();
    }

    ~CudaExecutor() override {
        cudaSetDevice(device_);
        for (auto& [k, p] : plans_)
            if (p.graph) cudaGraphExecDestroy(p.graph);
        plans_.clear();
        if (staging_) cudaFree(staging_);
        if (host_in_) cudaFreeHost(host_in_);
        if (host_out_) cudaFreeHost(host_out_);
        if (err_host_) cudaFreeHost(err_host_);
        if (done_) cudaEventDestroy(done_);
        if (err_event_) cudaEventDestroy(err_event_);
        if (stream_) cudaStreamDestroy(stream_);
    }

    void prepare(int image_width, int image_height, int input_size) override {
        const ImageShape s = network_shape(image_width, image_height, input_size);
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        plan(1, s.width, s.height);
    }

    void infer(const float* chw, int w, int h, float* depth) override { infer_resized(chw, w, h, depth, w, h); }

    void infer_resized(const float* chw, int w, int h, float* depth, int ow, int oh) override {
        run_host_tensor(chw, 1, w, h, depth, ow, oh);
    }

    void infer_batch(const float* chw, int batch, int w, int h, float* depth) override {
        run_host_tensor(chw, batch, w, h, depth, w, h);
    }

    void infer_bgr8(const uint8_t* bgr, int batch, int w, int h, std::ptrdiff_t row_stride,
                    std::ptrdiff_t image_stride, int input_size, float* depth, bool device_memory,
                    void* user_stream) override {
        ImagesCall c{bgr, batch, w, h, row_stride, image_stride, {}, Source::kBgr8Bicubic, false, false,
                     depth, device_memory, user_stream};
        if (w > 0 && h > 0) c.net = network_shape(w, h, input_size);
        run_images(c);
    }

    void infer_frames_bgr8(const uint8_t* bgr, int batch, int w, int h, std::ptrdiff_t row_stride,
                           std::ptrdiff_t image_stride, int network_size, float* depth, void* stream) override {
        if (network_size <= 0 || network_size % 14)
            throw std::invalid_argument("network size must be a positive multiple of 14");
        ImagesCall c{bgr, batch, w, h, row_stride, image_stride, {network_size, network_size}, Source::kBgr8Bilinear,
                     false, false, depth, true, stream};
        run_images(c);
    }

    void submit_pixels(const uint8_t* pixels, int batch, int w, int h, std::ptrdiff_t row_stride,
                       std::ptrdiff_t image_stride, bool rgba, int input_size, float* output, void* stream) override {
        ImagesCall c{pixels, batch, w, h, row_stride, image_stride, {}, Source::kPixels32, rgba, true, output, true,
                     stream};
        if (w > 0 && h > 0) c.net = network_shape(w, h, input_size);
        run_images(c);
    }

    void probe_block(int batch, int w, int h, int block, const float* x_in, float* x_out, int8_t* codes,
                     float* scales) override {
        if (!x_in || !x_out || batch <= 0) throw std::invalid_argument("null probe argument");
        if (block < 0 || block >= int(arch_.blocks)) throw std::invalid_argument("block index out of range");
        if ((codes || scales) && !int8_)
            throw std::invalid_argument("LayerNorm codes exist only at int8 precision");
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        poll_device_error();
        Plan& p = plan(batch, w, h);
        order_after_previous_call(stream_);
        const uint64_t rows = uint64_t(batch) * p.T, D = arch_.d;
        cuda_check(cudaMemcpyAsync(p.x, x_in, rows * D * 4, cudaMemcpyHostToDevice, stream_), "H2D");
        if (codes || scales) {
            enqueue_ln1(p, uint32_t(block), stream_);
            if (codes) cuda_check(cudaMemcpyAsync(codes, p.xn, rows * D, cudaMemcpyDeviceToHost, stream_), "D2H");
            if (scales) cuda_check(cudaMemcpyAsync(scales, p.xn_s, rows * 4, cudaMemcpyDeviceToHost, stream_), "D2H");
        }
        enqueue_block(p, uint32_t(block), stream_);
        cuda_check(cudaMemcpyAsync(x_out, p.x, rows * D * 4, cudaMemcpyDeviceToHost, stream_), "D2H");
        queue_error_read(stream_);
        finish_call(stream_);
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        raise_device_error();
    }

    void probe_head(int batch, int w, int h, const float* tap_x, float* depth) override {
        if (!tap_x || !depth || batch <= 0) throw std::invalid_argument("null probe argument");
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        poll_device_error();
        Plan& p = plan(batch, w, h);
        order_after_previous_call(stream_);
        const uint64_t rows = uint64_t(batch) * p.T, D = arch_.d;
        for (int k = 0; k < 4; ++k) {
            cuda_check(cudaMemcpyAsync(p.x, tap_x + k * rows * D, rows * D * 4, cudaMemcpyHostToDevice, stream_),
                       "H2D");
            enqueue_tap(p, k, stream_);
        }
        op(launch_store_pointer(reinterpret_cast<void**>(p.depth_slot), p.depth, stream_), "store_pointer");
        enqueue_head(p, stream_);
        cuda_check(cudaMemcpyAsync(depth, p.depth, uint64_t(batch) * w * h * 4, cudaMemcpyDeviceToHost, stream_),
                   "D2H");
        queue_error_read(stream_);
        finish_call(stream_);
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        raise_device_error();
    }

    uint64_t kernel_launches() const override { return launches_; }
    std::string profile_json(int batch, int w, int h) override { return profile(batch, w, h); }

    void synchronize() override {
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        // everything queued by this context, on any stream, precedes done_
        cuda_check(cudaStreamWaitEvent(stream_, done_, 0), "wait");
        queue_error_read(stream_);
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        raise_device_error();
    }

    GpuCapabilities gpu_capabilities() const override {
        GpuCapabilities c;
        c.flags = DAV2_GPU_CAP_NO_HOST_PIXEL_STAGING | DAV2_GPU_CAP_NO_HOST_DEPTH_STAGING;
        c.maximum_in_flight_jobs = 1;
        return c;
    }

    void transfer_counters(uint64_t& up_bytes, uint64_t& down_bytes) const override {
        up_bytes = upload_bytes_;
        down_bytes = download_bytes_;
    }

    dav2_encoder encoder() const override { return encoder_; }
    float metric_max_depth() const override { return model_.metric_max_depth(); }

private:
    // ------------------------------------------------------------- images
    // Image entry points: packed 8-bit images (host or device memory) ->
    // GPU preprocessing to the network shape -> graph -> optional per-image
    // min/max normalization -> depth at the source size (resized on the
    // device when the network shape differs).
    enum class Source {
        kBgr8Bicubic,   // BGR8, OpenCV-exact bicubic (dav2_infer_bgr8, src/image.cpp:163-269)
        kBgr8Bilinear,  // BGR8, bilinear half-pixel to a square network input (video frames)
        kPixels32,      // BGRA8 / RGBA8 words, bicubic (preprocess_rgba.glsl; the GPU submit path)
    };
    struct ImagesCall {
        const uint8_t* pixels;
        int batch, w, h;
        std::ptrdiff_t row_stride, image_stride;
        ImageShape net;
        Source source;
        bool rgba;       // kPixels32 channel order
        bool normalize;  // min/max normalization at the network shape (submit path)
        float* out;
        bool device_memory;
        void* stream;
    };

    void run_images(const ImagesCall& c) {
        const std::ptrdiff_t bpp = c.source == Source::kPixels32 ? 4 : 3;
        if (!c.pixels || !c.out || c.batch <= 0 || c.w <= 0 || c.h <= 0 || c.row_stride < std::ptrdiff_t(c.w) * bpp ||
            (c.batch > 1 && c.image_stride < c.row_stride * c.h) ||
            (bpp == 4 && (c.row_stride % 4 || c.image_stride % 4)))
            throw std::invalid_argument("invalid source image");
        const ImageShape s = c.net;
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        poll_device_error();
        Plan& p = plan(c.batch, s.width, s.height);
        cudaStream_t st = c.stream ? static_cast<cudaStream_t>(c.stream) : stream_;
        order_after_previous_call(st);
        const int batch = c.batch, w = c.w, h = c.h;
        const uint64_t img_bytes = uint64_t(c.image_stride > 0 ? c.image_stride : c.row_stride * h);
        const uint64_t in_bytes = img_bytes * (batch - 1) + uint64_t(c.row_stride) * (h - 1) + uint64_t(w) * bpp;
        const uint8_t* src_dev = c.pixels;
        const bool pinned_in = !c.device_memory && is_pinned(c.pixels);
        const bool pinned_out = !c.device_memory && is_pinned(c.out);
        if (!c.device_memory) {
            ensure_staging(in_bytes);
            ensure_host(pinned_in ? 0 : in_bytes, pinned_out ? 0 : uint64_t(batch) * w * h * 4);
            const void* src = c.pixels;
            if (!pinned_in) {
                std::memcpy(host_in_, c.pixels, in_bytes);
                src = host_in_;
            }
            cuda_check(cudaMemcpyAsync(staging_, src, in_bytes, cudaMemcpyHostToDevice, st), "H2D");
            upload_bytes_ += in_bytes;
            src_dev = staging_;
        }
        const bool resize = w != s.width || h != s.height;
        // The graph's last convolution writes where the plan's slot points:
        // straight into the caller's device buffer when no resize follows.
        float* graph_out = c.device_memory && !resize ? c.out : p.depth;
        op(launch_store_pointer(reinterpret_cast<void**>(p.depth_slot), graph_out, st), "store_pointer");
        if (c.source == Source::kPixels32)
            op(launch_preprocess_u32_batched(p.image, reinterpret_cast<const uint32_t*>(src_dev), batch, w, h,
                                             uint32_t(c.row_stride / 4), img_bytes / 4, c.rgba ? 1u : 0u, s.width,
                                             s.height, st),
               "preprocess_u32");
        else
            op(launch_preprocess_bgr8(p.image, src_dev, batch, w, h, c.row_stride, img_bytes, s.width, s.height,
                                      c.source == Source::kBgr8Bilinear ? 1 : 0, st),
               "preprocess_bgr8");
        launches_ += 2;
        launch_plan(p, st);
        if (c.normalize) {
            // src/vulkan_executor.cpp:763-786: min/max at the network resolution,
            // relative [0,1] or the metric 25 m presentation span, then the
            // (convex) bilinear expansion below
            const uint64_t n = uint64_t(s.width) * s.height;
            op(launch_minmax_batched(graph_out, p.range, n, batch, st), "reduce_minmax");
            op(launch_normalize_batched(graph_out, p.range, n, batch, model_.metric_max_depth() > 0 ? 25.0f : 0.0f,
                                        st),
               "normalize");
            launches_ += 4;
        }
        float* result = graph_out;
        if (resize) {
            float* target = c.device_memory ? c.out : resized_buffer(uint64_t(batch) * w * h);
            op(launch_bilinear_align<float, float>(target, p.depth, s.width, s.height, w, h, batch, st),
               "resize depth");
            ++launches_;
            result = target;
        }
        const uint64_t out_bytes = uint64_t(batch) * w * h * 4;
        if (!c.device_memory) {
            cuda_check(cudaMemcpyAsync(pinned_out ? static_cast<void*>(c.out) : host_out_, result, out_bytes,
                                       cudaMemcpyDeviceToHost, st),
                       "D2H");
            download_bytes_ += out_bytes;
        }
        queue_error_read(st);
        finish_call(st);
        if (c.device_memory && c.stream) return;  // asynchronous: checked at the next call or dav2_synchronize
        cuda_check(cudaStreamSynchronize(st), "sync");
        if (!c.device_memory && !pinned_out) std::memcpy(c.out, host_out_, out_bytes);
        raise_device_error();
    }

    // ------------------------------------------------------------ weights
    const TensorView& t(const std::string& name) const { return model_.tensor(name); }

    const float* f32(const std::string& name) {
        const TensorView& v = t(name);
        float* d = wa_.take<float>(v.elements * 4);
        if (d) cuda_check(cudaMemcpy(d, v.data, v.elements * 4, cudaMemcpyHostToDevice), "upload");
        return d;
    }

    // Uploads a float tensor to the staging buffer (weights pass only).
    const float* stage(const std::string& name) {
        const TensorView& v = t(name);
        if (!wa_used_pass_) return nullptr;
        cuda_check(cudaMemcpy(wstage_, v.data, v.elements * 4, cudaMemcpyHostToDevice), "upload");
        return wstage_;
    }

    // kind: 0 plain [n][K]; 1 conv-transpose; 2 conv (ky,kx,c) with cip
    Linear make_linear(const std::string& wname, const std::string& bname, bool int8, int kind, uint32_t n,
                       uint32_t K, uint32_t kp, uint32_t co = 0, uint32_t k = 0, uint32_t ci = 0, uint32_t cip = 0) {
        Linear L;
        L.n = n;
        L.kp = kp;
        if (int8) {
            L.w = wa_.take<uint8_t>(uint64_t(n) * kp);
            L.s = wa_.take<float>(uint64_t(n) * 4);
        } else {
            L.w = wa_.take<uint16_t>(uint64_t(n) * kp * 2);
        }
        if (!bname.empty()) L.b = kind == 1 ? wa_.take<float>(uint64_t(n) * 4) : f32(bname);
        const float* src = stage(wname);
        if (src) {
            if (int8)
                op(launch_pack_weight_s8(static_cast<uint8_t*>(L.w), L.s, src, kind, n, K, kp, co, k, ci, nullptr),
                   "pack_weight_s8");
            else
                op(bf16_ ? launch_half_weight<__nv_bfloat16>(static_cast<__nv_bfloat16*>(L.w), src, kind, n, K, kp, co,
                                                             k, ci, cip, nullptr)
                         : launch_half_weight<__half>(static_cast<__half*>(L.w), src, kind, n, K, kp, co, k, ci, cip,
                                                      nullptr),
                   "half_weight");
            if (kind == 1 && L.b) {
                const float* b = f32(bname);
                op(launch_expand_bias(const_cast<float*>(L.b), b, co, k * k, nullptr), "expand_bias");
            }
            cuda_check(cudaDeviceSynchronize(), "weight prep");
        } else if (kind == 1 && L.b) {
            f32(bname);  // sizing of the per-channel bias
        }
        return L;
    }

    void build_weights() {
        const Arch& a = arch_;
        const bool q = int8_;
        cls_ = f32("pretrained.cls_token");
        pos_ = f32("pretrained.pos_embed");
        patch_ = make_linear("pretrained.patch_embed.proj.weight", "pretrained.patch_embed.proj.bias", q, 0, a.d, 588,
                             592);
        norm_w_ = f32("pretrained.norm.weight");
        norm_b_ = f32("pretrained.norm.bias");
        blocks_.resize(a.blocks);
        for (uint32_t i = 0; i < a.blocks; ++i) {
            const std::string p = "pretrained.blocks." + std::to_string(i);
            Block& b = blocks_[i];
            b.ln1_w = f32(p + ".norm1.weight");
            b.ln1_b = f32(p + ".norm1.bias");
            b.ln2_w = f32(p + ".norm2.weight");
            b.ln2_b = f32(p + ".norm2.bias");
            b.ls1 = f32(p + ".ls1.gamma");
            b.ls2 = f32(p + ".ls2.gamma");
            b.qkv = make_linear(p + ".attn.qkv.weight", p + ".attn.qkv.bias", q, 0, 3 * a.d, a.d, a.d);
            b.proj = make_linear(p + ".attn.proj.weight", p + ".attn.proj.bias", q, 0, a.d, a.d, a.d);
            b.fc1 = make_linear(p + ".mlp.fc1.weight", p + ".mlp.fc1.bias", q, 0, 4 * a.d, a.d, a.d);
            b.fc2 = make_linear(p + ".mlp.fc2.weight", p + ".mlp.fc2.bias", q, 0, a.d, 4 * a.d, 4 * a.d);
        }
        const std::string h = "depth_head.";
        for (int i = 0; i < 4; ++i) {
            const uint32_t oc = a.oc[i];
            cp_[i] = up(oc, 64);
            projects_[i] = make_linear(h + "projects." + std::to_string(i) + ".weight",
                                       h + "projects." + std::to_string(i) + ".bias", q, 0, oc, a.d, a.d);
        }
        for (int i = 0; i < 2; ++i) {
            const uint32_t oc = a.oc[i], k = i == 0 ? 4 : 2;
            const std::string r = h + "resize_layers." + std::to_string(i);
            resize_[i] = make_linear(r + ".weight", r + ".bias", q, 1, k * k * oc, oc, q ? up(oc, 16) : cp_[i], oc, k,
                                     oc);
        }
        {
            const uint32_t oc = a.oc[3];
            const std::string r = h + "resize_layers.3";
            resize_[3] = q ? make_linear(r + ".weight", r + ".bias", true, 2, oc, 9 * oc, 9 * oc, oc, 3, oc)
                           : make_linear(r + ".weight", r + ".bias", false, 2, oc, 9 * oc, 9 * cp_[3], oc, 3, oc, cp_[3]);
        }
        const uint32_t F = a.f;
        for (int i = 0; i < 4; ++i)
            layer_rn_[i] = make_linear(h + "scratch.layer" + std::to_string(i + 1) + "_rn.weight", "", false, 2, F,
                                       9 * a.oc[i], 9 * cp_[i], F, 3, a.oc[i], cp_[i]);
        for (int i = 0; i < 4; ++i) {
            const std::string r = h + "scratch.refinenet" + std::to_string(i + 1);
            for (int u = 0; u < 2; ++u)
                for (int c = 0; c < 2; ++c) {
                    const std::string n = r + ".resConfUnit" + std::to_string(u + 1) + ".conv" + std::to_string(c + 1);
                    refine_[i].rcu[u][c] = make_linear(n + ".weight", n + ".bias", false, 2, F, 9 * F, 9 * F, F, 3, F, F);
                }
            refine_[i].out = make_linear(r + ".out_conv.weight", r + ".out_conv.bias", false, 0, F, F, F);
        }
        half_f_ = F / 2;
        cp_half_ = up(F / 2, 64);
        out_conv1_ = make_linear(h + "scratch.output_conv1.weight", h + "scratch.output_conv1.bias", false, 2, F / 2,
                                 9 * F, 9 * F, F / 2, 3, F, F);
        out_conv2_ = make_linear(h + "scratch.output_conv2.0.weight", h + "scratch.output_conv2.0.bias", false, 2, 32,
                                 9 * (F / 2), 9 * cp_half_, 32, 3, F / 2, cp_half_);
        head_w_ = f32(h + "scratch.output_conv2.2.weight");
        head_b_ = t(h + "scratch.output_conv2.2.bias").data[0];
    }

    void load_weights() {
        // pass 1 sizes the arena, pass 2 fills it
        uint64_t largest = 0;
        for (auto n : model_.names()) largest = std::max<uint64_t>(largest, model_.tensor(n).elements * 4);
        wa_used_pass_ = false;
        build_weights();
        const uint64_t need = wa_.used() + 4096;
        wa_.rewind();
        wa_.reserve(need);
        cuda_check(cudaMalloc(&wstage_, largest), "cudaMalloc staging");
        wa_used_pass_ = true;
        build_weights();
        cudaFree(wstage_);
        wstage_ = nullptr;
        cuda_check(cudaDeviceSynchronize(), "weights");
    }

    // --------------------------------------------------------------- plans
    struct Plan {
        uint32_t B = 0, W = 0, H = 0, pw = 0, ph = 0, hw = 0, T = 0;
        std::unique_ptr<Arena> arena;
        float* image = nullptr;   // [B][3][H][W]
        float* depth = nullptr;   // [B][H][W]
        float** depth_slot = nullptr;  // destination of the graph's last convolution
        float* range = nullptr;        // [B][2] per-image depth min/max (normalizing entry points)
        float* pos = nullptr;     // [hw][D]
        void* patch_a = nullptr;  // int8 [B*hw][592] or f16
        float* patch_s = nullptr;
        float* x = nullptr;
        void* xn = nullptr;
        float* xn_s = nullptr;
        __half* qkv = nullptr;
        void* att = nullptr;      // attention output: f32 (int8 path, the quantizer's input) or f16
        void* att_q = nullptr;
        float* att_s = nullptr;
        void* hid = nullptr;      // GELU(fc1) output: f32 (int8 path) or f16
        void* hid_q = nullptr;
        float* hid_s = nullptr;
        void* taps[4] = {};
        float* taps_s[4] = {};
        __half* proj[4] = {};     // f16 channels-last projections (those the f16 convolutions read)
        float* projf[4] = {};     // int8 path: f32 projections that are quantized next (0, 1, 3)
        void* ct_q[2] = {};
        float* ct_s[2] = {};
        __half* layer[4] = {};
        void* r3_col = nullptr;
        float* r3_s = nullptr;
        uint32_t lh[4] = {}, lw[4] = {};
        __half *rn[4] = {}, *rn_relu[4] = {};
        __half *t = nullptr, *y = nullptr, *pth = nullptr, *pth_relu = nullptr, *upb = nullptr;
        __half *path[2] = {};
        __half *oc1 = nullptr, *full = nullptr;
        cudaGraphExec_t graph = nullptr;
        uint64_t kernels = 0;  // kernel nodes in the captured graph
    };

    void alloc(Plan& p, Arena& A) {
        const Arch& a = arch_;
        const uint64_t B = p.B, R = B * p.T, PH = B * p.hw, D = a.d, F = a.f;
        const bool q = int8_;
        p.image = A.take<float>(B * 3 * p.H * p.W * 4);
        p.depth = A.take<float>(B * p.H * p.W * 4);
        p.depth_slot = A.take<float*>(sizeof(float*));
        p.range = A.take<float>(B * 2 * 4);
        p.pos = A.take<float>(uint64_t(p.hw) * D * 4);
        p.patch_a = A.take<uint8_t>(PH * 592 * (q ? 1 : 2));
        if (q) p.patch_s = A.take<float>(PH * 4);
        p.x = A.take<float>(R * D * 4);
        p.xn = A.take<uint8_t>(R * D * (q ? 1 : 2));
        if (q) p.xn_s = A.take<float>(R * 4);
        p.qkv = A.take<__half>(R * 3 * D * 2);
        p.att = A.take<uint8_t>(R * D * (q ? 4 : 2));
        if (q) {
            p.att_q = A.take<uint8_t>(R * D);
            p.att_s = A.take<float>(R * 4);
        }
        p.hid = A.take<uint8_t>(R * 4 * D * (q ? 4 : 2));
        if (q) {
            p.hid_q = A.take<uint8_t>(R * 4 * D);
            p.hid_s = A.take<float>(R * 4);
        }
        for (int i = 0; i < 4; ++i) {
            p.taps[i] = A.take<uint8_t>(PH * D * (q ? 1 : 2));
            if (q) p.taps_s[i] = A.take<float>(PH * 4);
            if (q && i != 2)
                p.projf[i] = A.take<float>(PH * a.oc[i] * 4);
            else
                p.proj[i] = A.take<__half>(PH * cp_[i] * 2);
        }
        for (int i = 0; i < 2; ++i) {
            const uint32_t k = i == 0 ? 4 : 2;
            if (q) {
                p.ct_q[i] = A.take<uint8_t>(PH * up(a.oc[i], 16));
                p.ct_s[i] = A.take<float>(PH * 4);
            }
            p.lh[i] = p.ph * k;
            p.lw[i] = p.pw * k;
            p.layer[i] = A.take<__half>(B * p.lh[i] * p.lw[i] * cp_[i] * 2);
        }
        p.lh[2] = p.ph;
        p.lw[2] = p.pw;
        p.layer[2] = p.proj[2];
        p.lh[3] = (p.ph - 1) / 2 + 1;
        p.lw[3] = (p.pw - 1) / 2 + 1;
        p.layer[3] = A.take<__half>(B * p.lh[3] * p.lw[3] * cp_[3] * 2);
        const uint64_t r3rows = B * p.lh[3] * p.lw[3];
        if (q) {
            p.r3_col = A.take<uint8_t>(r3rows * 9 * a.oc[3]);
            p.r3_s = A.take<float>(r3rows * 4);
        } else {
            p.r3_col = A.take<__half>(r3rows * 9 * cp_[3] * 2);
        }
        for (int i = 0; i < 4; ++i) {
            const uint64_t n = B * p.lh[i] * p.lw[i] * F * 2;
            p.rn[i] = A.take<__half>(n);
            p.rn_relu[i] = A.take<__half>(n);
        }
        const uint64_t big = B * p.lh[0] * p.lw[0] * F * 2;  // largest RCU scale
        p.t = A.take<__half>(big);
        p.y = A.take<__half>(big);
        p.pth = A.take<__half>(big);
        p.pth_relu = A.take<__half>(big);
        p.upb = A.take<__half>(4 * big);
        p.path[0] = A.take<__half>(4 * big);
        p.path[1] = A.take<__half>(4 * big);
        p.oc1 = A.take<__half>(B * 4 * p.lh[0] * p.lw[0] * cp_half_ * 2);
        p.full = A.take<__half>(B * p.H * p.W * cp_half_ * 2);
    }

    Plan& plan(int batch, int w, int h) {
        if (w <= 0 || h <= 0 || w % 14 || h % 14)
            throw std::invalid_argument("network dimensions must be positive multiples of 14");
        const auto key = std::make_tuple(batch, w, h);
        auto it = plans_.find(key);
        if (it != plans_.end()) return it->second;
        Plan& p = plans_[key];
        p.B = batch;
        p.W = w;
        p.H = h;
        p.pw = w / 14;
        p.ph = h / 14;
        p.hw = p.pw * p.ph;
        p.T = p.hw + 1;
        Arena sizing;
        alloc(p, sizing);
        p.arena = std::make_unique<Arena>();
        p.arena->reserve(sizing.used() + 4096);
        alloc(p, *p.arena);
        op(launch_position_bicubic(p.pos, pos_, arch_.d, p.pw, p.ph, stream_), "position_bicubic");
        // warm-up run (sets kernel attributes), then capture
        cuda_check(cudaStreamWaitEvent(stream_, done_, 0), "wait");
        op(launch_store_pointer(reinterpret_cast<void**>(p.depth_slot), p.depth, stream_), "store_pointer");
        enqueue(p, stream_);
        queue_error_read(stream_);
        cuda_check(cudaStreamSynchronize(stream_), "warm-up");
        raise_device_error();
        cudaGraph_t g = nullptr;
        cuda_check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "capture");
        try {
            enqueue(p, stream_);
        } catch (...) {
            cudaStreamEndCapture(stream_, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        cuda_check(cudaStreamEndCapture(stream_, &g), "end capture");
        size_t nodes = 0;
        cuda_check(cudaGraphGetNodes(g, nullptr, &nodes), "graph nodes");
        p.kernels = nodes;
        cuda_check(cudaGraphInstantiate(&p.graph, g, 0), "instantiate");
        cudaGraphDestroy(g);
        return p;
    }

    // Launch bookkeeping: in profiling mode every launch is followed by an
    // event on the launching stream (the analogue of DAV2_VULKAN_PROFILE=1,
    // src/vulkan.cpp:628-644), giving per-operation device durations.
    void step(cudaStream_t st, int rc, const char* name) {
        op(rc, name);
        if (profiling_) {
            cudaEvent_t e;
            cuda_check(cudaEventCreate(&e), "event");
            cuda_check(cudaEventRecord(e, st), "event record");
            marks_.push_back({name, e});
        }
    }

public:
    std::string profile(int batch, int w, int h) {
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        Plan& p = plan(batch, w, h);
        cudaEvent_t start;
        cuda_check(cudaEventCreate(&start), "event");
        marks_.clear();
        cuda_check(cudaStreamWaitEvent(stream_, done_, 0), "wait");
        op(launch_store_pointer(reinterpret_cast<void**>(p.depth_slot), p.depth, stream_), "store_pointer");
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        cuda_check(cudaEventRecord(start, stream_), "event record");
        profiling_ = true;
        try {
            enqueue(p, stream_);
        } catch (...) {
            profiling_ = false;
            throw;
        }
        profiling_ = false;
        queue_error_read(stream_);
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        raise_device_error();
        std::string out = "{\"batch\": " + std::to_string(batch) + ", \"width\": " + std::to_string(w) +
                          ", \"height\": " + std::to_string(h) + ", \"ops\": [";
        cudaEvent_t prev = start;
        float total = 0.f;
        for (size_t i = 0; i < marks_.size(); ++i) {
            float ms = 0.f;
            cuda_check(cudaEventElapsedTime(&ms, prev, marks_[i].second), "elapsed");
            total += ms;
            char buf[160];
            snprintf(buf, sizeof buf, "%s{\"name\": \"%s\", \"ms\": %.6f}", i ? ", " : "", marks_[i].first, ms);
            out += buf;
            if (prev != start) cudaEventDestroy(prev);
            prev = marks_[i].second;
        }
        if (prev != start) cudaEventDestroy(prev);
        cudaEventDestroy(start);
        marks_.clear();
        char tail[64];
        snprintf(tail, sizeof tail, "], \"total_ms\": %.6f}", total);
        return out + tail;
    }

private:
    void launch_plan(Plan& p, cudaStream_t st) {
        cuda_check(cudaGraphLaunch(p.graph, st), "graph launch");
        launches_ += p.kernels;
    }

    // ---------------------------------------------------------- the graph
    // 16-bit launches in the context's 16-bit type (f16, or bf16 when bf16_).
    int half_ln() const { return bf16_ ? kLnOutBF16 : kLnOutF16; }
    int bilinear16(void* out, const void* in, uint32_t B, uint32_t ih, uint32_t iw, uint32_t oh, uint32_t ow,
                   uint32_t c, cudaStream_t st) const {
        if (bf16_)
            return launch_bilinear_nhwc<__nv_bfloat16>(static_cast<__nv_bfloat16*>(out),
                                                       static_cast<const __nv_bfloat16*>(in), B, ih, iw, oh, ow, c, st);
        return launch_bilinear_nhwc<__half>(static_cast<__half*>(out), static_cast<const __half*>(in), B, ih, iw, oh, ow,
                                            c, st);
    }
    int im2col_nhwc16(void* out, const void* in, uint32_t B, uint32_t h, uint32_t w, uint32_t c, uint32_t k,
                      uint32_t s, uint32_t pad, uint32_t oh, uint32_t ow, uint32_t kp, cudaStream_t st) const {
        if (bf16_)
            return launch_im2col_nhwc<__nv_bfloat16>(static_cast<__nv_bfloat16*>(out),
                                                     static_cast<const __nv_bfloat16*>(in), B, h, w, c, k, s, pad, oh,
                                                     ow, kp, st);
        return launch_im2col_nhwc<__half>(static_cast<__half*>(out), static_cast<const __half*>(in), B, h, w, c, k, s,
                                          pad, oh, ow, kp, st);
    }

    GemmArgs gemm(const Linear& L, const void* a, uint64_t lda, uint32_t m, bool int8_operands) const {
        GemmArgs g;
        g.elem = int8_operands ? kElemS8 : bf16_ ? kElemBF16 : kElemF16;
        g.out_half_bf16 = bf16_;  // 16-bit outputs in the 16-bit operand type
        g.a = a;
        g.lda = lda;
        g.b = L.w;
        g.ldb = L.kp;
        g.m = m;
        g.n = L.n;
        g.k = L.kp;
        g.bias = L.b;
        g.flags = L.b ? kEpiBias : 0u;
        if (int8_operands) {
            g.flags |= kEpiDequant;
            g.s_w = L.s;
        }
        return g;
    }

    GemmArgs conv3x3(const Linear& L, const __half* in, uint32_t B, uint32_t h, uint32_t w, uint32_t c) const {
        GemmArgs g = gemm(L, in, 0, B * h * w, false);
        g.a_mode = kAModeConv3x3;
        g.conv_batch = B;
        g.conv_h = h;
        g.conv_w = w;
        g.conv_c = c;
        return g;
    }

    // The whole graph: embedding, blocks (with the tap LayerNorms), head.
    // The stage functions below are also what the stage probes run, so a
    // probe exercises exactly the launches of the captured graph.
    void enqueue(Plan& p, cudaStream_t st) {
        enqueue_embed(p, st);
        int tap = 0;
        for (uint32_t i = 0; i < arch_.blocks; ++i) {
            enqueue_block(p, i, st);
            if (tap < 4 && i == arch_.taps[tap]) enqueue_tap(p, tap++, st);
        }
        enqueue_head(p, st);
    }

    // ---- patch embedding + cls + positions (src/operators.cpp:1211-1406)
    void enqueue_embed(Plan& p, cudaStream_t st) {
        const Arch& a = arch_;
        const bool q = int8_;
        const uint32_t B = p.B, D = a.d, PH = B * p.hw;
        step(st, launch_fill_tokens(p.x, cls_, pos_, p.pos, D, p.T, B, st), "fill_tokens");
        if (q)
            step(st, launch_im2col_quantize(static_cast<uint32_t*>(p.patch_a), p.patch_s, p.image, B, p.W, p.H, 3, p.pw,
                                      p.ph, 14, 14, 0, 592 / 4, st),
               "patch im2col_quantize");
        else
            step(st,
                 bf16_ ? launch_patch_im2col<__nv_bfloat16>(static_cast<__nv_bfloat16*>(p.patch_a), p.image, B, p.H,
                                                            p.W, 592, st)
                       : launch_patch_im2col<__half>(static_cast<__half*>(p.patch_a), p.image, B, p.H, p.W, 592, st),
                 "patch im2col");
        GemmArgs g = gemm(patch_, p.patch_a, 592, PH, q);
        g.s_in = p.patch_s;
        g.flags |= kEpiResidual1;
        g.res1 = p.x;
        g.out = p.x;
        g.out_kind = kOutF32Rows;
        g.ldo = D;
        g.rows_per_img = p.hw;
        g.out_rows_per_img = p.T;
        g.row_offset = 1;
        step(st, launch_gemm(g, st), "patch gemm");
    }

    // block i's first LayerNorm: residual p.x -> p.xn (int8 codes + p.xn_s, or f16)
    void enqueue_ln1(Plan& p, uint32_t i, cudaStream_t st) {
        const Block& b = blocks_[i];
        step(st, launch_layer_norm(p.xn, p.xn_s, p.x, b.ln1_w, b.ln1_b, p.B * p.T, arch_.d, 1e-6f,
                                   int8_ ? kLnOutS8 : half_ln(), 1, 1, 0, st),
             "ln1");
    }

    // ---- transformer block i (src/encoder.cpp:426-591), p.x updated in place
    void enqueue_block(Plan& p, uint32_t i, cudaStream_t st) {
        const Arch& a = arch_;
        const bool q = int8_;
        const uint32_t B = p.B, D = a.d;
        const uint32_t R = B * p.T;
        const Block& b = blocks_[i];
        enqueue_ln1(p, i, st);
        {
            GemmArgs g = gemm(b.qkv, p.xn, D, R, q);
            g.s_in = p.xn_s;
            g.out = p.qkv;
            g.out_kind = kOutHalfRows;
            g.ldo = 3 * D;
            step(st, launch_gemm(g, st), "qkv");
        }
        // int8 path: attention output and GELU hidden stay f32 up to their
        // quantizers, as the reference's int8 mode keeps them
        // (src/operators.cpp:1098-1209 writes f32; src/encoder.cpp:526-528)
        step(st, launch_attention_tc(p.att, q, p.qkv, bf16_, B, p.T, a.heads, 3 * D, D, st), "attention");
        const void* att_in = p.att;
        if (q) {
            step(st, launch_quantize_rows<float>(static_cast<uint32_t*>(p.att_q), p.att_s,
                                                 static_cast<const float*>(p.att), R, D, 0, R, 0, D, D / 4, st),
               "quantize attention");
            att_in = p.att_q;
        }
        {
            GemmArgs g = gemm(b.proj, att_in, D, R, q);
            g.s_in = p.att_s;
            g.flags |= kEpiLayerScale;
            g.gamma = b.ls1;
            g.res1 = p.x;
            g.out = p.x;
            g.out_kind = kOutF32Rows;
            g.ldo = D;
            step(st, launch_gemm(g, st), "proj");
        }
        step(st, launch_layer_norm(p.xn, p.xn_s, p.x, b.ln2_w, b.ln2_b, R, D, 1e-6f, q ? kLnOutS8 : half_ln(), 1, 1, 0,
                             st),
           "ln2");
        {
            GemmArgs g = gemm(b.fc1, p.xn, D, R, q);
            g.s_in = p.xn_s;
            g.flags |= kEpiGelu;
            g.out = p.hid;
            g.out_kind = q ? kOutF32Rows : kOutHalfRows;
            g.ldo = 4 * D;
            step(st, launch_gemm(g, st), "fc1");
        }
        const void* hid_in = p.hid;
        if (q) {
            step(st, launch_quantize_rows<float>(static_cast<uint32_t*>(p.hid_q), p.hid_s,
                                                 static_cast<const float*>(p.hid), R, 4 * D, 0, R, 0, 4 * D, D, st),
               "quantize hidden");
            hid_in = p.hid_q;
        }
        {
            GemmArgs g = gemm(b.fc2, hid_in, 4 * D, R, q);
            g.s_in = p.hid_s;
            g.flags |= kEpiLayerScale;
            g.gamma = b.ls2;
            g.res1 = p.x;
            g.out = p.x;
            g.out_kind = kOutF32Rows;
            g.ldo = D;
            step(st, launch_gemm(g, st), "fc2");
        }
    }

    // pretrained.norm of tap k on the patch rows only (cls dropped)
    void enqueue_tap(Plan& p, int k, cudaStream_t st) {
        step(st, launch_layer_norm(p.taps[k], p.taps_s[k], p.x, norm_w_, norm_b_, p.B * p.hw, arch_.d, 1e-6f,
                                   int8_ ? kLnOutS8 : half_ln(), p.hw, p.T, 1, st),
             "tap norm");
    }

    // ---- DPT head (src/dpt.cpp:628-863): taps -> depth (through p.depth_slot)
    void enqueue_head(Plan& p, cudaStream_t st) {
        const Arch& a = arch_;
        const bool q = int8_;
        const uint32_t B = p.B, D = a.d, F = a.f;
        const uint32_t PH = B * p.hw;
        // ---- DPT projections and resize layers (src/dpt.cpp:641-731)
        // int8 path: the projections that are quantized next (0, 1, 3) are
        // written f32, the reference's FeatureMap precision (src/dpt.cpp:494-499)
        for (int i = 0; i < 4; ++i) {
            GemmArgs g = gemm(projects_[i], p.taps[i], D, PH, q);
            g.s_in = p.taps_s[i];
            if (p.projf[i]) {
                g.out = p.projf[i];
                g.out_kind = kOutF32Rows;
                g.ldo = a.oc[i];
            } else {
                g.out = p.proj[i];
                g.out_kind = kOutHalfRows;
                g.ldo = cp_[i];
            }
            step(st, launch_gemm(g, st), "project");
        }
        for (int i = 0; i < 2; ++i) {
            const uint32_t k = i == 0 ? 4 : 2, oc = a.oc[i];
            GemmArgs g;
            if (q) {
                const uint32_t kp = up(oc, 16);
                // per-pixel channel quantization with the im2col rule x * (1/scale),
                // as conv_transpose_nonoverlap_int8 does (src/operators.cpp:1952-1955)
                step(st, launch_im2col_quantize_nhwc<float>(static_cast<uint8_t*>(p.ct_q[i]), p.ct_s[i], p.projf[i], B,
                                                            p.ph, p.pw, oc, oc, 1, 1, 0, p.ph, p.pw, kp, st),
                   "quantize convT input");
                g = gemm(resize_[i], p.ct_q[i], kp, PH, true);
                g.s_in = p.ct_s[i];
            } else {
                g = gemm(resize_[i], p.proj[i], cp_[i], PH, false);
            }
            g.out = p.layer[i];
            g.out_kind = kOutConvTHalf;
            g.ldo = cp_[i];
            g.convt_k = k;
            g.convt_cout = oc;
            g.convt_w = p.pw;
            g.convt_h = p.ph;
            step(st, launch_gemm(g, st), "conv transpose");
        }
        {
            const uint32_t oc = a.oc[3], rows = B * p.lh[3] * p.lw[3];
            GemmArgs g;
            if (q) {
                step(st, launch_im2col_quantize_nhwc<float>(static_cast<uint8_t*>(p.r3_col), p.r3_s, p.projf[3], B,
                                                            p.ph, p.pw, oc, oc, 3, 2, 1, p.lh[3], p.lw[3], 9 * oc, st),
                   "resize3 im2col_quantize");
                g = gemm(resize_[3], p.r3_col, 9 * oc, rows, true);
                g.s_in = p.r3_s;
            } else {
                step(st, im2col_nhwc16(p.r3_col, p.proj[3], B, p.ph, p.pw, cp_[3], 3, 2, 1,
                                              p.lh[3], p.lw[3], 9 * cp_[3], st),
                   "resize3 im2col");
                g = gemm(resize_[3], p.r3_col, 9 * cp_[3], rows, false);
            }
            g.out = p.layer[3];
            g.out_kind = kOutHalfRows;
            g.ldo = cp_[3];
            step(st, launch_gemm(g, st), "resize3");
        }
        // ---- scratch.layerN_rn (3x3, no bias) with a ReLU copy for the RCUs
        for (int i = 0; i < 4; ++i) {
            GemmArgs g = conv3x3(layer_rn_[i], p.layer[i], B, p.lh[i], p.lw[i], cp_[i]);
            g.out = p.rn[i];
            g.out2 = p.rn_relu[i];
            g.flags |= kEpiReluCopy;
            g.out_kind = kOutHalfRows;
            g.ldo = F;
            step(st, launch_gemm(g, st), "layer_rn");
        }
        // ---- refinenets (src/dpt.cpp:537-615, 759-790)
        const __half* path = nullptr;
        int pi = 0;
        for (int r = 3; r >= 0; --r) {
            const RefineNet& rf = refine_[r];
            const uint32_t h = p.lh[r], w = p.lw[r];
            const __half* x = p.rn[r];
            const __half* xr = p.rn_relu[r];
            if (path) {
                // RCU1 on the skip, fused with the fusion add: p' = path + (conv2(...) + skip)
                GemmArgs g1 = conv3x3(rf.rcu[0][0], xr, B, h, w, F);
                g1.flags |= kEpiRelu;
                g1.out = p.t;
                g1.out_kind = kOutHalfRows;
                g1.ldo = F;
                step(st, launch_gemm(g1, st), "rcu1.conv1");
                GemmArgs g2 = conv3x3(rf.rcu[0][1], p.t, B, h, w, F);
                g2.flags |= kEpiResidual1 | kEpiResidual2 | kEpiReluCopy;
                g2.res1 = x;
                g2.res2 = path;
                g2.out = p.pth;
                g2.out2 = p.pth_relu;
                g2.out_kind = kOutHalfRows;
                g2.ldo = F;
                step(st, launch_gemm(g2, st), "rcu1.conv2");
                x = p.pth;
                xr = p.pth_relu;
            }
            GemmArgs g3 = conv3x3(rf.rcu[1][0], xr, B, h, w, F);
            g3.flags |= kEpiRelu;
            g3.out = p.t;
            g3.out_kind = kOutHalfRows;
            g3.ldo = F;
            step(st, launch_gemm(g3, st), "rcu2.conv1");
            GemmArgs g4 = conv3x3(rf.rcu[1][1], p.t, B, h, w, F);
            g4.flags |= kEpiResidual1;
            g4.res1 = x;
            g4.out = p.y;
            g4.out_kind = kOutHalfRows;
            g4.ldo = F;
            step(st, launch_gemm(g4, st), "rcu2.conv2");
            const uint32_t oh = r > 0 ? p.lh[r - 1] : 2 * p.lh[0];
            const uint32_t ow = r > 0 ? p.lw[r - 1] : 2 * p.lw[0];
            step(st, bilinear16(p.upb, p.y, B, h, w, oh, ow, F, st), "fusion resize");
            GemmArgs g5 = gemm(rf.out, p.upb, F, B * oh * ow, false);
            g5.out = p.path[pi];
            g5.out_kind = kOutHalfRows;
            g5.ldo = F;
            step(st, launch_gemm(g5, st), "out_conv");
            path = p.path[pi];
            pi ^= 1;
        }
        // ---- output head (src/dpt.cpp:813-854)
        const uint32_t h1 = 2 * p.lh[0], w1 = 2 * p.lw[0];
        if (conv3x3_halo_supported(F, out_conv1_.n, cp_half_)) {
            step(st, launch_conv3x3_halo(p.oc1, path, out_conv1_.w, out_conv1_.b, bf16_, B, h1, w1, F, st),
                 "output_conv1");
        } else {
            GemmArgs g = conv3x3(out_conv1_, path, B, h1, w1, F);
            g.out = p.oc1;
            g.out_kind = kOutHalfRows;
            g.ldo = cp_half_;
            step(st, launch_gemm(g, st), "output_conv1");
        }
        step(st, bilinear16(p.full, p.oc1, B, h1, w1, p.H, p.W, cp_half_, st), "head resize");
        if (conv_head_halo_supported(cp_half_, out_conv2_.n)) {
            const float max_depth = model_.metric_max_depth();
            step(st,
                 launch_conv_head_halo(p.depth, p.depth_slot, p.full, out_conv2_.w, out_conv2_.b, head_w_, head_b_,
                                       max_depth, max_depth > 0, bf16_, B, p.H, p.W, cp_half_, st),
                 "output_conv2");
        } else {
            GemmArgs g = conv3x3(out_conv2_, p.full, B, p.H, p.W, cp_half_);
            g.flags |= kEpiHeadDot | (model_.metric_max_depth() > 0 ? kEpiMetricHead : 0u);
            g.head_w = head_w_;
            g.head_b = head_b_;
            g.head_max_depth = model_.metric_max_depth();
            g.out = p.depth;
            g.out_slot = p.depth_slot;
            g.out_kind = kOutHeadF32;
            step(st, launch_gemm(g, st), "output_conv2");
        }
    }

    void run_host_tensor(const float* chw, int batch, int w, int h, float* depth, int ow, int oh) {
        if (!chw || !depth || batch <= 0) throw std::invalid_argument("null inference argument");
        std::lock_guard<std::mutex> lock(mutex_);
        cuda_check(cudaSetDevice(device_), "cudaSetDevice");
        poll_device_error();
        Plan& p = plan(batch, w, h);
        order_after_previous_call(stream_);
        const uint64_t in_bytes = uint64_t(batch) * 3 * w * h * 4;
        const uint64_t out_bytes = uint64_t(batch) * ow * oh * 4;
        ensure_host(in_bytes, out_bytes);
        std::memcpy(host_in_, chw, in_bytes);
        cuda_check(cudaMemcpyAsync(p.image, host_in_, in_bytes, cudaMemcpyHostToDevice, stream_), "H2D");
        upload_bytes_ += in_bytes;
        op(launch_store_pointer(reinterpret_cast<void**>(p.depth_slot), p.depth, stream_), "store_pointer");
        ++launches_;
        launch_plan(p, stream_);
        float* result = p.depth;
        if (ow != w || oh != h) {
            float* resized = resized_buffer(uint64_t(batch) * ow * oh);
            op(launch_bilinear_align<float, float>(resized, p.depth, w, h, ow, oh, batch, stream_), "resize depth");
            ++launches_;
            result = resized;
        }
        cuda_check(cudaMemcpyAsync(host_out_, result, out_bytes, cudaMemcpyDeviceToHost, stream_), "D2H");
        queue_error_read(stream_);
        finish_call(stream_);
        cuda_check(cudaStreamSynchronize(stream_), "sync");
        std::memcpy(depth, host_out_, out_bytes);
        download_bytes_ += out_bytes;
        raise_device_error();
    }

    void ensure_host(uint64_t in, uint64_t out) {
        if (in > host_in_cap_) {
            if (host_in_) cudaFreeHost(host_in_);
            cuda_check(cudaMallocHost(&host_in_, in), "cudaMallocHost");
            host_in_cap_ = in;
        }
        if (out > host_out_cap_) {
            if (host_out_) cudaFreeHost(host_out_);
            cuda_check(cudaMallocHost(&host_out_, out), "cudaMallocHost");
            host_out_cap_ = out;
        }
    }

    void ensure_staging(uint64_t bytes) {
        if (bytes > staging_cap_) {
            if (staging_) cudaFree(staging_);
            cuda_check(cudaMalloc(&staging_, bytes), "cudaMalloc");
            staging_cap_ = bytes;
        }
    }

    float* resized_buffer(uint64_t n) {
        if (n * 4 > resized_cap_) {
            resized_.reset();
            resized_ = std::make_unique<Arena>();
            resized_->reserve(n * 4 + 256);
            resized_cap_ = n * 4;
            resized_ptr_ = resized_->take<float>(n * 4);
        }
        return resized_ptr_;
    }

    // Device-side failures (a bounded pipeline wait that gave up) set the
    // device error word, which stays set until the host clears it. Every
    // call queues an asynchronous read of the word into pinned host memory
    // behind its own work: a synchronous call checks it after its stream
    // synchronisation; after an asynchronous call (a caller stream) it is
    // checked by the next call of this context once that read has completed,
    // or by synchronize(), which waits for it.
    void queue_error_read(cudaStream_t st) {
        int* word = device_error_word();
        if (!word) throw std::runtime_error("the device error word is unavailable");
        cuda_check(cudaMemcpyAsync(err_host_, word, sizeof(int), cudaMemcpyDeviceToHost, st), "error word read");
        cuda_check(cudaEventRecord(err_event_, st), "event record");
        err_pending_ = true;
    }

    // Throws (DAV2_STATUS_INFERENCE_FAILED) when the last completed read saw
    // the word set, after clearing it on the device.
    void raise_device_error() {
        if (!err_pending_) return;
        err_pending_ = false;
        if (*err_host_ == 0) return;
        *err_host_ = 0;
        if (int* word = device_error_word()) {
            cuda_check(cudaMemsetAsync(word, 0, sizeof(int), stream_), "error word clear");
            cuda_check(cudaStreamSynchronize(stream_), "sync");
        }
        throw_inference_failed("a kernel pipeline wait timed out on the device");
    }

    void poll_device_error() {
        if (err_pending_ && cudaEventQuery(err_event_) == cudaSuccess) raise_device_error();
    }

    // A context's plans and buffers are shared by all its calls: a call on
    // another stream than the previous call's starts after that call's work.
    void order_after_previous_call(cudaStream_t st) {
        if (last_stream_ != nullptr && last_stream_ != st) cuda_check(cudaStreamWaitEvent(st, done_, 0), "wait");
    }

    void finish_call(cudaStream_t st) {
        cuda_check(cudaEventRecord(done_, st), "event record");
        last_stream_ = st;
    }

    ModelFile model_;
    dav2_encoder encoder_;
    int device_;
    Arch arch_;
    bool int8_ = false;
    bool bf16_ = false;  // 16-bit operands and activations bf16 instead of f16 (not with int8_)
    cudaStream_t stream_ = nullptr;
    cudaEvent_t done_ = nullptr;       // end of the last call's work (on last_stream_)
    cudaStream_t last_stream_ = nullptr;
    cudaEvent_t err_event_ = nullptr;  // completion of the last queued error-word read
    int* err_host_ = nullptr;          // pinned copy of the device error word
    bool err_pending_ = false;
    std::mutex mutex_;

    Arena wa_;
    bool wa_used_pass_ = false;
    float* wstage_ = nullptr;
    const float *cls_ = nullptr, *pos_ = nullptr, *norm_w_ = nullptr, *norm_b_ = nullptr, *head_w_ = nullptr;
    float head_b_ = 0.f;
    Linear patch_;
    std::vector<Block> blocks_;
    Linear projects_[4], resize_[4], layer_rn_[4];
    RefineNet refine_[4];
    Linear out_conv1_, out_conv2_;
    uint32_t cp_[4] = {}, half_f_ = 0, cp_half_ = 0;

    std::map<std::tuple<int, int, int>, Plan> plans_;
    uint8_t* staging_ = nullptr;
    uint64_t staging_cap_ = 0;
    void* host_in_ = nullptr;
    void* host_out_ = nullptr;
    uint64_t host_in_cap_ = 0, host_out_cap_ = 0;
    std::unique_ptr<Arena> resized_;
    uint64_t resized_cap_ = 0;
    float* resized_ptr_ = nullptr;
    uint64_t upload_bytes_ = 0, download_bytes_ = 0;
    uint64_t launches_ = 0;
    bool profiling_ = false;
    std::vector<std::pair<const char*, cudaEvent_t>> marks_;
};

}  // namespace

std::unique_ptr<Executor> create_executor(const std::string& model_path, dav2_encoder encoder, int device_index,
                                          std::uint32_t flags, const std::string& cache_path) {
    (void)cache_path;
    if ((flags & DAV2_CREATE_FORCE_METAL) && (flags & DAV2_CREATE_FORCE_VULKAN))
        throw std::invalid_argument("Metal and Vulkan cannot both be forced");
    // The reference keeps fp32 weights and scores for these requests
    // (src/vulkan_executor.cpp:505-518, src/encoder.cpp:389-396). This
    // executor has no fp32-exact tensor path, so it refuses them instead of
    // running a lower precision under an fp32 request.
    if (flags & (DAV2_CREATE_FORCE_FP32 | DAV2_CREATE_FORCE_FP32_WEIGHTS | DAV2_CREATE_FORCE_FP32_ATTENTION))
        throw_unsupported("fp32 execution is not available in the CUDA executor (use the default / FORCE_FP16 "
                          "or FORCE_INT8 precision)");
    return std::make_unique<CudaExecutor>(model_path, encoder, device_index, flags);
}

GpuCapabilities probe_gpu_capabilities(int device_index) {
    GpuCapabilities c;
    int count = 0;
    if (cudaGetDeviceCount(&count) == cudaSuccess && device_index >= 0 && device_index < count) {
        c.flags = DAV2_GPU_CAP_NO_HOST_PIXEL_STAGING | DAV2_GPU_CAP_NO_HOST_DEPTH_STAGING;
        c.maximum_in_flight_jobs = 1;
    }
    return c;
}

}  // namespace dav2
