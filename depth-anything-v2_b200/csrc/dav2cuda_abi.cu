// C ABI of the operator layer (include/dav2cuda.h). Each entry validates its
// sizes the way src/operators.cpp does before dispatching (there:
// require_bytes / std::invalid_argument; here: DAV2CUDA_INVALID_ARGUMENT),
// then launches the sm_100a kernels asynchronously on the caller's stream.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <string>

#include "kernels.cuh"

namespace dav2cuda {

namespace {
thread_local std::string t_last_error;
std::atomic<uint64_t> g_launches{0};
__device__ int g_device_error = 0;
std::atomic<int*> g_error_word[64];
}  // namespace

// Device address of the error word on the current device, resolved once per
// device with cudaGetSymbolAddress (a cudaDeviceReset invalidates it, as it
// invalidates every device allocation this library and its contexts hold).
int* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    int* cached = g_error_word[dev].load(std::memory_order_acquire);
    if (!cached) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        cached = static_cast<int*>(p);
        g_error_word[dev].store(cached, std::memory_order_release);
    }
    return cached;
}

int sm_count(int dev) {
    static std::atomic<int> cache[64];
    if (dev < 0 || dev >= 64) return 0;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n == 0 && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
        cache[dev].store(n, std::memory_order_relaxed);
    return n > 0 ? n : 0;
}

int set_error(int status, const char* message) {
    t_last_error = message ? message : "";
    return status;
}

int check_launch(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
        return set_error(DAV2CUDA_LAUNCH_FAILED, msg);
    }
    return DAV2CUDA_OK;
}

namespace {

__global__ void pad_byte_rows_kernel(uint8_t* __restrict__ out, const uint8_t* __restrict__ in, uint64_t rows,
                                     uint32_t in_bytes, uint32_t out_bytes) {
    const uint64_t n = rows * out_bytes;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t r = i / out_bytes;
        const uint32_t c = (uint32_t)(i % out_bytes);
        out[i] = c < in_bytes ? in[r * in_bytes + c] : 0;
    }
}

__global__ void f16_to_f32_kernel(float* __restrict__ out, const __half* __restrict__ in, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __half2float(in[i]);
}

// One 32-thread block: thread 0 waits on an mbarrier phase that completes
// only when `arrive` is set, through the pipelines' bounded wait.
__global__ void wait_probe_kernel(unsigned long long limit_ns, uint32_t arrive, int* err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (arrive) mbar_arrive(&bar);
        mbar_wait_for(&bar, 0, &abort_flag, err, limit_ns);
    }
}

int pad_byte_rows(uint8_t* out, const void* in, uint64_t rows, uint32_t in_bytes, uint32_t out_bytes,
                  cudaStream_t st) {
    const uint64_t n = rows * out_bytes;
    const unsigned grid = (unsigned)std::min<uint64_t>((n + 255) / 256 + 1, 148 * 16);
    pad_byte_rows_kernel<<<grid, 256, 0, st>>>(out, static_cast<const uint8_t*>(in), rows, in_bytes, out_bytes);
    return check_launch("pad_byte_rows");
}

constexpr uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }
constexpr uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

// Bump allocator over a caller workspace.
struct Carve {
    uint8_t* base;
    uint64_t size, used = 0;
    Carve(void* b, uint64_t s) : base(static_cast<uint8_t*>(b)), size(s) {}
    template <typename T>
    T* take(uint64_t bytes) {
        const uint64_t at = align256(used);
        used = at + bytes;
        return reinterpret_cast<T*>(base + at);
    }
    bool ok() const { return used <= size; }
};

bool null_any() { return false; }
template <typename P, typename... R>
bool null_any(P p, R... rest) {
    return p == nullptr || null_any(rest...);
}

}  // namespace
}  // namespace dav2cuda

using namespace dav2cuda;

#define REQUIRE(cond, msg) \
    do {                   \
        if (!(cond)) return set_error(DAV2CUDA_INVALID_ARGUMENT, msg); \
    } while (0)

extern "C" {

const char* dav2cuda_last_error(void) { return t_last_error.c_str(); }

const char* dav2cuda_build_info(void) {
    return "dav2cuda sm_100a: tcgen05 GEMM (TMA, TMEM, kind::f16 / kind::i8), flash attention, "
           "bandwidth-bound row/elementwise/resample kernels";
}

int dav2cuda_device_error(void) {
    cudaDeviceSynchronize();
    int value = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&value, g_device_error, sizeof(int)) != cudaSuccess) return -1;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    return value;
}

int dav2cuda_wait_probe(uint64_t limit_ns, uint32_t arrive, void* stream) {
    REQUIRE(limit_ns > 0 && limit_ns <= 1000000000ull, "wait probe: limit must be in (0, 1 s]");
    int* err = device_error_word();
    if (!err) return set_error(DAV2CUDA_INTERNAL_ERROR, "wait probe: no device error word");
    wait_probe_kernel<<<1, 32, 0, as_stream(stream)>>>(limit_ns, arrive, err);
    return check_launch("wait_probe");
}

uint64_t dav2cuda_launch_count(int reset) {
    return reset ? g_launches.exchange(0) : g_launches.load();
}

int dav2cuda_layer_norm(float* output, const float* input, const float* weight, const float* bias, uint32_t rows,
                        uint32_t columns, float epsilon, void* stream) {
    REQUIRE(rows != 0 && columns != 0 && epsilon > 0.0f, "invalid layer norm parameters");
    REQUIRE(!null_any(output, input, weight, bias), "layer norm: null buffer");
    return launch_layer_norm(output, nullptr, input, weight, bias, rows, columns, epsilon, kLnOutF32, 1, 1, 0,
                             as_stream(stream));
}

int dav2cuda_gelu(float* output, const float* input, uint64_t count, void* stream) {
    REQUIRE(count != 0 && !null_any(output, input), "invalid GELU parameters");
    return launch_gelu(output, input, count, as_stream(stream));
}

int dav2cuda_softmax_rows(float* output, const float* input, uint64_t rows, uint32_t columns, float scale,
                          void* stream) {
    REQUIRE(rows != 0 && columns != 0 && !null_any(output, input), "invalid softmax parameters");
    return launch_softmax(output, input, rows, columns, scale, as_stream(stream));
}

int dav2cuda_add_scaled(float* output, const float* residual, const float* addend, const float* scale,
                        uint64_t count, uint32_t columns, void* stream) {
    REQUIRE(count != 0 && columns != 0 && count % columns == 0, "invalid add-scaled dimensions");
    REQUIRE(!null_any(output, residual, addend, scale), "add-scaled: null buffer");
    return launch_add_scaled(output, residual, addend, scale, count, columns, as_stream(stream));
}

int dav2cuda_relu(float* output, const float* input, uint64_t count, void* stream) {
    REQUIRE(!null_any(output, input), "ReLU: null buffer");
    if (count == 0) return DAV2CUDA_OK;
    return launch_relu(output, input, count, as_stream(stream));
}

int dav2cuda_add(float* output, const float* left, const float* right, uint64_t count, void* stream) {
    REQUIRE(!null_any(output, left, right), "add: null buffer");
    if (count == 0) return DAV2CUDA_OK;
    return launch_add(output, left, right, count, as_stream(stream));
}

int dav2cuda_sigmoid_scale(float* output, const float* input, uint64_t count, float scale, void* stream) {
    REQUIRE(!null_any(output, input), "sigmoid_scale: null buffer");
    if (count == 0) return DAV2CUDA_OK;
    return launch_sigmoid_scale(output, input, count, scale, as_stream(stream));
}

int dav2cuda_bilinear_align_true(float* output, const float* input, uint32_t iw, uint32_t ih, uint32_t ow,
                                 uint32_t oh, uint32_t channels, void* stream) {
    REQUIRE(iw && ih && ow && oh && channels, "invalid bilinear dimensions");
    REQUIRE(!null_any(output, input), "bilinear: null buffer");
    return launch_bilinear_align<float, float>(output, input, iw, ih, ow, oh, channels, as_stream(stream));
}

int dav2cuda_bilinear_align_nhwc_16(void* output, const void* input, uint32_t batch, uint32_t iw, uint32_t ih,
                                    uint32_t ow, uint32_t oh, uint32_t channels, uint32_t bf16, void* stream) {
    REQUIRE(batch && iw && ih && ow && oh && channels, "invalid bilinear dimensions");
    REQUIRE(!null_any(output, input), "bilinear: null buffer");
    REQUIRE(reinterpret_cast<uintptr_t>(output) % 16 == 0 && reinterpret_cast<uintptr_t>(input) % 16 == 0,
            "bilinear: buffers must be 16-byte aligned");
    if (bf16)
        return launch_bilinear_nhwc<__nv_bfloat16>(static_cast<__nv_bfloat16*>(output),
                                                   static_cast<const __nv_bfloat16*>(input), batch, ih, iw, oh, ow,
                                                   channels, as_stream(stream));
    return launch_bilinear_nhwc<__half>(static_cast<__half*>(output), static_cast<const __half*>(input), batch, ih,
                                        iw, oh, ow, channels, as_stream(stream));
}

int dav2cuda_reduce_minmax(const float* input, float* range, uint64_t count, void* stream) {
    REQUIRE(count != 0, "empty depth reduction");
    REQUIRE(!null_any(input, range), "reduce_minmax: null buffer");
    return launch_minmax(input, range, count, as_stream(stream));
}

int dav2cuda_normalize_relative(float* depth, const float* range, uint64_t count, void* stream) {
    REQUIRE(count != 0, "empty relative depth");
    REQUIRE(!null_any(depth, range), "normalize: null buffer");
    return launch_normalize(depth, range, count, 0.0f, as_stream(stream));
}

int dav2cuda_normalize_metric(float* depth, const float* range, uint64_t count, float maximum_depth,
                              void* stream) {
    REQUIRE(count != 0 && maximum_depth > 0.0f, "invalid metric depth normalization");
    REQUIRE(!null_any(depth, range), "normalize: null buffer");
    return launch_normalize(depth, range, count, maximum_depth, as_stream(stream));
}

int dav2cuda_preprocess_u32(float* output_chw, const uint32_t* pixels, uint32_t sw, uint32_t sh,
                            uint32_t row_stride_pixels, uint32_t rgba_order, uint32_t dw, uint32_t dh,
                            void* stream) {
    REQUIRE(sw && sh && dw && dh && row_stride_pixels >= sw, "invalid preprocessing dimensions");
    REQUIRE(!null_any(output_chw, pixels), "preprocess: null buffer");
    return launch_preprocess_u32(output_chw, pixels, sw, sh, row_stride_pixels, rgba_order, dw, dh,
                                 as_stream(stream));
}

int dav2cuda_preprocess_bgr8(float* output_chw, const uint8_t* bgr, uint32_t batch, uint32_t sw, uint32_t sh,
                             uint64_t row_stride, uint64_t image_stride, uint32_t dw, uint32_t dh, void* stream) {
    REQUIRE(batch && sw && sh && dw && dh && row_stride >= 3ull * sw, "invalid source image");
    REQUIRE(batch == 1 || image_stride >= row_stride * sh, "invalid image stride");
    REQUIRE(!null_any(output_chw, bgr), "preprocess: null buffer");
    return launch_preprocess_bgr8(output_chw, bgr, batch, sw, sh, row_stride, image_stride, dw, dh, 0,
                                  as_stream(stream));
}

int dav2cuda_preprocess_bgr8_bilinear(float* output_chw, const uint8_t* bgr, uint32_t batch, uint32_t sw,
                                      uint32_t sh, uint64_t row_stride, uint64_t image_stride, uint32_t dw,
                                      uint32_t dh, void* stream) {
    REQUIRE(batch && sw && sh && dw && dh && row_stride >= 3ull * sw, "invalid source image");
    REQUIRE(batch == 1 || image_stride >= row_stride * sh, "invalid image stride");
    REQUIRE(!null_any(output_chw, bgr), "preprocess: null buffer");
    return launch_preprocess_bgr8(output_chw, bgr, batch, sw, sh, row_stride, image_stride, dw, dh, 1,
                                  as_stream(stream));
}

int dav2cuda_quantize_rows_s8(uint32_t* packed, float* scales, const float* input, uint32_t rows,
                              uint32_t columns, uint64_t input_offset, void* stream) {
    REQUIRE(rows && columns && columns % 4 == 0, "invalid INT8 row quantization dimensions");
    REQUIRE(!null_any(packed, scales, input), "quantize: null buffer");
    return launch_quantize_rows<float>(packed, scales, input, rows, columns, input_offset, rows,
                                       (uint64_t)rows * columns, columns, columns / 4, as_stream(stream));
}

int dav2cuda_pack_weight_s8(uint8_t* codes, float* scales, const float* weight, uint32_t layout, uint32_t rows,
                            uint32_t columns, uint32_t padded_columns, uint32_t output_channels, uint32_t kernel,
                            uint32_t input_channels, void* stream) {
    REQUIRE(rows && columns && padded_columns >= columns && layout <= 2, "invalid weight packing dimensions");
    REQUIRE(layout != 1 || (output_channels && kernel && input_channels == columns &&
                            rows == kernel * kernel * output_channels),
            "weight packing: conv-transpose shape mismatch");
    REQUIRE(layout != 2 || (output_channels == rows && kernel && input_channels &&
                            columns == kernel * kernel * input_channels),
            "weight packing: convolution shape mismatch");
    REQUIRE(!null_any(codes, scales, weight), "weight packing: null buffer");
    return launch_pack_weight_s8(codes, scales, weight, (int)layout, rows, columns, padded_columns, output_channels,
                                 kernel, input_channels, as_stream(stream));
}

int dav2cuda_im2col_quantize_s8(uint32_t* packed, float* scales, const float* input, uint32_t iw, uint32_t ih,
                                uint32_t ic, uint32_t ow, uint32_t oh, uint32_t kernel, uint32_t stride,
                                int32_t padding, void* stream) {
    REQUIRE(iw && ih && ic && ow && oh && kernel && stride && padding >= 0, "invalid im2col dimensions");
    REQUIRE(!null_any(packed, scales, input), "im2col: null buffer");
    return launch_im2col_quantize(packed, scales, input, 1, iw, ih, ic, ow, oh, kernel, stride, padding,
                                  (ic * kernel * kernel + 3) / 4, as_stream(stream));
}

int dav2cuda_linear_s8_packed(float* output, const uint32_t* packed_input, const uint32_t* packed_weight,
                              const float* input_scales, const float* weight_scales, const float* bias,
                              uint32_t rows, uint32_t input_columns, uint32_t output_columns,
                              uint32_t output_row_offset, uint32_t output_row_stride, uint32_t output_transposed,
                              uint32_t has_bias, void* stream) {
    REQUIRE(rows && input_columns && output_columns, "invalid INT8 linear dimensions");
    REQUIRE(input_columns % 16 == 0, "INT8 linear: input_columns must be a multiple of 16");
    REQUIRE(!null_any(output, packed_input, packed_weight, input_scales, weight_scales), "INT8 linear: null buffer");
    REQUIRE(!has_bias || bias, "INT8 linear: null bias");
    GemmArgs g;
    g.elem = kElemS8;
    g.a = packed_input;
    g.lda = input_columns;
    g.b = packed_weight;
    g.ldb = input_columns;
    g.m = rows;
    g.n = output_columns;
    g.k = input_columns;
    g.flags = kEpiDequant | (has_bias ? kEpiBias : 0u);
    g.s_in = input_scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.out = output;
    if (output_transposed) {
        g.out_kind = kOutF32Planar;
        g.img_stride = 0;
        g.col_stride = output_row_stride;
        g.row_offset = output_row_offset;
    } else {
        g.out_kind = kOutF32Rows;
        g.ldo = output_columns;
        g.rows_per_img = rows;
        g.out_rows_per_img = rows + output_row_offset;
        g.row_offset = output_row_offset;
    }
    return launch_gemm(g, as_stream(stream));
}

uint64_t dav2cuda_linear_int8_workspace_size(uint32_t rows, uint32_t input_columns, uint32_t output_columns) {
    const uint64_t kp = ((uint64_t)input_columns + 15) / 16 * 16;  // 64-bit: no wrap near UINT32_MAX
    return align256((uint64_t)rows * kp) + align256((uint64_t)rows * 4) +
           (kp != input_columns ? align256((uint64_t)output_columns * kp) : 0) + 256;
}

int dav2cuda_linear_int8(float* output, const float* input, const uint32_t* int8_weight, const float* weight_scales,
                         const float* bias, uint32_t rows, uint32_t input_columns, uint32_t output_columns,
                         uint32_t gelu, void* workspace, uint64_t workspace_bytes, void* stream) {
    REQUIRE(rows && input_columns && output_columns && input_columns % 4 == 0, "invalid INT8 linear dimensions");
    REQUIRE(input_columns <= 0xFFFFFFF0u, "INT8 linear: input_columns too large");
    REQUIRE(!null_any(output, input, int8_weight, weight_scales, bias, workspace), "INT8 linear: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_linear_int8_workspace_size(rows, input_columns, output_columns),
            "INT8 linear: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t kp = round_up(input_columns, 16);
    Carve ws(workspace, workspace_bytes);
    uint32_t* codes = ws.take<uint32_t>((uint64_t)rows * kp);
    float* scales = ws.take<float>((uint64_t)rows * 4);
    const uint32_t* w = int8_weight;
    if (kp != input_columns) {
        uint8_t* wp = ws.take<uint8_t>((uint64_t)output_columns * kp);
        if (int rc = pad_byte_rows(wp, int8_weight, output_columns, input_columns, kp, st)) return rc;
        w = reinterpret_cast<const uint32_t*>(wp);
    }
    if (int rc = launch_quantize_rows<float>(codes, scales, input, rows, input_columns, 0, rows,
                                             (uint64_t)rows * input_columns, input_columns, kp / 4, st))
        return rc;
    GemmArgs g;
    g.elem = kElemS8;
    g.a = codes;
    g.lda = kp;
    g.b = w;
    g.ldb = kp;
    g.m = rows;
    g.n = output_columns;
    g.k = kp;
    g.flags = kEpiDequant | kEpiBias | (gelu ? kEpiGelu : 0u);
    g.s_in = scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.out = output;
    g.out_kind = kOutF32Rows;
    g.ldo = output_columns;
    return launch_gemm(g, st);
}

// The encoder's int8 residual update in the form the executor runs it for
// proj and fc2: rows quantized into the workspace, then one GEMM whose
// epilogue reads each residual row, adds (dequant + bias) * layer_scale in the
// reference's order and writes the row back in place.
int dav2cuda_linear_int8_residual(float* residual, const float* input, const uint32_t* int8_weight,
                                  const float* weight_scales, const float* bias, const float* layer_scale,
                                  uint32_t rows, uint32_t input_columns, uint32_t output_columns, void* workspace,
                                  uint64_t workspace_bytes, void* stream) {
    REQUIRE(rows && input_columns && output_columns && input_columns % 4 == 0, "invalid INT8 residual dimensions");
    REQUIRE(input_columns <= 0xFFFFFFF0u, "INT8 residual: input_columns too large");
    REQUIRE(!null_any(residual, input, int8_weight, weight_scales, bias, layer_scale, workspace),
            "INT8 residual: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_linear_int8_workspace_size(rows, input_columns, output_columns),
            "INT8 residual: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t kp = round_up(input_columns, 16);
    Carve ws(workspace, workspace_bytes);
    uint32_t* codes = ws.take<uint32_t>((uint64_t)rows * kp);
    float* scales = ws.take<float>((uint64_t)rows * 4);
    const uint32_t* w = int8_weight;
    if (kp != input_columns) {
        uint8_t* wp = ws.take<uint8_t>((uint64_t)output_columns * kp);
        if (int rc = pad_byte_rows(wp, int8_weight, output_columns, input_columns, kp, st)) return rc;
        w = reinterpret_cast<const uint32_t*>(wp);
    }
    if (int rc = launch_quantize_rows<float>(codes, scales, input, rows, input_columns, 0, rows,
                                             (uint64_t)rows * input_columns, input_columns, kp / 4, st))
        return rc;
    GemmArgs g;
    g.elem = kElemS8;
    g.a = codes;
    g.lda = kp;
    g.b = w;
    g.ldb = kp;
    g.m = rows;
    g.n = output_columns;
    g.k = kp;
    g.flags = kEpiDequant | kEpiBias | kEpiLayerScale;
    g.s_in = scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.gamma = layer_scale;
    g.res1 = residual;
    g.out = residual;
    g.out_kind = kOutF32Rows;
    g.ldo = output_columns;
    return launch_gemm(g, st);
}

// The graph's channels-last im2col-quantize (f32 maps): one block per output
// pixel, columns in (ky, kx, c) order, row_bytes apart, zero past k*k*c.
int dav2cuda_im2col_quantize_nhwc(uint8_t* codes, float* scales, const float* input, uint32_t batch,
                                  uint32_t height, uint32_t width, uint32_t channels, uint32_t kernel,
                                  uint32_t stride, uint32_t padding, uint32_t row_bytes, void* stream) {
    REQUIRE(batch && height && width && channels && kernel && stride && (uint64_t)height + 2ull * padding >= kernel &&
                (uint64_t)width + 2ull * padding >= kernel,
            "invalid channels-last im2col dimensions");
    const uint64_t cols = (uint64_t)kernel * kernel * channels;
    REQUIRE(cols < 0x80000000ull, "channels-last im2col: kernel*kernel*channels too large");
    REQUIRE(row_bytes >= cols, "channels-last im2col: row_bytes below kernel*kernel*channels");
    REQUIRE(!null_any(codes, scales, input), "channels-last im2col: null buffer");
    const uint32_t oh = (height + 2 * padding - kernel) / stride + 1, ow = (width + 2 * padding - kernel) / stride + 1;
    REQUIRE((uint64_t)batch * oh * ow <= 0x7FFFFFFFull, "channels-last im2col: too many output pixels");
    return launch_im2col_quantize_nhwc<float>(codes, scales, input, batch, height, width, channels, channels, kernel,
                                              stride, padding, oh, ow, row_bytes, as_stream(stream));
}

uint64_t dav2cuda_conv2d_int8_workspace_size(uint32_t iw, uint32_t ih, uint32_t ic, uint32_t oc, uint32_t k,
                                             uint32_t s, uint32_t p) {
    if (!iw || !ih || !k || !s || iw + 2 * p < k || ih + 2 * p < k) return 0;
    const uint64_t ow = (iw + 2 * p - k) / s + 1, oh = (ih + 2 * p - k) / s + 1;
    const uint32_t kp = round_up(ic * k * k, 16);
    return align256(ow * oh * kp) + align256(ow * oh * 4) + align256((uint64_t)oc * kp) + 256;
}

int dav2cuda_conv2d_int8(float* output, const float* input, const uint32_t* int8_weight, const float* weight_scales,
                         const float* bias, uint32_t iw, uint32_t ih, uint32_t ic, uint32_t oc, uint32_t k,
                         uint32_t s, uint32_t p, uint32_t has_bias, void* workspace, uint64_t workspace_bytes,
                         void* stream) {
    REQUIRE(iw && ih && ic && oc && k && s && iw + 2 * p >= k && ih + 2 * p >= k,
            "invalid INT8 convolution dimensions");
    REQUIRE((ic * k * k) % 4 == 0, "INT8 convolution inner size is not packed");
    REQUIRE(!null_any(output, input, int8_weight, weight_scales, workspace), "INT8 convolution: null buffer");
    REQUIRE(!has_bias || bias, "INT8 convolution: null bias");
    REQUIRE(workspace_bytes >= dav2cuda_conv2d_int8_workspace_size(iw, ih, ic, oc, k, s, p),
            "INT8 convolution: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t ow = (iw + 2 * p - k) / s + 1, oh = (ih + 2 * p - k) / s + 1;
    const uint32_t K = ic * k * k, kp = round_up(K, 16);
    const uint64_t rows = (uint64_t)ow * oh;
    Carve ws(workspace, workspace_bytes);
    uint32_t* codes = ws.take<uint32_t>(rows * kp);
    float* scales = ws.take<float>(rows * 4);
    const void* w = int8_weight;
    if (kp != K) {
        uint8_t* wp = ws.take<uint8_t>((uint64_t)oc * kp);
        if (int rc = pad_byte_rows(wp, int8_weight, oc, K, kp, st)) return rc;
        w = wp;
    }
    if (int rc = launch_im2col_quantize(codes, scales, input, 1, iw, ih, ic, ow, oh, k, s, (int)p, kp / 4, st))
        return rc;
    GemmArgs g;
    g.elem = kElemS8;
    g.a = codes;
    g.lda = kp;
    g.b = w;
    g.ldb = kp;
    g.m = (uint32_t)rows;
    g.n = oc;
    g.k = kp;
    g.flags = kEpiDequant | (has_bias ? kEpiBias : 0u);
    g.s_in = scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.out = output;
    g.out_kind = kOutF32Planar;
    g.col_stride = rows;
    return launch_gemm(g, st);
}

uint64_t dav2cuda_conv_transpose_int8_workspace_size(uint32_t iw, uint32_t ih, uint32_t ic, uint32_t oc, uint32_t k) {
    const uint32_t kp = round_up(ic, 16);
    const uint64_t rows = (uint64_t)iw * ih;
    return align256(rows * kp) + align256(rows * 4) + align256((uint64_t)k * k * oc * kp) +
           align256((uint64_t)k * k * oc * 4) + 256;
}

int dav2cuda_conv_transpose_int8(float* output, const float* input, const uint32_t* int8_weight,
                                 const float* weight_scales, const float* bias, uint32_t iw, uint32_t ih, uint32_t ic,
                                 uint32_t oc, uint32_t k, void* workspace, uint64_t workspace_bytes, void* stream) {
    REQUIRE(iw && ih && ic && oc && k && ic % 4 == 0, "invalid INT8 transposed convolution");
    REQUIRE(!null_any(output, input, int8_weight, weight_scales, bias, workspace), "INT8 transposed conv: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_conv_transpose_int8_workspace_size(iw, ih, ic, oc, k),
            "INT8 transposed convolution: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t kp = round_up(ic, 16);
    const uint64_t rows = (uint64_t)iw * ih;
    const uint32_t wrows = k * k * oc;
    Carve ws(workspace, workspace_bytes);
    uint32_t* codes = ws.take<uint32_t>(rows * kp);
    float* scales = ws.take<float>(rows * 4);
    const void* w = int8_weight;
    if (kp != ic) {
        uint8_t* wp = ws.take<uint8_t>((uint64_t)wrows * kp);
        if (int rc = pad_byte_rows(wp, int8_weight, wrows, ic, kp, st)) return rc;
        w = wp;
    }
    // per-pixel channel quantization: im2col with k=1 (src/operators.cpp:1951-1957)
    if (int rc = launch_im2col_quantize(codes, scales, input, 1, iw, ih, ic, iw, ih, 1, 1, 0, kp / 4, st)) return rc;
    GemmArgs g;
    g.elem = kElemS8;
    g.a = codes;
    g.lda = kp;
    g.b = w;
    g.ldb = kp;
    g.m = (uint32_t)rows;
    g.n = wrows;
    g.k = kp;
    g.flags = kEpiDequant;
    g.s_in = scales;
    g.s_w = weight_scales;
    g.out = output;
    g.out_kind = kOutConvTF32;
    g.convt_k = k;
    g.convt_cout = oc;
    g.convt_w = iw;
    g.convt_h = ih;
    // bias is per output channel, not per GEMM column: added by the scatter
    // through a column-expanded bias below.
    float* bias_cols = ws.take<float>((uint64_t)wrows * 4);
    if (!ws.ok()) return set_error(DAV2CUDA_INVALID_ARGUMENT, "INT8 transposed convolution: workspace is too small");
    for (uint32_t t = 0; t < k * k; ++t)
        if (cudaMemcpyAsync(bias_cols + (uint64_t)t * oc, bias, oc * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return set_error(DAV2CUDA_LAUNCH_FAILED, "INT8 transposed convolution: bias copy failed");
    g.flags |= kEpiBias;
    g.bias = bias_cols;
    return launch_gemm(g, st);
}

// ------------------------------------------------------------ token ops
// VulkanOperators::prepare_tokens (src/operators.cpp:1211-1406): patch
// embedding (conv 14/14 as a GEMM over 588-column patches, padded to 592),
// class token at row 0, the 37x37 positional grid bicubic-resized to the
// patch grid (identity at 37x37) and added. tokens = 1 + (w/14)(h/14).
uint64_t dav2cuda_prepare_tokens_workspace_size(uint32_t w, uint32_t h, uint32_t embedding) {
    const uint64_t hw = (uint64_t)(w / 14) * (h / 14);
    return align256(hw * embedding * 4) + align256(hw * 592 * 2) + align256(hw * 4) +
           align256((uint64_t)embedding * 592 * 2) + 256;
}

namespace {

int prepare_tokens_common(float* output, const float* image, const void* weight, const float* weight_scales,
                          const float* bias, const float* class_token, const float* position, uint32_t w,
                          uint32_t h, uint32_t e, int elem, void* workspace, uint64_t workspace_bytes,
                          cudaStream_t st) {
    const uint32_t pw = w / 14, ph = h / 14, hw = pw * ph;
    Carve ws(workspace, workspace_bytes);
    float* interp = ws.take<float>((uint64_t)hw * e * 4);
    void* patches = ws.take<uint8_t>((uint64_t)hw * 592 * 2);
    float* scales = ws.take<float>((uint64_t)hw * 4);
    void* wts = ws.take<uint8_t>((uint64_t)e * 592 * 2);
    if (!ws.ok()) return set_error(DAV2CUDA_INVALID_ARGUMENT, "prepare_tokens: workspace is too small");
    if (int rc = launch_position_bicubic(interp, position, e, pw, ph, st)) return rc;
    if (int rc = launch_fill_tokens(output, class_token, position, interp, e, hw + 1, 1, st)) return rc;
    int rc = 0;
    if (elem == kElemS8) {
        rc = launch_im2col_quantize(static_cast<uint32_t*>(patches), scales, image, 1, w, h, 3, pw, ph, 14, 14, 0,
                                    592 / 4, st);
        if (!rc) rc = pad_byte_rows(static_cast<uint8_t*>(wts), weight, e, 588, 592, st);
    } else if (elem == kElemBF16) {
        rc = launch_patch_im2col<__nv_bfloat16>(static_cast<__nv_bfloat16*>(patches), image, 1, h, w, 592, st);
        if (!rc)
            rc = launch_pad_rows_half<__nv_bfloat16>(static_cast<__nv_bfloat16*>(wts), static_cast<const float*>(weight),
                                                     e, 588, 592, st);
    } else {
        rc = launch_patch_im2col<__half>(static_cast<__half*>(patches), image, 1, h, w, 592, st);
        if (!rc)
            rc = launch_pad_rows_half<__half>(static_cast<__half*>(wts), static_cast<const float*>(weight), e, 588,
                                              592, st);
    }
    if (rc) return rc;
    GemmArgs g;
    g.elem = elem;
    g.a = patches;
    g.lda = 592;
    g.b = wts;
    g.ldb = 592;
    g.m = hw;
    g.n = e;
    g.k = 592;
    g.flags = kEpiBias | kEpiResidual1 | (elem == kElemS8 ? kEpiDequant : 0u);
    g.s_in = scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.res1 = output;  // the class row and positions written above: out = patch + bias + position
    g.out = output;
    g.out_kind = kOutF32Rows;
    g.ldo = e;
    g.rows_per_img = hw;
    g.out_rows_per_img = hw + 1;
    g.row_offset = 1;
    return launch_gemm(g, st);
}

}  // namespace

int dav2cuda_prepare_tokens_half(float* output, const float* image, const float* patch_weight, const float* patch_bias,
                                 const float* class_token, const float* position, uint32_t w, uint32_t h,
                                 uint32_t embedding, uint32_t precision, void* workspace, uint64_t workspace_bytes,
                                 void* stream) {
    REQUIRE(w && h && w % 14 == 0 && h % 14 == 0 && embedding && (precision == 1 || precision == 2),
            "invalid patch embedding dimensions");
    REQUIRE(!null_any(output, image, patch_weight, patch_bias, class_token, position, workspace),
            "prepare_tokens: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_prepare_tokens_workspace_size(w, h, embedding),
            "prepare_tokens: workspace is too small");
    return prepare_tokens_common(output, image, patch_weight, nullptr, patch_bias, class_token, position, w, h,
                                 embedding, precision == 1 ? kElemBF16 : kElemF16, workspace, workspace_bytes,
                                 as_stream(stream));
}

int dav2cuda_prepare_tokens_int8(float* output, const float* image, const uint32_t* patch_int8_weight,
                                 const float* patch_weight_scales, const float* patch_bias, const float* class_token,
                                 const float* position, uint32_t w, uint32_t h, uint32_t embedding, void* workspace,
                                 uint64_t workspace_bytes, void* stream) {
    REQUIRE(w && h && w % 14 == 0 && h % 14 == 0 && embedding, "invalid patch embedding dimensions");
    REQUIRE(!null_any(output, image, patch_int8_weight, patch_weight_scales, patch_bias, class_token, position,
                      workspace),
            "prepare_tokens: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_prepare_tokens_workspace_size(w, h, embedding),
            "prepare_tokens: workspace is too small");
    return prepare_tokens_common(output, image, patch_int8_weight, patch_weight_scales, patch_bias, class_token,
                                 position, w, h, embedding, kElemS8, workspace, workspace_bytes, as_stream(stream));
}

// VulkanOperators::project_tokens* (src/operators.cpp:1408-1526): 1x1
// convolution of the patch tokens (the class row skipped) into planar
// output [Cout][height*width].
uint64_t dav2cuda_project_tokens_workspace_size(uint32_t w, uint32_t h, uint32_t embedding, uint32_t output_channels) {
    const uint64_t hw = (uint64_t)w * h;
    const uint64_t kp = ((uint64_t)embedding + 15) / 16 * 16;
    return align256(hw * kp * 2) + align256(hw * 4) + align256((uint64_t)output_channels * kp * 2) + 256;
}

namespace {

int project_tokens_common(float* output, const float* tokens, const void* weight, const float* weight_scales,
                          const float* bias, uint32_t w, uint32_t h, uint32_t e, uint32_t co, int elem,
                          void* workspace, uint64_t workspace_bytes, cudaStream_t st) {
    const uint32_t hw = w * h, kp = round_up(e, 16);
    Carve ws(workspace, workspace_bytes);
    void* a = ws.take<uint8_t>((uint64_t)hw * kp * 2);
    float* scales = ws.take<float>((uint64_t)hw * 4);
    void* b = ws.take<uint8_t>((uint64_t)co * kp * 2);
    if (!ws.ok()) return set_error(DAV2CUDA_INVALID_ARGUMENT, "project_tokens: workspace is too small");
    int rc = 0;
    const void* wb = b;
    if (elem == kElemS8) {
        // quantize_rows_int8_fused with the input offset of one row (src/operators.cpp:1510-1522)
        rc = launch_quantize_rows<float>(static_cast<uint32_t*>(a), scales, tokens, hw, e, e, hw, (uint64_t)hw * e, e,
                                         kp / 4, st);
        if (!rc && kp != e) rc = pad_byte_rows(static_cast<uint8_t*>(b), weight, co, e, kp, st);
        if (kp == e) wb = weight;
    } else if (elem == kElemBF16) {
        rc = launch_pad_rows_half<__nv_bfloat16>(static_cast<__nv_bfloat16*>(a), tokens + e, hw, e, kp, st);
        if (!rc)
            rc = launch_pad_rows_half<__nv_bfloat16>(static_cast<__nv_bfloat16*>(b), static_cast<const float*>(weight),
                                                     co, e, kp, st);
    } else {
        rc = launch_pad_rows_half<__half>(static_cast<__half*>(a), tokens + e, hw, e, kp, st);
        if (!rc) rc = launch_pad_rows_half<__half>(static_cast<__half*>(b), static_cast<const float*>(weight), co, e, kp, st);
    }
    if (rc) return rc;
    GemmArgs g;
    g.elem = elem;
    g.a = a;
    g.lda = kp;
    g.b = wb;
    g.ldb = kp;
    g.m = hw;
    g.n = co;
    g.k = kp;
    g.flags = (bias ? kEpiBias : 0u) | (elem == kElemS8 ? kEpiDequant : 0u);
    g.s_in = scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.out = output;
    g.out_kind = kOutF32Planar;
    g.img_stride = 0;
    g.col_stride = hw;
    g.row_offset = 0;
    return launch_gemm(g, st);
}

}  // namespace

int dav2cuda_project_tokens_half(float* output, const float* tokens, const float* weight, const float* bias,
                                 uint32_t w, uint32_t h, uint32_t embedding, uint32_t output_channels,
                                 uint32_t precision, void* workspace, uint64_t workspace_bytes, void* stream) {
    REQUIRE(w && h && embedding && output_channels && (precision == 1 || precision == 2),
            "invalid token projection dimensions");
    REQUIRE(!null_any(output, tokens, weight, workspace), "project_tokens: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_project_tokens_workspace_size(w, h, embedding, output_channels),
            "project_tokens: workspace is too small");
    return project_tokens_common(output, tokens, weight, nullptr, bias, w, h, embedding, output_channels,
                                 precision == 1 ? kElemBF16 : kElemF16, workspace, workspace_bytes, as_stream(stream));
}

int dav2cuda_project_tokens_int8(float* output, const float* tokens, const uint32_t* int8_weight,
                                 const float* weight_scales, const float* bias, uint32_t w, uint32_t h,
                                 uint32_t embedding, uint32_t output_channels, void* workspace,
                                 uint64_t workspace_bytes, void* stream) {
    REQUIRE(w && h && embedding && output_channels && embedding % 4 == 0, "invalid token projection dimensions");
    REQUIRE(!null_any(output, tokens, int8_weight, weight_scales, workspace), "project_tokens: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_project_tokens_workspace_size(w, h, embedding, output_channels),
            "project_tokens: workspace is too small");
    return project_tokens_common(output, tokens, int8_weight, weight_scales, bias, w, h, embedding, output_channels,
                                 kElemS8, workspace, workspace_bytes, as_stream(stream));
}

// VulkanOperators::conv_transpose_nonoverlap (src/operators.cpp:1807-1906)
// with 16-bit operands: kernel == stride k, weight [Ci][Co][k][k], planar
// f32 in [Ci][H][W] and out [Co][H*k][W*k].
uint64_t dav2cuda_conv_transpose_half_workspace_size(uint32_t w, uint32_t h, uint32_t ic, uint32_t oc, uint32_t k) {
    const uint64_t cp = ((uint64_t)ic + 7) / 8 * 8;
    return align256((uint64_t)w * h * cp * 2) + align256((uint64_t)k * k * oc * cp * 2) +
           align256((uint64_t)k * k * oc * 4) + 256;
}

int dav2cuda_conv_transpose_half(float* output, const float* input, const float* weight, const float* bias,
                                 uint32_t w, uint32_t h, uint32_t ic, uint32_t oc, uint32_t k, uint32_t precision,
                                 void* workspace, uint64_t workspace_bytes, void* stream) {
    REQUIRE(w && h && ic && oc && k && (precision == 1 || precision == 2), "invalid transposed convolution");
    REQUIRE(!null_any(output, input, weight, bias, workspace), "transposed convolution: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_conv_transpose_half_workspace_size(w, h, ic, oc, k),
            "transposed convolution: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t cp = round_up(ic, 8), wrows = k * k * oc;
    const bool bf = precision == 1;
    Carve ws(workspace, workspace_bytes);
    void* a = ws.take<uint8_t>((uint64_t)w * h * cp * 2);
    void* b = ws.take<uint8_t>((uint64_t)wrows * cp * 2);
    float* bias_cols = ws.take<float>((uint64_t)wrows * 4);
    int rc = bf ? launch_nchw_to_nhwc<__nv_bfloat16>(static_cast<__nv_bfloat16*>(a), input, 1, ic, h, w, cp, st)
                : launch_nchw_to_nhwc<__half>(static_cast<__half*>(a), input, 1, ic, h, w, cp, st);
    if (!rc)
        rc = bf ? launch_half_weight<__nv_bfloat16>(static_cast<__nv_bfloat16*>(b), weight, 1, wrows, ic, cp, oc, k, ic,
                                                    cp, st)
                : launch_half_weight<__half>(static_cast<__half*>(b), weight, 1, wrows, ic, cp, oc, k, ic, cp, st);
    if (!rc) rc = launch_expand_bias(bias_cols, bias, oc, k * k, st);
    if (rc) return rc;
    GemmArgs g;
    g.elem = bf ? kElemBF16 : kElemF16;
    g.a = a;
    g.lda = cp;
    g.b = b;
    g.ldb = cp;
    g.m = w * h;
    g.n = wrows;
    g.k = cp;
    g.flags = kEpiBias;
    g.bias = bias_cols;
    g.out = output;
    g.out_kind = kOutConvTF32;
    g.convt_k = k;
    g.convt_cout = oc;
    g.convt_w = w;
    g.convt_h = h;
    return launch_gemm(g, st);
}

// BASELINE configuration 2(d): the reference's conv2d_int8 (3x3, pad 1;
// src/operators.cpp:1735-1805) then bilinear_align_true 2x
// (src/operators.cpp:1978-2012), batched. Row scales come exactly from a
// per-pixel channel abs-max pre-pass and a 3x3 maximum, so the im2col
// quantizer needs no row reduction and reads the planar input directly; its
// codes are in (ky, kx, c) column order and the weight codes are permuted
// alike, which leaves each row's scale, codes and integer dot products
// unchanged.
uint64_t dav2cuda_conv3x3_int8_up2_workspace_size(uint32_t batch, uint32_t w, uint32_t h, uint32_t ic, uint32_t oc) {
    const uint32_t kp = round_up(ic * 9, 16);
    const uint64_t rows = (uint64_t)batch * w * h;
    return align256(rows * 4) + align256(rows * kp) + align256(rows * 4) + align256((uint64_t)oc * kp) +
           align256((uint64_t)batch * oc * w * h * 4) + 256;
}

int dav2cuda_conv3x3_int8_up2(float* output, const float* input, const uint32_t* int8_weight,
                              const float* weight_scales, const float* bias, uint32_t batch, uint32_t w, uint32_t h,
                              uint32_t ic, uint32_t oc, void* workspace, uint64_t workspace_bytes, void* stream) {
    REQUIRE(batch && w && h && ic && oc && (ic * 9) % 4 == 0, "invalid INT8 convolution dimensions");
    REQUIRE(!null_any(output, input, int8_weight, weight_scales, bias, workspace), "conv3x3_int8_up2: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_conv3x3_int8_up2_workspace_size(batch, w, h, ic, oc),
            "conv3x3_int8_up2: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t K = ic * 9, kp = round_up(K, 16);
    const uint64_t hw = (uint64_t)w * h, rows = batch * hw;
    Carve ws(workspace, workspace_bytes);
    float* pix = ws.take<float>(rows * 4);
    uint8_t* codes = ws.take<uint8_t>(rows * kp);
    float* scales = ws.take<float>(rows * 4);
    uint8_t* wt = ws.take<uint8_t>((uint64_t)oc * kp);
    float* conv = ws.take<float>((uint64_t)batch * oc * hw * 4);
    int rc = launch_conv_codes_tap_major(wt, reinterpret_cast<const uint8_t*>(int8_weight), oc, ic, 9, K, kp, st);
    if (!rc) rc = launch_im2col_quantize_3x3_planar(codes, scales, pix, input, batch, ic, h, w, kp, st);
    if (rc) return rc;
    GemmArgs g;
    g.elem = kElemS8;
    g.a = codes;
    g.lda = kp;
    g.b = wt;
    g.ldb = kp;
    g.m = (uint32_t)rows;
    g.n = oc;
    g.k = kp;
    g.flags = kEpiDequant | kEpiBias;
    g.s_in = scales;
    g.s_w = weight_scales;
    g.bias = bias;
    g.out = conv;
    if (bilinear_nhwc_to_planar_supported(w, oc, 2 * w)) {
        // channels-last conv output (thread-row TMA epilogue), then the upsample
        // writes the planar result
        g.out_kind = kOutF32Rows;
        g.ldo = oc;
        if (int rc2 = launch_gemm(g, st)) return rc2;
        return launch_bilinear_nhwc_to_planar(output, conv, batch, h, w, oc, 2 * h, 2 * w, st);
    }
    g.out_kind = kOutF32Planar;
    g.rows_per_img = (uint32_t)hw;
    g.img_stride = (uint64_t)oc * hw;
    g.col_stride = hw;
    if (int rc2 = launch_gemm(g, st)) return rc2;
    return launch_bilinear_align<float, float>(output, conv, w, h, 2 * w, 2 * h, batch * oc, st);
}

int dav2cuda_conv3x3_c128_16(void* output, const void* input, const void* weight, const float* bias, uint32_t batch,
                             uint32_t width, uint32_t height, uint32_t input_channels, uint32_t bf16, void* stream) {
    REQUIRE(batch && width && height && input_channels, "invalid convolution dimensions");
    REQUIRE(!null_any(output, input, weight, bias), "conv3x3_c128: null buffer");
    REQUIRE(conv3x3_halo_supported(input_channels, 128, 128), "conv3x3_c128: input channels must be a multiple of 64");
    return launch_conv3x3_halo(output, input, weight, bias, bf16 != 0, batch, height, width, input_channels,
                               as_stream(stream));
}

int dav2cuda_conv3x3_head_16(float* depth, const void* input, const void* weight, const float* bias,
                             const float* head_weight, float head_bias, float max_depth, uint32_t batch,
                             uint32_t width, uint32_t height, uint32_t channels, uint32_t bf16, void* stream) {
    REQUIRE(batch && width && height && channels, "invalid head dimensions");
    REQUIRE(!null_any(depth, input, weight, bias, head_weight), "conv3x3_head: null buffer");
    REQUIRE(conv_head_halo_supported(channels, 32), "conv3x3_head: channels must be 64 or 128");
    return launch_conv_head_halo(depth, nullptr, input, weight, bias, head_weight, head_bias, max_depth,
                                 max_depth > 0.0f, bf16 != 0, batch, height, width, channels, as_stream(stream));
}

uint64_t dav2cuda_attention_head64_workspace_size(uint32_t batch, uint32_t tokens, uint32_t heads) {
    const uint64_t e = (uint64_t)heads * 64;
    return align256((uint64_t)batch * tokens * 3 * e * 2) + align256((uint64_t)batch * tokens * e * 2) + 256;
}

int dav2cuda_attention_head64(float* output, const float* qkv, uint32_t batch, uint32_t tokens, uint32_t heads,
                              void* workspace, uint64_t workspace_bytes, void* stream) {
    REQUIRE(batch && tokens && heads, "invalid attention dimensions");
    REQUIRE(!null_any(output, qkv, workspace), "attention: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_attention_head64_workspace_size(batch, tokens, heads),
            "attention: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint64_t e = (uint64_t)heads * 64;
    Carve ws(workspace, workspace_bytes);
    __half* q = ws.take<__half>((uint64_t)batch * tokens * 3 * e * 2);
    __half* o = ws.take<__half>((uint64_t)batch * tokens * e * 2);
    if (int rc = launch_to_half<__half>(q, qkv, (uint64_t)batch * tokens * 3 * e, st)) return rc;
    if (int rc = launch_attention<__half>(o, q, batch, tokens, heads, 3 * e, e, st)) return rc;
    const uint64_t n = (uint64_t)batch * tokens * e;
    f16_to_f32_kernel<<<(unsigned)std::min<uint64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(output, o, n);
    return check_launch("attention_out");
}

uint64_t dav2cuda_linear_half_workspace_size(uint32_t rows, uint32_t in_cols, uint32_t out_cols) {
    const uint32_t kp = round_up(in_cols, 8);
    return align256((uint64_t)rows * kp * 2) + align256((uint64_t)out_cols * kp * 2) + 256;
}

int dav2cuda_linear_half(float* output, const float* input, const float* weight, const float* bias, uint32_t rows,
                         uint32_t in_cols, uint32_t out_cols, uint32_t gelu, uint32_t precision, void* workspace,
                         uint64_t workspace_bytes, void* stream) {
    REQUIRE(rows && in_cols && out_cols && (precision == 1 || precision == 2), "invalid linear parameters");
    REQUIRE(!null_any(output, input, weight, workspace), "linear: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_linear_half_workspace_size(rows, in_cols, out_cols),
            "linear: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t kp = round_up(in_cols, 8);
    Carve ws(workspace, workspace_bytes);
    void* a = ws.take<uint8_t>((uint64_t)rows * kp * 2);
    void* b = ws.take<uint8_t>((uint64_t)out_cols * kp * 2);
    const bool bf = precision == 1;
    int rc = bf ? launch_pad_rows_half<__nv_bfloat16>((__nv_bfloat16*)a, input, rows, in_cols, kp, st)
                : launch_pad_rows_half<__half>((__half*)a, input, rows, in_cols, kp, st);
    if (rc) return rc;
    rc = bf ? launch_pad_rows_half<__nv_bfloat16>((__nv_bfloat16*)b, weight, out_cols, in_cols, kp, st)
            : launch_pad_rows_half<__half>((__half*)b, weight, out_cols, in_cols, kp, st);
    if (rc) return rc;
    GemmArgs g;
    g.elem = bf ? kElemBF16 : kElemF16;
    g.a = a;
    g.lda = kp;
    g.b = b;
    g.ldb = kp;
    g.m = rows;
    g.n = out_cols;
    g.k = kp;
    g.flags = (bias ? kEpiBias : 0u) | (gelu ? kEpiGelu : 0u);
    g.bias = bias;
    g.out = output;
    g.out_kind = kOutF32Rows;
    g.ldo = out_cols;
    return launch_gemm(g, st);
}

uint64_t dav2cuda_conv2d_half_workspace_size(uint32_t iw, uint32_t ih, uint32_t ic, uint32_t oc, uint32_t k,
                                             uint32_t s, uint32_t p) {
    if (!iw || !ih || !k || !s || iw + 2 * p < k || ih + 2 * p < k) return 0;
    const uint64_t ow = (iw + 2 * p - k) / s + 1, oh = (ih + 2 * p - k) / s + 1;
    const bool implicit = k == 3 && s == 1 && p == 1;
    const uint32_t cp = implicit ? round_up(ic, 64) : round_up(ic, 8);
    uint64_t bytes = align256((uint64_t)iw * ih * cp * 2) + align256((uint64_t)oc * k * k * cp * 2) + 256;
    if (!implicit && k != 1) bytes += align256(ow * oh * (uint64_t)k * k * cp * 2);
    if (k == 1 && (s != 1 || p != 0)) bytes += align256(ow * oh * (uint64_t)cp * 2);
    return bytes;
}

int dav2cuda_conv2d_half(float* output, const float* input, const float* weight, const float* bias, uint32_t iw,
                         uint32_t ih, uint32_t ic, uint32_t oc, uint32_t k, uint32_t s, uint32_t p, void* workspace,
                         uint64_t workspace_bytes, void* stream) {
    REQUIRE(iw && ih && ic && oc && k && s && iw + 2 * p >= k && ih + 2 * p >= k, "invalid convolution dimensions");
    REQUIRE(!null_any(output, input, weight, workspace), "convolution: null buffer");
    REQUIRE(workspace_bytes >= dav2cuda_conv2d_half_workspace_size(iw, ih, ic, oc, k, s, p),
            "convolution: workspace is too small");
    cudaStream_t st = as_stream(stream);
    const uint32_t ow = (iw + 2 * p - k) / s + 1, oh = (ih + 2 * p - k) / s + 1;
    const bool implicit = k == 3 && s == 1 && p == 1;
    const uint32_t cp = implicit ? round_up(ic, 64) : round_up(ic, 8);
    Carve ws(workspace, workspace_bytes);
    __half* x = ws.take<__half>((uint64_t)iw * ih * cp * 2);
    __half* wt = ws.take<__half>((uint64_t)oc * k * k * cp * 2);
    if (int rc = launch_nchw_to_nhwc<__half>(x, input, 1, ic, ih, iw, cp, st)) return rc;
    if (int rc = launch_conv_weight_to_half<__half>(wt, weight, oc, ic, k, cp, st)) return rc;
    GemmArgs g;
    g.elem = kElemF16;
    g.b = wt;
    g.ldb = (uint64_t)k * k * cp;
    g.n = oc;
    g.k = k * k * cp;
    g.m = ow * oh;
    g.flags = bias ? kEpiBias : 0u;
    g.bias = bias;
    g.out = output;
    g.out_kind = kOutF32Planar;
    g.col_stride = (uint64_t)ow * oh;
    if (implicit) {
        g.a_mode = kAModeConv3x3;
        g.a = x;
        g.conv_batch = 1;
        g.conv_h = ih;
        g.conv_w = iw;
        g.conv_c = cp;
    } else if (k == 1 && s == 1 && p == 0) {
        g.a = x;
        g.lda = cp;
    } else {
        __half* col = ws.take<__half>((uint64_t)ow * oh * k * k * cp * 2);
        if (int rc = launch_im2col_nhwc<__half>(col, x, 1, ih, iw, cp, k, s, p, oh, ow, k * k * cp, st)) return rc;
        g.a = col;
        g.lda = (uint64_t)k * k * cp;
    }
    return launch_gemm(g, st);
}

}  // extern "C"
