// Host-side declarations of the kernel launchers (no device code), shared
// by the C ABI and the executor runtime.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "dav2cuda.h"

namespace dav2cuda {

int set_error(int status, const char* message);
int check_launch(const char* what);
int* device_error_word();
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Per-device one-time kernel set-up (cudaFuncSetAttribute): one bit per
// device ordinal, set atomically once the attributes are applied. Threads
// driving different devices (or the same one) may both apply them, which is
// idempotent; none can skip them.
inline bool configured_on(const std::atomic<uint64_t>& mask, int dev) {
    return (mask.load(std::memory_order_acquire) >> (dev & 63)) & 1ull;
}
inline void mark_configured(std::atomic<uint64_t>& mask, int dev) {
    mask.fetch_or(1ull << (dev & 63), std::memory_order_release);
}
// Multiprocessor count of a device (cached per ordinal; 0 when the query fails).
int sm_count(int dev);


// ------------------------------------------------------------ memory-bound
enum LnOutKind { kLnOutF32 = 0, kLnOutF16 = 1, kLnOutBF16 = 2, kLnOutS8 = 3 };
int launch_layer_norm(void* out, float* out_scales, const float* in, const float* w, const float* b,
                      uint32_t rows, uint32_t cols, float eps, int out_kind, uint32_t out_group,
                      uint32_t in_group, uint32_t in_offset, cudaStream_t st);
int launch_gelu(float* out, const float* in, uint64_t n, cudaStream_t st);
int launch_softmax(float* out, const float* in, uint64_t rows, uint32_t cols, float scale, cudaStream_t st);
int launch_add_scaled(float* out, const float* res, const float* add, const float* scale, uint64_t n,
                      uint32_t cols, cudaStream_t st);
int launch_relu(float* out, const float* in, uint64_t n, cudaStream_t st);
int launch_add(float* out, const float* a, const float* b, uint64_t n, cudaStream_t st);
int launch_sigmoid_scale(float* out, const float* in, uint64_t n, float s, cudaStream_t st);
template <typename TI, typename TO>
int launch_bilinear_align(TO* out, const TI* in, uint32_t iw, uint32_t ih, uint32_t ow, uint32_t oh,
                          uint32_t planes, cudaStream_t st);
// Align-corners bilinear of channels-last f32 maps [B][ih][iw][C] (C % 32 == 0)
// into planar f32 [B][C][oh][ow]; _supported() says whether two source rows of
// iw pixels and the ow-column coordinate table fit the kernel's shared memory.
bool bilinear_nhwc_to_planar_supported(uint32_t iw, uint32_t c, uint32_t ow);
int launch_bilinear_nhwc_to_planar(float* out, const float* in, uint32_t batch, uint32_t ih, uint32_t iw, uint32_t c,
                                   uint32_t oh, uint32_t ow, cudaStream_t st);
// The DPT head's output_conv2 (3x3, cp -> 32, + bias, ReLU) and 1x1 32 -> 1
// head (+ head_b, ReLU or sigmoid * head_max) as one halo-loading tcgen05
// kernel over channels-last 16-bit maps [batch][h][w][cp] -> f32 [batch][h][w]
// (destination read from out_slot when set); weight [32][9 * cp] 16-bit,
// column (ky*3 + kx)*cp + c.
// 3x3 convolution (pad 1) + bias to 128 channels on channels-last 16-bit maps
// [batch][h][w][cin] -> [batch][h][w][128] (cin a multiple of 64), as one
// halo-loading tcgen05 kernel; weight [128][9 * cin], column (ky*3 + kx)*cin + c.
bool conv3x3_halo_supported(uint32_t cin, uint32_t cout, uint32_t ldo);
int launch_conv3x3_halo(void* out, const void* in, const void* weight, const float* bias, bool bf16, uint32_t batch,
                        uint32_t h, uint32_t w, uint32_t cin, cudaStream_t st);
bool conv_head_halo_supported(uint32_t cp, uint32_t cout);
int launch_conv_head_halo(float* out, float* const* out_slot, const void* in, const void* weight, const float* bias,
                          const float* head_w, float head_b, float head_max, bool metric, bool bf16, uint32_t batch,
                          uint32_t h, uint32_t w, uint32_t cp, cudaStream_t st);
int launch_minmax(const float* in, float* range, uint64_t n, cudaStream_t st);
int launch_normalize(float* d, const float* range, uint64_t n, float maximum, cudaStream_t st);
// Per-image forms over `batch` images of n values each: ranges [batch][2].
int launch_minmax_batched(const float* in, float* ranges, uint64_t n, uint32_t batch, cudaStream_t st);
int launch_normalize_batched(float* d, const float* ranges, uint64_t n, uint32_t batch, float maximum,
                             cudaStream_t st);
int launch_preprocess_u32(float* out, const uint32_t* px, uint32_t sw, uint32_t sh, uint32_t stride,
                          uint32_t rgba, uint32_t dw, uint32_t dh, cudaStream_t st);
// `batch` packed-pixel images img_stride pixels apart -> planar [batch][3][dh][dw].
int launch_preprocess_u32_batched(float* out, const uint32_t* px, uint32_t batch, uint32_t sw, uint32_t sh,
                                  uint32_t stride, uint64_t img_stride, uint32_t rgba, uint32_t dw, uint32_t dh,
                                  cudaStream_t st);
int launch_preprocess_bgr8(float* out, const uint8_t* bgr, uint32_t batch, uint32_t sw, uint32_t sh,
                           uint64_t row_stride, uint64_t img_stride, uint32_t dw, uint32_t dh, int bilinear,
                           cudaStream_t st);
template <typename T>
int launch_quantize_rows(uint32_t* packed, float* scales, const T* in, uint64_t rows, uint32_t cols,
                         uint64_t offset, uint32_t group, uint64_t group_stride, uint32_t row_stride,
                         uint32_t out_words, cudaStream_t st);
// 3x3 / stride 1 / pad 1 im2col-quantize of planar f32 maps [B][C][H][W]:
// codes [B*H*W][kp] in (ky, kx, c) column order (the reference's (c, ky, kx)
// order permuted; rows and scales unchanged), exact row scales from a
// per-pixel channel abs-max pre-pass (pix_absmax: [B*H*W] floats of scratch).
int launch_im2col_quantize_3x3_planar(uint8_t* codes, float* scales, float* pix_absmax, const float* in,
                                      uint32_t batch, uint32_t c, uint32_t h, uint32_t w, uint32_t kp,
                                      cudaStream_t st);
int launch_im2col_quantize(uint32_t* packed, float* scales, const float* in, uint32_t batch, uint32_t iw,
                           uint32_t ih, uint32_t ic, uint32_t ow, uint32_t oh, uint32_t k, uint32_t s, int pad,
                           uint32_t out_words, cudaStream_t st);

// --------------------------------------------------------- layout helpers
// planar f32 [B][C][H][W] -> channels-last [B][H][W][Cp] half or f32
// (channels beyond C are zero).
template <typename H>
int launch_nchw_to_nhwc(H* out, const float* in, uint32_t batch, uint32_t c, uint32_t h, uint32_t w,
                        uint32_t cp, cudaStream_t st);
// int8 convolution weight codes [Co][Ci*k*k] ((ci, ky, kx) columns, rows k_in
// bytes apart) -> (ky, kx, ci) columns, rows padded to kp bytes.
int launch_conv_codes_tap_major(uint8_t* out, const uint8_t* in, uint32_t co, uint32_t ci, uint32_t kk, uint32_t k_in,
                                uint32_t kp, cudaStream_t st);
// f32 -> half (elementwise, any count).
template <typename H>
int launch_to_half(H* out, const float* in, uint64_t n, cudaStream_t st);
// f32 matrix [rows, cols] -> half [rows, cols_p] with zero padding.
template <typename H>
int launch_pad_rows_half(H* out, const float* in, uint64_t rows, uint32_t cols, uint32_t cols_p,
                         cudaStream_t st);
// Explicit im2col of a channels-last half map (any stride/padding); column
// order (ky, kx, c) and rows padded to kp columns.
template <typename H>
int launch_im2col_nhwc(H* out, const H* in, uint32_t batch, uint32_t h, uint32_t w, uint32_t c, uint32_t k,
                       uint32_t s, uint32_t pad, uint32_t oh, uint32_t ow, uint32_t kp, cudaStream_t st);
// Weight reorders: [Co][Ci][k][k] f32 -> [Co][k][k][Cip] half.
template <typename H>
int launch_conv_weight_to_half(H* out, const float* w, uint32_t co, uint32_t ci, uint32_t k, uint32_t cip,
                               cudaStream_t st);

// ------------------------------------------------------------ graph pieces
// Stream-ordered store of one device pointer into a device-side slot (the
// graph's final convolution reads its destination from such a slot, so a
// captured graph can write straight into each call's output buffer).
int launch_store_pointer(void** slot, void* value, cudaStream_t st);
template <typename H>
int launch_patch_im2col(H* out, const float* img, uint32_t batch, uint32_t h, uint32_t w, uint32_t kp,
                        cudaStream_t st);
int launch_position_bicubic(float* out, const float* pos, uint32_t d, uint32_t pw, uint32_t ph, cudaStream_t st);
int launch_fill_tokens(float* x, const float* cls, const float* pos, const float* interp, uint32_t d,
                       uint32_t tokens, uint32_t batch, cudaStream_t st);
template <typename H>
int launch_bilinear_nhwc(H* out, const H* in, uint32_t batch, uint32_t ih, uint32_t iw, uint32_t oh, uint32_t ow,
                         uint32_t c, cudaStream_t st);
template <typename H>
int launch_im2col_quantize_nhwc(uint8_t* out, float* scales, const H* in, uint32_t batch, uint32_t h, uint32_t w,
                                uint32_t c, uint32_t ldc, uint32_t k, uint32_t s, uint32_t pad, uint32_t oh,
                                uint32_t ow, uint32_t kp, cudaStream_t st);
// Weight layouts: 0 = [rows][K] as stored; 1 = conv-transpose [Ci][Co][k][k]
// read as rows (ky*k+kx)*Co+co over Ci; 2 = conv [Co][Ci][k][k] read with
// columns in (ky, kx, ci) order (half: channels padded to cip).
int launch_pack_weight_s8(uint8_t* out, float* scales, const float* w, int kind, uint64_t rows, uint32_t K,
                          uint32_t kp, uint32_t co, uint32_t k, uint32_t ci, cudaStream_t st);
template <typename H>
int launch_half_weight(H* out, const float* w, int kind, uint64_t rows, uint32_t K, uint32_t kp, uint32_t co,
                       uint32_t k, uint32_t ci, uint32_t cip, cudaStream_t st);
int launch_expand_bias(float* out, const float* bias, uint32_t co, uint32_t reps, cudaStream_t st);

// ------------------------------------------------------------- attention
// tcgen05 flash attention over interleaved qkv [B*T][3*heads*64] of f16 (or
// bf16 when bf16) values; out [B*T][out_ld] of the same type, or f32 when
// out_f32.
int launch_attention_tc(void* out, bool out_f32, const void* qkv, bool bf16, uint32_t batch, uint32_t tokens,
                        uint32_t heads, uint64_t qkv_ld, uint64_t out_ld, cudaStream_t st);
template <typename H>
int launch_attention(H* out, const H* qkv, uint32_t batch, uint32_t tokens, uint32_t heads, uint64_t qkv_ld,
                     uint64_t out_ld, cudaStream_t st);

// ------------------------------------------------------------------ GEMM
enum GemmElem { kElemS8 = 0, kElemF16 = 1, kElemBF16 = 2 };
enum GemmAMode { kAModeRows = 0, kAModeConv3x3 = 1 };
enum EpiFlags : uint32_t {
    kEpiBias = 1u << 0,
    kEpiDequant = 1u << 1,      // int8: acc * s_in[row] * s_w[col]
    kEpiGelu = 1u << 2,
    kEpiLayerScale = 1u << 3,   // res + v * gamma[col] (f32 residual, rounded separately)
    kEpiResidual1 = 1u << 4,    // v + res1
    kEpiResidual2 = 1u << 5,    // res2 + (...)
    kEpiRelu = 1u << 6,
    kEpiReluCopy = 1u << 7,     // also store relu(v) to out2
    kEpiHeadDot = 1u << 8,      // relu(v) . w2 + b2 -> one value per row (output head)
    kEpiMetricHead = 1u << 9,   // head output: sigmoid * max_depth instead of relu
};
enum OutKind {
    kOutF32Rows = 0,    // row-major, ldo elements per row
    kOutHalfRows = 1,   // row-major half (f16 / bf16 per out_half_bf16)
    kOutF32Planar = 2,  // per image planar: [img][col][plane]
    kOutConvTF32 = 3,   // conv-transpose scatter into planar f32 [img][co][H*k][W*k]
    kOutConvTHalf = 4,  // conv-transpose scatter into channels-last half [img][H*k][W*k][ldo]
    kOutHeadF32 = 5,    // kEpiHeadDot result, one f32 per row at out[row_remap]
};

struct GemmArgs {
    int elem = kElemBF16;
    int a_mode = kAModeRows;
    // operands
    const void* a = nullptr;        // rows mode: [M][lda] ; conv mode: NHWC [img][H][W][C]
    uint64_t lda = 0;               // elements per A row (rows mode)
    const void* b = nullptr;        // [N][ldb] (K-major weights)
    uint64_t ldb = 0;
    uint32_t m = 0, n = 0, k = 0;   // GEMM extents (k = reduction length in elements)
    // conv mode geometry (3x3, stride 1, pad 1, channels-last input)
    uint32_t conv_batch = 0, conv_h = 0, conv_w = 0, conv_c = 0;
    // epilogue
    uint32_t flags = 0;
    int out_kind = kOutF32Rows;
    bool out_half_bf16 = false;     // half outputs: bf16 (true) or f16 (false)
    void* out = nullptr;
    void* out2 = nullptr;           // relu copy (same layout as out)
    uint64_t ldo = 0;
    const float* bias = nullptr;
    const float* s_in = nullptr;
    const float* s_w = nullptr;
    const float* gamma = nullptr;
    const void* res1 = nullptr;     // residual tensors: same layout and type as out
    const void* res2 = nullptr;
    const float* head_w = nullptr;  // kEpiHeadDot
    float* const* out_slot = nullptr;  // kOutHeadF32: destination read from this device slot when set
    float head_b = 0.f;
    float head_max_depth = 0.f;
    // row remap: out_row = (r / rows_per_img) * out_rows_per_img + row_offset + r % rows_per_img
    uint32_t rows_per_img = 0;      // 0 = no remap (identity)
    uint32_t out_rows_per_img = 0;
    uint32_t row_offset = 0;
    // planar outputs: image stride and channel stride in elements
    uint64_t img_stride = 0, col_stride = 0;
    // conv-transpose scatter
    uint32_t convt_k = 0, convt_cout = 0, convt_w = 0, convt_h = 0;
    int block_n = 0;                // 0 = choose
    int max_ctas = 0;               // 0 = all SMs
};

int launch_gemm(const GemmArgs& args, cudaStream_t st);

}  // namespace dav2cuda
