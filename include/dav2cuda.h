/*
 * dav2cuda: C ABI of the B200 (sm_100a) tensor-operator layer.
 *
 * Each entry point replaces one method of the reference runtime's operator
 * layer, class VulkanOperators (src/operators.h:11-305, implemented in
 * src/operators.cpp), keeping its argument meaning, its size validation and
 * its layouts: token matrices are row-major [rows, columns], feature maps are
 * planar [channels, height, width], int8 activations/weights are packed four
 * codes per uint32 (column 4k+j in byte j of word k) with one float scale per
 * row. Differences are stated per function (e.g. extra "batch" or "scale"
 * arguments, whose neutral values reproduce the reference call exactly).
 *
 * Conventions:
 *  - every pointer argument is a device pointer unless it is named host_*;
 *  - "stream" is a cudaStream_t passed as void* (NULL = legacy default
 *    stream); launches are asynchronous on it;
 *  - return values are dav2cuda_status codes; the functions never throw;
 *    dav2cuda_last_error() gives the message of the last failure on the
 *    calling thread. Size/shape problems return DAV2CUDA_INVALID_ARGUMENT
 *    before anything is launched (the reference throws
 *    std::invalid_argument from the same checks).
 */
#ifndef DAV2CUDA_H
#define DAV2CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DAV2CUDA_API __attribute__((visibility("default")))
#else
#define DAV2CUDA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dav2cuda_status {
    DAV2CUDA_OK = 0,
    DAV2CUDA_INVALID_ARGUMENT = 1,
    DAV2CUDA_OUT_OF_MEMORY = 5,
    DAV2CUDA_LAUNCH_FAILED = 6,
    DAV2CUDA_UNSUPPORTED = 8,
    DAV2CUDA_INTERNAL_ERROR = 9
} dav2cuda_status;

/* Library / device queries. */
DAV2CUDA_API const char* dav2cuda_last_error(void);
DAV2CUDA_API const char* dav2cuda_build_info(void);
/* Reads and clears the device error word that kernels set instead of
 * trapping (1 = a pipeline wait timed out). Synchronizes the device. */
DAV2CUDA_API int dav2cuda_device_error(void);
/* Number of kernels this library launched since the last reset. */
DAV2CUDA_API uint64_t dav2cuda_launch_count(int reset);
/* Failure-detection check of the bounded device waits (no counterpart in
 * the reference, whose Vulkan fences have host-side timeouts): one 32-thread
 * block waits on an mbarrier phase through the same bounded wait the
 * pipeline kernels use, with a limit of limit_ns (at most 1 s). With
 * arrive != 0 the phase completes at once; with arrive == 0 nothing
 * completes it, the wait gives up after limit_ns, sets the device error
 * word to 1 exactly as a timed-out pipeline wait does, and the kernel
 * returns. Asynchronous on the stream. */
DAV2CUDA_API int dav2cuda_wait_probe(uint64_t limit_ns, uint32_t arrive, void* stream);

/* --------------------------------------------------------------- row ops */

/* VulkanOperators::layer_norm (src/operators.h:99-106,
 * src/operators.cpp:1016-1042; shader src/shaders/layer_norm.glsl). */
DAV2CUDA_API int dav2cuda_layer_norm(float* output, const float* input, const float* weight,
                                     const float* bias, uint32_t rows, uint32_t columns,
                                     float epsilon, void* stream);

/* gelu.glsl dispatch inside VulkanOperators::linear* (src/operators.cpp:838-844,
 * src/shaders/gelu.glsl:16-49): exact-erf GELU, elementwise. */
DAV2CUDA_API int dav2cuda_gelu(float* output, const float* input, uint64_t count, void* stream);

/* softmax_lastdim.glsl as dispatched by VulkanOperators::attention_head64
 * (src/operators.cpp:1189-1198). Extra argument "scale" multiplies the
 * input before the softmax (1.0 reproduces the reference shader). */
DAV2CUDA_API int dav2cuda_softmax_rows(float* output, const float* input, uint64_t rows,
                                       uint32_t columns, float scale, void* stream);

/* VulkanOperators::add_scaled (src/operators.h:116-122,
 * src/operators.cpp:1072-1096): output = residual + addend * scale[col]. */
DAV2CUDA_API int dav2cuda_add_scaled(float* output, const float* residual, const float* addend,
                                     const float* scale, uint64_t count, uint32_t columns,
                                     void* stream);

/* VulkanOperators::relu / add / sigmoid_scale (src/operators.h:280-287). */
DAV2CUDA_API int dav2cuda_relu(float* output, const float* input, uint64_t count, void* stream);
DAV2CUDA_API int dav2cuda_add(float* output, const float* left, const float* right, uint64_t count,
                              void* stream);
DAV2CUDA_API int dav2cuda_sigmoid_scale(float* output, const float* input, uint64_t count,
                                        float scale, void* stream);

/* ------------------------------------------------------------- resampling */

/* VulkanOperators::bilinear_align_true (src/operators.h:254-261,
 * src/operators.cpp:1978-2012), planar [channels, H, W]. */
DAV2CUDA_API int dav2cuda_bilinear_align_true(float* output, const float* input,
                                              uint32_t input_width, uint32_t input_height,
                                              uint32_t output_width, uint32_t output_height,
                                              uint32_t channels, void* stream);

/* The DPT head's resizes in this executor's layout (src/dpt.cpp:598-605,
 * 813-820 run bilinear_align_true on planar maps): batch x [H][W][channels]
 * channels-last 16-bit maps (f16, or bf16 when bf16 != 0), channels a
 * multiple of 8 (8..2048), 16-byte aligned buffers; the reference's f32
 * arithmetic, the result rounded to the 16-bit type. */
DAV2CUDA_API int dav2cuda_bilinear_align_nhwc_16(void* output, const void* input, uint32_t batch,
                                                 uint32_t input_width, uint32_t input_height,
                                                 uint32_t output_width, uint32_t output_height,
                                                 uint32_t channels, uint32_t bf16, void* stream);

/* VulkanOperators::reduce_minmax (src/operators.cpp:2050-2058): writes
 * range[0]=min, range[1]=max over count floats. */
DAV2CUDA_API int dav2cuda_reduce_minmax(const float* input, float* range, uint64_t count,
                                        void* stream);
/* VulkanOperators::normalize_relative / normalize_metric
 * (src/operators.cpp:2060-2090), in place. */
DAV2CUDA_API int dav2cuda_normalize_relative(float* depth, const float* range, uint64_t count,
                                             void* stream);
DAV2CUDA_API int dav2cuda_normalize_metric(float* depth, const float* range, uint64_t count,
                                           float maximum_depth, void* stream);

/* GpuPreprocessor::run (src/gpu_preprocess.cpp:41-104, shader
 * src/shaders/preprocess_rgba.glsl:53-108): packed 8-bit pixels
 * (BGRA when rgba_order == 0) -> bicubic -> ImageNet-normalized planar RGB. */
DAV2CUDA_API int dav2cuda_preprocess_u32(float* output_chw, const uint32_t* pixels,
                                         uint32_t source_width, uint32_t source_height,
                                         uint32_t row_stride_pixels, uint32_t rgba_order,
                                         uint32_t destination_width,
                                         uint32_t destination_height, void* stream);

/* The CPU preprocess_bgr8 of dav2_infer_bgr8 (src/image.cpp:163-269) done
 * on the device for a batch of equally sized BGR8 images (interleaved,
 * row_stride_bytes apart, image_stride_bytes between images):
 * OpenCV-style bicubic (a=-0.75, half-pixel, clamp) then ImageNet
 * normalization, output planar [batch][3][dh][dw]. */
DAV2CUDA_API int dav2cuda_preprocess_bgr8(float* output_chw, const uint8_t* bgr, uint32_t batch,
                                          uint32_t source_width, uint32_t source_height,
                                          uint64_t row_stride_bytes, uint64_t image_stride_bytes,
                                          uint32_t destination_width,
                                          uint32_t destination_height, void* stream);

/* Square frame resize of the high-resolution configuration: BGR8 ->
 * bilinear (align_corners=False) -> normalized planar RGB, batched. */
DAV2CUDA_API int dav2cuda_preprocess_bgr8_bilinear(float* output_chw, const uint8_t* bgr,
                                                   uint32_t batch, uint32_t source_width,
                                                   uint32_t source_height,
                                                   uint64_t row_stride_bytes,
                                                   uint64_t image_stride_bytes,
                                                   uint32_t destination_width,
                                                   uint32_t destination_height, void* stream);

/* ------------------------------------------------------------------- int8 */

/* quantize_rows_int8_fused.glsl dispatch (src/operators.cpp:812-821): per-row
 * symmetric int8 codes of input[input_offset + row*columns + c].
 * columns % 4 == 0; packed is [rows, columns/4] uint32. */
DAV2CUDA_API int dav2cuda_quantize_rows_s8(uint32_t* packed, float* scales, const float* input,
                                           uint32_t rows, uint32_t columns,
                                           uint64_t input_offset, void* stream);

/* The executor's on-device int8 weight packing (GpuModel's per-output-row
 * symmetric quantization, src/gpu_model.cpp:207-284: scale = max(absmax/127,
 * 1e-8), code = nearbyint(clamp(w/scale))): codes [rows][padded_columns]
 * (int8, zero beyond `columns`) + f32 scales [rows]. layout 0: weight is
 * [rows][columns]; 1: a conv-transpose [Ci][Co][k][k] packed as rows
 * (ky*k+kx)*Co+co over Ci (rows = k*k*Co, columns = Ci); 2: a convolution
 * [Co][Ci][k][k] with columns in (ky, kx, ci) order (rows = Co, columns =
 * k*k*Ci). output_channels / kernel / input_channels describe layouts 1, 2. */
DAV2CUDA_API int dav2cuda_pack_weight_s8(uint8_t* codes, float* scales, const float* weight, uint32_t layout,
                                         uint32_t rows, uint32_t columns, uint32_t padded_columns,
                                         uint32_t output_channels, uint32_t kernel, uint32_t input_channels,
                                         void* stream);

/* The same im2col-quantize (im2col_quantize_int8.glsl, src/operators.cpp:
 * 1787-1801) on a channels-last f32 map [batch][H][W][C], as the executor
 * runs it for the resize-3 convolution and the conv-transpose inputs: one
 * row of row_bytes bytes per output pixel, columns in (ky, kx, c) order —
 * the reference's (c, ky, kx) order permuted, with the weight columns
 * permuted alike, which leaves every row scale and code unchanged — and zero
 * bytes past kernel*kernel*C. Row scale = max(absmax/127, 1e-8). */
DAV2CUDA_API int dav2cuda_im2col_quantize_nhwc(uint8_t* codes, float* scales, const float* input, uint32_t batch,
                                               uint32_t height, uint32_t width, uint32_t channels,
                                               uint32_t kernel, uint32_t stride, uint32_t padding,
                                               uint32_t row_bytes, void* stream);

/* im2col_quantize_int8.glsl dispatch (src/operators.cpp:1787-1801) on a
 * planar [C,H,W] input: rows = output pixels, padded to ceil(C*k*k/4) words
 * (the reference layout). */
DAV2CUDA_API int dav2cuda_im2col_quantize_s8(uint32_t* packed, float* scales, const float* input,
                                             uint32_t input_width, uint32_t input_height,
                                             uint32_t input_channels, uint32_t output_width,
                                             uint32_t output_height, uint32_t kernel,
                                             uint32_t stride, int32_t padding, void* stream);

/* VulkanOperators::linear_int8_packed (src/operators.cpp:847-880, shader
 * linear_int8_tiled.glsl): s8 x s8 -> s32 on tcgen05 tensor cores, then
 * float(acc)*input_scales[row]*weight_scales[col] (+bias[col]).
 * input_columns % 16 == 0 (the tensor-core operand rows are 16-byte
 * aligned). Transposed stores write output[col*row_stride + row_offset + row]. */
DAV2CUDA_API int dav2cuda_linear_s8_packed(float* output, const uint32_t* packed_input,
                                           const uint32_t* packed_weight,
                                           const float* input_scales, const float* weight_scales,
                                           const float* bias, uint32_t rows,
                                           uint32_t input_columns, uint32_t output_columns,
                                           uint32_t output_row_offset, uint32_t output_row_stride,
                                           uint32_t output_transposed, uint32_t has_bias,
                                           void* stream);

/* Workspace bytes that dav2cuda_linear_int8 / dav2cuda_conv2d_int8 need
 * (the reference keeps the same buffers in its Int8ActivationWorkspace). */
DAV2CUDA_API uint64_t dav2cuda_linear_int8_workspace_size(uint32_t rows, uint32_t input_columns,
                                                          uint32_t output_columns);
DAV2CUDA_API uint64_t dav2cuda_conv2d_int8_workspace_size(uint32_t input_width, uint32_t input_height,
                                                          uint32_t input_channels,
                                                          uint32_t output_channels, uint32_t kernel,
                                                          uint32_t stride, uint32_t padding);
DAV2CUDA_API uint64_t dav2cuda_conv_transpose_int8_workspace_size(uint32_t input_width,
                                                                  uint32_t input_height,
                                                                  uint32_t input_channels,
                                                                  uint32_t output_channels,
                                                                  uint32_t kernel);

/* VulkanOperators::linear_int8 (src/operators.h:84-94,
 * src/operators.cpp:770-845): quantize rows -> s8 GEMM -> dequant + bias
 * (-> GELU when gelu != 0). */
DAV2CUDA_API int dav2cuda_linear_int8(float* output, const float* input, const uint32_t* int8_weight,
                                      const float* weight_scales, const float* bias, uint32_t rows,
                                      uint32_t input_columns, uint32_t output_columns, uint32_t gelu,
                                      void* workspace, uint64_t workspace_bytes, void* stream);

/* The encoder block's int8 residual update, src/encoder.cpp:478-489 (proj,
 * ls1) and 561-572 (fc2, ls2): VulkanOperators::linear_int8
 * (src/operators.cpp:770-845, reached through DinoEncoder::linear at
 * src/encoder.cpp:292 in int8 mode) into a temporary, then add_scaled
 * (src/operators.cpp:1072-1096) into the residual stream, done here as one
 * GEMM whose epilogue updates the stream in place:
 *   residual[r][c] = residual[r][c] + ((acc * s_in[r]) * s_w[c] + bias[c]) * layer_scale[c]
 * with the reference's separate roundings. Workspace: the size
 * dav2cuda_linear_int8_workspace_size() returns for the same shape. */
DAV2CUDA_API int dav2cuda_linear_int8_residual(float* residual, const float* input, const uint32_t* int8_weight,
                                               const float* weight_scales, const float* bias,
                                               const float* layer_scale, uint32_t rows, uint32_t input_columns,
                                               uint32_t output_columns, void* workspace, uint64_t workspace_bytes,
                                               void* stream);

/* dav2cuda_linear_int8 for callers that may not allocate device memory —
 * host applications that own the device heap (video pipelines, game
 * engines, inference servers that reserve memory at start-up and treat a
 * later cudaMalloc as a failure) or run on real-time paths where an
 * allocation is not allowed. No counterpart in the reference (its operators
 * own a reusable workspace). Scratch: one 16 MiB device array per GPU that
 * loads the library (dav2cuda_linear_int8_noalloc_scratch_limit()), held
 * until exit; larger problems return DAV2CUDA_INVALID_ARGUMENT. The first
 * call on a device resolves the array's address (make it before any stream
 * capture); the address is kept for the life of the process, so no call may
 * follow a cudaDeviceReset. All calls share the array: calls that overlap on
 * the GPU race. Allocates nothing. */
DAV2CUDA_API uint64_t dav2cuda_linear_int8_noalloc_scratch_limit(void);
DAV2CUDA_API int dav2cuda_linear_int8_noalloc(float* output, const float* input,
                                              const uint32_t* int8_weight, const float* weight_scales,
                                              const float* bias, uint32_t rows, uint32_t input_columns,
                                              uint32_t output_columns, uint32_t gelu, void* stream);

/* VulkanOperators::conv2d_int8 (src/operators.h:183-196,
 * src/operators.cpp:1735-1805): im2col-quantize -> s8 GEMM -> planar
 * dequantized output [Co, OH, OW]. */
DAV2CUDA_API int dav2cuda_conv2d_int8(float* output, const float* input, const uint32_t* int8_weight,
                                      const float* weight_scales, const float* bias,
                                      uint32_t input_width, uint32_t input_height,
                                      uint32_t input_channels, uint32_t output_channels,
                                      uint32_t kernel, uint32_t stride, uint32_t padding,
                                      uint32_t has_bias, void* workspace, uint64_t workspace_bytes,
                                      void* stream);

/* VulkanOperators::conv_transpose_nonoverlap_int8 (src/operators.h:231-241,
 * src/operators.cpp:1908-1976): per-pixel channel quantize -> s8 GEMM
 * against weight rows (ky*k+kx)*Cout+co -> scatter to planar
 * [Cout, H*k, W*k]. */
DAV2CUDA_API int dav2cuda_conv_transpose_int8(float* output, const float* input,
                                              const uint32_t* int8_weight,
                                              const float* weight_scales, const float* bias,
                                              uint32_t input_width, uint32_t input_height,
                                              uint32_t input_channels, uint32_t output_channels,
                                              uint32_t kernel, void* workspace,
                                              uint64_t workspace_bytes, void* stream);

/* BASELINE configuration 2(d) as one call: conv2d_int8 (3x3, pad 1) over a
 * batch of planar images followed by the 2x align-corners bilinear upsample,
 * output [batch, Co, 2H, 2W]. */
DAV2CUDA_API uint64_t dav2cuda_conv3x3_int8_up2_workspace_size(uint32_t batch, uint32_t width,
                                                               uint32_t height,
                                                               uint32_t input_channels,
                                                               uint32_t output_channels);
DAV2CUDA_API int dav2cuda_conv3x3_int8_up2(float* output, const float* input,
                                           const uint32_t* int8_weight, const float* weight_scales,
                                           const float* bias, uint32_t batch, uint32_t width,
                                           uint32_t height, uint32_t input_channels,
                                           uint32_t output_channels, void* workspace,
                                           uint64_t workspace_bytes, void* stream);

/* VulkanOperators::conv2d (src/operators.cpp:1528-1675) for the DPT head's
 * output_conv1 shape, as the executor runs it: 3x3, pad 1, + bias, from a
 * channels-last 16-bit map [batch][H][W][input_channels] (f16, or bf16 when
 * bf16 != 0; input_channels a multiple of 64) to [batch][H][W][128] 16-bit;
 * weight [128][9 * input_channels] 16-bit with column (ky*3 + kx)*C + c, bias
 * 128 floats; 16-byte aligned buffers. */
DAV2CUDA_API int dav2cuda_conv3x3_c128_16(void* output, const void* input, const void* weight,
                                          const float* bias, uint32_t batch, uint32_t width,
                                          uint32_t height, uint32_t input_channels, uint32_t bf16,
                                          void* stream);

/* The DPT output head's last layers (src/dpt.cpp:830-854): output_conv2.0
 * (3x3, pad 1, channels -> 32, + bias), ReLU, output_conv2.2 (1x1, 32 -> 1,
 * + head_bias), then ReLU (max_depth <= 0: relative depth) or
 * sigmoid * max_depth (metric), as the executor runs them: channels-last
 * 16-bit input [batch][H][W][channels] (f16, or bf16 when bf16 != 0),
 * channels 64 or 128, weight [32][9 * channels] 16-bit with column
 * (ky*3 + kx)*channels + c, bias and head_weight 32 floats, output depth
 * [batch][H][W]; 16-byte aligned buffers. */
DAV2CUDA_API int dav2cuda_conv3x3_head_16(float* depth, const void* input, const void* weight,
                                          const float* bias, const float* head_weight,
                                          float head_bias, float max_depth, uint32_t batch,
                                          uint32_t width, uint32_t height, uint32_t channels,
                                          uint32_t bf16, void* stream);

/* ------------------------------------------------------------ token ops */

/* VulkanOperators::prepare_tokens (src/operators.h:127-141,
 * src/operators.cpp:1211-1406): planar image [3][h][w] (w, h multiples of
 * 14) -> tokens [1 + (w/14)(h/14)][embedding]: the patch embedding (a 14x14
 * stride-14 convolution, weight [embedding][3][14][14], + bias), the class
 * token at row 0, and the 37x37 positional grid of `position` ([1370]
 * [embedding]) resized bicubically to the patch grid (exact copy at 37x37,
 * src/shaders/position_bicubic.glsl) and added. _half: weight f32, computed
 * with bf16 (precision 1) or f16 (precision 2) operands and f32
 * accumulation; _int8: the reference's int8 route — per-patch im2col
 * quantization and packed int8 weight codes [embedding][147] with scales. */
DAV2CUDA_API uint64_t dav2cuda_prepare_tokens_workspace_size(uint32_t input_width, uint32_t input_height,
                                                             uint32_t embedding);
DAV2CUDA_API int dav2cuda_prepare_tokens_half(float* output, const float* image, const float* patch_weight,
                                              const float* patch_bias, const float* class_token,
                                              const float* position, uint32_t input_width,
                                              uint32_t input_height, uint32_t embedding, uint32_t precision,
                                              void* workspace, uint64_t workspace_bytes, void* stream);
DAV2CUDA_API int dav2cuda_prepare_tokens_int8(float* output, const float* image,
                                              const uint32_t* patch_int8_weight,
                                              const float* patch_weight_scales, const float* patch_bias,
                                              const float* class_token, const float* position,
                                              uint32_t input_width, uint32_t input_height, uint32_t embedding,
                                              void* workspace, uint64_t workspace_bytes, void* stream);

/* VulkanOperators::project_tokens / _fp16 / _int8 (src/operators.h:143-171,
 * src/operators.cpp:1408-1526): tokens [1 + width*height][embedding] (row 0,
 * the class token, is skipped) -> planar [output_channels][height*width]
 * through a 1x1 convolution (weight [output_channels][embedding], bias
 * nullable). _half: bf16 (precision 1) or f16 (precision 2) operands; _int8:
 * per-row int8 tokens x packed int8 weight codes [output_channels]
 * [embedding/4] with scales. */
DAV2CUDA_API uint64_t dav2cuda_project_tokens_workspace_size(uint32_t width, uint32_t height, uint32_t embedding,
                                                             uint32_t output_channels);
DAV2CUDA_API int dav2cuda_project_tokens_half(float* output, const float* tokens, const float* weight,
                                              const float* bias, uint32_t width, uint32_t height,
                                              uint32_t embedding, uint32_t output_channels, uint32_t precision,
                                              void* workspace, uint64_t workspace_bytes, void* stream);
DAV2CUDA_API int dav2cuda_project_tokens_int8(float* output, const float* tokens, const uint32_t* int8_weight,
                                              const float* weight_scales, const float* bias, uint32_t width,
                                              uint32_t height, uint32_t embedding, uint32_t output_channels,
                                              void* workspace, uint64_t workspace_bytes, void* stream);

/* VulkanOperators::conv_transpose_nonoverlap / _fp16 (src/operators.h:
 * 214-230, src/operators.cpp:1807-1906): transposed convolution with kernel
 * == stride k, weight [Ci][Co][k][k], bias [Co]: planar [Ci][H][W] ->
 * [Co][H*k][W*k], with bf16 (precision 1) or f16 (precision 2) operands and
 * f32 accumulation. */
DAV2CUDA_API uint64_t dav2cuda_conv_transpose_half_workspace_size(uint32_t input_width, uint32_t input_height,
                                                                  uint32_t input_channels,
                                                                  uint32_t output_channels, uint32_t kernel);
DAV2CUDA_API int dav2cuda_conv_transpose_half(float* output, const float* input, const float* weight,
                                              const float* bias, uint32_t input_width, uint32_t input_height,
                                              uint32_t input_channels, uint32_t output_channels, uint32_t kernel,
                                              uint32_t precision, void* workspace, uint64_t workspace_bytes,
                                              void* stream);

/* ------------------------------------------------------------- attention */

/* VulkanOperators::attention_head64 (src/operators.h:124-131,
 * src/operators.cpp:1098-1209): qkv [tokens, 3*heads*64] (q|k|v, head-major
 * inside each), softmax(q*0.125 . k) . v -> [tokens, heads*64]. Computed
 * as fused (flash) attention with f16 operands and f32 accumulation — the
 * reference's fp16 attention precision — never materializing scores.
 * "batch" stacks independent token matrices (1 reproduces the reference). */
DAV2CUDA_API int dav2cuda_attention_head64(float* output, const float* qkv, uint32_t batch,
                                           uint32_t tokens, uint32_t heads, void* workspace,
                                           uint64_t workspace_bytes, void* stream);
DAV2CUDA_API uint64_t dav2cuda_attention_head64_workspace_size(uint32_t batch, uint32_t tokens,
                                                               uint32_t heads);

/* ------------------------------------------------------------ fp32 family */

/* VulkanOperators::linear (src/operators.h:15-27): Y = X W^T + b with fp32
 * in/out, computed on tcgen05 with bf16 operands and fp32 accumulation
 * (precision = 1) or f16 operands (precision = 2). Optional GELU. */
DAV2CUDA_API uint64_t dav2cuda_linear_half_workspace_size(uint32_t rows, uint32_t input_columns,
                                                          uint32_t output_columns);
DAV2CUDA_API int dav2cuda_linear_half(float* output, const float* input, const float* weight,
                                      const float* bias, uint32_t rows, uint32_t input_columns,
                                      uint32_t output_columns, uint32_t gelu, uint32_t precision,
                                      void* workspace, uint64_t workspace_bytes, void* stream);

/* VulkanOperators::conv2d (src/operators.h:147-163) for planar f32 input,
 * weights [Co,Ci,k,k] (bias may be NULL), computed as an implicit GEMM on
 * tcgen05 with f16 operands and fp32 accumulation. stride 1 uses shifted
 * tensor-memory-access tiles over a channels-last copy of the input;
 * other shapes use an explicit channels-last im2col. */
DAV2CUDA_API uint64_t dav2cuda_conv2d_half_workspace_size(uint32_t input_width, uint32_t input_height,
                                                          uint32_t input_channels,
                                                          uint32_t output_channels, uint32_t kernel,
                                                          uint32_t stride, uint32_t padding);
DAV2CUDA_API int dav2cuda_conv2d_half(float* output, const float* input, const float* weight,
                                      const float* bias, uint32_t input_width,
                                      uint32_t input_height, uint32_t input_channels,
                                      uint32_t output_channels, uint32_t kernel, uint32_t stride,
                                      uint32_t padding, void* workspace, uint64_t workspace_bytes,
                                      void* stream);

#ifdef __cplusplus
}
#endif

#endif
