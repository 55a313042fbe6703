/*
 * CPU oracle for the Depth Anything V2 tensor-operator hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This library restates, in plain C, the arithmetic
 * of the reference runtime's Vulkan compute shaders and CPU helpers so that the
 * CUDA kernels can be checked against it. Nothing in the product links it: only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * load it, and only as the checker or as the timed CPU baseline.
 *
 * Every function cites the reference file:line whose algorithm it restates
 * (paths relative to the reference project root). Layouts follow the
 * reference: token matrices are row-major [rows, columns]; feature maps are
 * planar [channels, height, width]; int8 codes are packed four per uint32,
 * least-significant byte first (column 4k+j in byte j of word k).
 *
 * Build: gcc -O2 -ffp-contract=off -fopenmp (no FMA contraction, so the
 * shader operation order is kept literally).
 */
#ifndef DAV2_ORACLE_H
#define DAV2_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* src/gpu_model.cpp:100-125 (tests/vulkan_smoke.cpp:68-69 pins "123456789"). */
uint32_t dav2o_crc32(const void* data, size_t bytes);

/* src/image.cpp:138-161. Returns 0, or -1 for non-positive arguments. */
int dav2o_network_shape(int width, int height, int input_size,
                        int* out_width, int* out_height);

/* src/image.cpp:163-269: BGR8 -> RGB/255 -> OpenCV-style bicubic (float
 * coefficients, double accumulation) -> (v-mean)/std -> planar f32 [3,dh,dw]. */
int dav2o_preprocess_bgr8(const uint8_t* bgr, int width, int height,
                          ptrdiff_t stride, int dst_width, int dst_height,
                          float* rgb_chw);

/* src/image.cpp:289-337: InferBridge BGRA nearest resize, channels kept in
 * byte order (B,G,R), float arithmetic. */
int dav2o_preprocess_inferbridge_bgra8(const uint8_t* bgra, int width,
                                       int height, ptrdiff_t stride,
                                       int dst_width, int dst_height,
                                       float* chw);

/* src/shaders/preprocess_rgba.glsl:53-108: packed u32 pixels -> bicubic in
 * f32 (a=-0.75, half-pixel, clamp) -> normalized planar f32. rgba_order=0
 * means BGRA (blue in the low byte). */
void dav2o_preprocess_u32_bicubic(const uint32_t* pixels, int src_width,
                                  int src_height, int row_stride_pixels,
                                  int rgba_order, int dst_width,
                                  int dst_height, float* rgb_chw);

/* Square bilinear (align_corners=False, PyTorch F.interpolate rule) resize of
 * BGR8 frames to normalized planar RGB f32: the GPU frame-resize path of the
 * high-resolution benchmark configuration. */
void dav2o_preprocess_bgr8_bilinear(const uint8_t* bgr, int width, int height,
                                    ptrdiff_t stride, int dst_width,
                                    int dst_height, float* rgb_chw);

/* src/shaders/layer_norm.glsl:27-67. */
void dav2o_layer_norm(const float* input, const float* weight,
                      const float* bias, float* output, size_t rows,
                      int columns, float epsilon);

/* src/shaders/gelu.glsl:16-49 (Numerical Recipes erfc form of exact GELU). */
void dav2o_gelu(const float* input, float* output, size_t count);

/* src/shaders/softmax_lastdim.glsl:19-69 applied to input*scale
 * (scale=1 reproduces the shader; 0.125 is the 1/sqrt(64) query scale that
 * the reference folds into bmm.glsl:57-61, exact for a power of two). */
void dav2o_softmax_rows(const float* input, float* output, size_t rows,
                        int columns, float scale);

/* src/shaders/add_scaled.glsl:23-31 (precise: no FMA). */
void dav2o_add_scaled(const float* residual, const float* addend,
                      const float* scale, float* output, size_t count,
                      int columns);

/* src/shaders/relu.glsl, add.glsl, sigmoid_scale.glsl. */
void dav2o_relu(const float* input, float* output, size_t count);
void dav2o_add(const float* left, const float* right, float* output,
               size_t count);
void dav2o_sigmoid_scale(const float* input, float* output, size_t count,
                         float scale);

/* src/shaders/bilinear_align_true.glsl:27-63, planar [C,H,W]. */
void dav2o_bilinear_align_true(const float* input, int in_width,
                               int in_height, int out_width, int out_height,
                               int channels, float* output);

/* src/shaders/reduce_minmax.glsl:10-33 -> range[0]=min, range[1]=max. */
void dav2o_reduce_minmax(const float* input, size_t count, float* range);
/* src/shaders/normalize_relative.glsl:8-16 (in place). */
void dav2o_normalize_relative(float* depth, size_t count, const float* range);
/* src/shaders/normalize_metric.glsl (in place). */
void dav2o_normalize_metric(float* depth, size_t count, const float* range,
                            float maximum_depth);

/* src/shaders/quantize_rows_int8_fused.glsl:20-55. columns % 4 == 0.
 * scale = max(absmax/127, 1e-8); code = rint(clamp(x/scale, +-127)). */
void dav2o_quantize_rows_s8(const float* input, size_t rows, int columns,
                            size_t input_offset, uint32_t* packed,
                            float* scales);

/* src/shaders/im2col_quantize_int8.glsl:26-84 on planar [C,H,W].
 * Row = output pixel y*OW+x; column = c*k*k + ky*k + kx; rows padded to
 * ceil(C*k*k/4) words; code = rint(clamp(x*(1/scale), +-127)). */
void dav2o_im2col_quantize_s8(const float* input, int in_width, int in_height,
                              int in_channels, int out_width, int out_height,
                              int kernel, int stride, int padding,
                              uint32_t* packed, float* scales);

/* src/shaders/linear_int8_tiled.glsl:40-117: s8.s8 -> s32 per output, then
 * float(acc)*s_in[row]*s_w[col] (+bias[col]). Transposed stores write
 * out[col*row_stride + row + row_offset]; otherwise
 * out[(row + row_offset)*out_columns + col]. */
void dav2o_linear_s8(const uint32_t* packed_input, const uint32_t* packed_weight,
                     const float* input_scales, const float* weight_scales,
                     const float* bias, size_t rows, int in_columns,
                     int out_columns, size_t row_offset, size_t row_stride,
                     int transposed, int has_bias, float* output);

/* src/shaders/conv_transpose_int8.glsl:31-58. packed_input rows are pixels
 * (from im2col with k=1), weight rows are (ky*k+kx)*Cout+co. Output planar
 * [Cout, H*k, W*k]. */
void dav2o_conv_transpose_s8(const uint32_t* packed_input,
                             const uint32_t* packed_weight,
                             const float* input_scales,
                             const float* weight_scales, const float* bias,
                             int in_width, int in_height, int in_channels,
                             int out_channels, int kernel, float* output);

/* src/gpu_model.cpp:207-284: per-output-row symmetric int8 weight codes.
 * Ordinary weights: rows = dim0, columns = elements/dim0 (PyTorch layout).
 * ConvTranspose weights [Cin,Cout,k,k]: rows = (ky*k+kx)*Cout+co,
 * columns = Cin (transposed_layout=1, kernel=k, out_channels=Cout). */
void dav2o_pack_weight_s8(const float* weight, size_t rows, int columns,
                          int transposed_layout, int out_channels, int kernel,
                          uint32_t* packed, float* scales);

/* src/shaders/linear_common.glsl: Y = X W^T + b, W is [out, in]. */
void dav2o_linear_f32(const float* input, const float* weight,
                      const float* bias, size_t rows, int in_columns,
                      int out_columns, float* output);

/* src/shaders/conv2d_common.glsl:55-139: direct conv, planar CHW,
 * weights [Co,Ci,k,k]; bias may be NULL. */
void dav2o_conv2d_f32(const float* input, const float* weight,
                      const float* bias, int in_width, int in_height,
                      int in_channels, int out_channels, int kernel,
                      int stride, int padding, float* output);

/* src/shaders/conv_transpose_nonoverlap_common.glsl:55-91 (kernel==stride),
 * weights [Ci,Co,k,k]. */
void dav2o_conv_transpose_f32(const float* input, const float* weight,
                              const float* bias, int in_width, int in_height,
                              int in_channels, int out_channels, int kernel,
                              float* output);

/* src/shaders/project_tokens_common.glsl:60-150: tokens [1+hw, D] (row 0 =
 * cls, skipped) -> planar [Cout, hw]. */
void dav2o_project_tokens_f32(const float* tokens, const float* weight,
                              const float* bias, int width, int height,
                              int embedding, int out_channels, float* output);

/* src/shaders/prepare_tokens.glsl:28-65: direct 14x14/14 patch conv + bias,
 * row 0 = cls token. Output [1+pw*ph, D]. */
void dav2o_patch_embed_f32(const float* image, const float* weight,
                           const float* bias, const float* class_token,
                           int in_width, int in_height, int embedding,
                           float* tokens);

/* src/shaders/position_bicubic.glsl:76-105 with the scale rule of
 * src/operators.cpp:1346-1364: the 37x37 grid of pos_embed [1370, D]
 * (row 0 = cls) resized to planar [D, ph, pw]. */
void dav2o_position_bicubic(const float* pos_embed, int embedding,
                            int patch_width, int patch_height, float* planar);

/* src/shaders/add_position.glsl:25-40 (in place on tokens [1+pw*ph, D]). */
void dav2o_add_position(float* tokens, const float* planar_position,
                        const float* pos_embed, int patch_width,
                        int patch_height, int embedding);

/* src/operators.cpp:1098-1209 with bmm.glsl score/value modes and
 * softmax_lastdim.glsl: qkv [N, 3*H*64] -> out [N, H*64]. */
void dav2o_attention_head64(const float* qkv, int tokens, int heads,
                            float* output);

/* PyTorch's F.interpolate(mode="bilinear", align_corners=False) for planar
 * [C,H,W] f32 (used by the square frame resize). */
void dav2o_bilinear_half_pixel(const float* input, int in_width,
                               int in_height, int out_width, int out_height,
                               int channels, float* output);

/* Number of OpenMP threads the oracle uses (1 when built without OpenMP). */
int dav2o_threads(void);
void dav2o_set_threads(int threads);

#ifdef __cplusplus
}
#endif

#endif
