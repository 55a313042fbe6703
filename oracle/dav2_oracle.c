/*
 * CPU oracle for the Depth Anything V2 tensor-operator hot path.
 *
 * TEST INFRASTRUCTURE ONLY: a plain-C restatement of the reference shaders'
 * arithmetic, used by tests/ and by bench.py's CPU baseline as the checker.
 * The product library never links or calls it. Each function names the
 * reference file:line it restates. Built with -ffp-contract=off so that the
 * written operation order is the executed one.
 */
#include "dav2_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }
static float fmaxf_(float a, float b) { return a > b ? a : b; }

int dav2o_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void dav2o_set_threads(int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
}

/* ---------------------------------------------------------------- CRC-32 */
/* Reflected CRC-32 (polynomial 0xEDB88320), src/gpu_model.cpp:100-125. */
uint32_t dav2o_crc32(const void* data, size_t bytes) {
    static uint32_t table[256];
    static int ready = 0;
    if (!ready) {
        for (uint32_t n = 0; n < 256; ++n) {
            uint32_t c = n;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xedb88320u ^ (c >> 1) : c >> 1;
            table[n] = c;
        }
        ready = 1;
    }
    const unsigned char* p = (const unsigned char*)data;
    uint32_t crc = 0xffffffffu;
    for (size_t i = 0; i < bytes; ++i) crc = table[(crc ^ p[i]) & 0xffu] ^ (crc >> 8);
    return crc ^ 0xffffffffu;
}

/* --------------------------------------------------------- preprocessing */
/* src/image.cpp:138-161: scale = max(size/h, size/w); each side is
 * round-half-even(scale*side/14)*14, at least input_size, then rounded up to
 * a multiple of 14. */
int dav2o_network_shape(int width, int height, int input_size,
                        int* out_width, int* out_height) {
    if (width <= 0 || height <= 0 || input_size <= 0) return -1;
    const double sh = (double)input_size / (double)height;
    const double sw = (double)input_size / (double)width;
    const double scale = sh > sw ? sh : sw;
    int oh = (int)nearbyint(scale * height / 14.0) * 14;
    int ow = (int)nearbyint(scale * width / 14.0) * 14;
    oh = imax(oh, input_size);
    ow = imax(ow, input_size);
    if (oh % 14) oh = ((oh + 13) / 14) * 14;
    if (ow % 14) ow = ((ow + 13) / 14) * 14;
    *out_width = ow;
    *out_height = oh;
    return 0;
}

/* OpenCV interpolateCubic coefficients in float, src/image.cpp:21-39. */
static void cubic_coeffs_cv(float x, float c[4]) {
    const float a = -0.75f;
    c[0] = ((a * (x + 1.0f) - 5.0f * a) * (x + 1.0f) + 8.0f * a) * (x + 1.0f) - 4.0f * a;
    c[1] = ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
    const float o = 1.0f - x;
    c[2] = ((a + 2.0f) * o - (a + 3.0f)) * o * o + 1.0f;
    c[3] = 1.0f - c[0] - c[1] - c[2];
}

int dav2o_preprocess_bgr8(const uint8_t* bgr, int width, int height,
                          ptrdiff_t stride, int dw, int dh, float* out) {
    if (!bgr || width <= 0 || height <= 0 || stride < (ptrdiff_t)width * 3 || dw <= 0 || dh <= 0)
        return -1;
    static const double mean[3] = {0.485, 0.456, 0.406};
    static const double stdv[3] = {0.229, 0.224, 0.225};
    const double scale_x = (double)width / dw;
    const double scale_y = (double)height / dh;
    int* xi = (int*)malloc(sizeof(int) * (size_t)dw);
    float* xc = (float*)malloc(sizeof(float) * 4 * (size_t)dw);
    double* hor = (double*)malloc(sizeof(double) * (size_t)height * dw * 3);
    if (!xi || !xc || !hor) { free(xi); free(xc); free(hor); return -2; }
    for (int dx = 0; dx < dw; ++dx) {
        const float coord = (float)((dx + 0.5) * scale_x - 0.5);
        const int idx = (int)floorf(coord);
        xi[dx] = idx;
        cubic_coeffs_cv(coord - idx, xc + 4 * dx);
    }
    /* horizontal pass: double accumulation of unit = byte/255 (RGB order) */
#pragma omp parallel for schedule(static)
    for (int sy = 0; sy < height; ++sy) {
        const uint8_t* row = bgr + (ptrdiff_t)sy * stride;
        for (int dx = 0; dx < dw; ++dx) {
            const float* al = xc + 4 * dx;
            for (int ch = 0; ch < 3; ++ch) {
                double v = 0.0;
                for (int t = 0; t < 4; ++t) {
                    const int sx = imax(0, imin(xi[dx] - 1 + t, width - 1));
                    const double unit = (double)row[sx * 3 + (2 - ch)] / 255.0;
                    v += unit * al[t];
                }
                hor[((size_t)sy * dw + dx) * 3 + ch] = v;
            }
        }
    }
    const size_t plane = (size_t)dw * dh;
#pragma omp parallel for schedule(static)
    for (int dy = 0; dy < dh; ++dy) {
        const float coord = (float)((dy + 0.5) * scale_y - 0.5);
        const int base = (int)floorf(coord);
        float be[4];
        cubic_coeffs_cv(coord - base, be);
        int sy[4];
        for (int t = 0; t < 4; ++t) sy[t] = imax(0, imin(base - 1 + t, height - 1));
        for (int dx = 0; dx < dw; ++dx) {
            for (int ch = 0; ch < 3; ++ch) {
                const double r =
                    hor[((size_t)sy[0] * dw + dx) * 3 + ch] * be[0] +
                    hor[((size_t)sy[1] * dw + dx) * 3 + ch] * be[1] +
                    hor[((size_t)sy[2] * dw + dx) * 3 + ch] * be[2] +
                    hor[((size_t)sy[3] * dw + dx) * 3 + ch] * be[3];
                out[(size_t)ch * plane + (size_t)dy * dw + dx] =
                    (float)((r - mean[ch]) / stdv[ch]);
            }
        }
    }
    free(xi); free(xc); free(hor);
    return 0;
}

int dav2o_preprocess_inferbridge_bgra8(const uint8_t* src, int width,
                                       int height, ptrdiff_t stride,
                                       int dw, int dh, float* out) {
    if (!src || width <= 0 || height <= 0 || stride < (ptrdiff_t)width * 4 || dw <= 0 || dh <= 0)
        return -1;
    static const float mean[3] = {0.485f, 0.456f, 0.406f};
    static const float stdv[3] = {0.229f, 0.224f, 0.225f};
    const float scale_x = (float)width / dw;
    const float scale_y = (float)height / dh;
    const size_t plane = (size_t)dw * dh;
    for (int y = 0; y < dh; ++y) {
        const int sy = imin((int)floorf(y * scale_y), height - 1);
        const uint8_t* row = src + (ptrdiff_t)sy * stride;
        for (int x = 0; x < dw; ++x) {
            const int sx = imin((int)floorf(x * scale_x), width - 1);
            const uint8_t* px = row + (ptrdiff_t)sx * 4;
            for (int ch = 0; ch < 3; ++ch) {
                const float unit = (float)px[ch] / 255.0f;
                out[(size_t)ch * plane + (size_t)y * dw + x] = (unit - mean[ch]) / stdv[ch];
            }
        }
    }
    return 0;
}

/* Cubic coefficient as used by the GPU preprocess shader (a=-0.75). */
static float cubic_w(int tap, float t) {
    const float a = -0.75f;
    float x;
    switch (tap) {
        case 0: x = t + 1.0f; return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a;
        case 1: x = t; return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
        case 2: x = 1.0f - t; return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
        default: x = 2.0f - t; return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a;
    }
}

void dav2o_preprocess_u32_bicubic(const uint32_t* pixels, int sw, int sh,
                                  int stride_px, int rgba, int dw, int dh,
                                  float* out) {
    static const float mean[3] = {0.485f, 0.456f, 0.406f};
    static const float dev[3] = {0.229f, 0.224f, 0.225f};
    const size_t plane = (size_t)dw * dh;
#pragma omp parallel for schedule(static)
    for (int y = 0; y < dh; ++y) {
        for (int x = 0; x < dw; ++x) {
            const float src_x = ((float)x + 0.5f) * (float)sw / (float)dw - 0.5f;
            const float src_y = ((float)y + 0.5f) * (float)sh / (float)dh - 0.5f;
            const int bx = (int)floorf(src_x), by = (int)floorf(src_y);
            const float fx = src_x - (float)bx, fy = src_y - (float)by;
            for (int ch = 0; ch < 3; ++ch) {
                const int shift = ch == 1 ? 8 : (rgba ? (ch == 0 ? 0 : 16) : (ch == 0 ? 16 : 0));
                float resized = 0.0f;
                for (int ty = 0; ty < 4; ++ty) {
                    const int iy = imax(0, imin(by - 1 + ty, sh - 1));
                    float row = 0.0f;
                    for (int tx = 0; tx < 4; ++tx) {
                        const int ix = imax(0, imin(bx - 1 + tx, sw - 1));
                        const uint32_t p = pixels[(size_t)iy * stride_px + ix];
                        row += (float)((p >> shift) & 255u) / 255.0f * cubic_w(tx, fx);
                    }
                    resized += row * cubic_w(ty, fy);
                }
                out[(size_t)ch * plane + (size_t)y * dw + x] = (resized - mean[ch]) / dev[ch];
            }
        }
    }
}

/* PyTorch upsample_bilinear2d, align_corners=False: src = max(scale*(d+0.5)-0.5, 0),
 * i0 = floor, i1 = i0 + (i0 < in-1), lambda = src - i0. */
static void hp_coord(int d, int in, int out, int* i0, int* i1, float* l1) {
    const float scale = (float)in / (float)out;
    float src = scale * ((float)d + 0.5f) - 0.5f;
    if (src < 0.0f) src = 0.0f;
    int a = (int)src;
    if (a > in - 1) a = in - 1;
    *i0 = a;
    *i1 = a + (a < in - 1 ? 1 : 0);
    *l1 = src - (float)a;
}

void dav2o_preprocess_bgr8_bilinear(const uint8_t* bgr, int width, int height,
                                    ptrdiff_t stride, int dw, int dh,
                                    float* out) {
    static const float mean[3] = {0.485f, 0.456f, 0.406f};
    static const float dev[3] = {0.229f, 0.224f, 0.225f};
    const size_t plane = (size_t)dw * dh;
#pragma omp parallel for schedule(static)
    for (int y = 0; y < dh; ++y) {
        int y0, y1; float ly;
        hp_coord(y, height, dh, &y0, &y1, &ly);
        for (int x = 0; x < dw; ++x) {
            int x0, x1; float lx;
            hp_coord(x, width, dw, &x0, &x1, &lx);
            for (int ch = 0; ch < 3; ++ch) {
                const int b = 2 - ch;
                const float v00 = bgr[(ptrdiff_t)y0 * stride + x0 * 3 + b] / 255.0f;
                const float v01 = bgr[(ptrdiff_t)y0 * stride + x1 * 3 + b] / 255.0f;
                const float v10 = bgr[(ptrdiff_t)y1 * stride + x0 * 3 + b] / 255.0f;
                const float v11 = bgr[(ptrdiff_t)y1 * stride + x1 * 3 + b] / 255.0f;
                const float top = v00 * (1.0f - lx) + v01 * lx;
                const float bot = v10 * (1.0f - lx) + v11 * lx;
                const float v = top * (1.0f - ly) + bot * ly;
                out[(size_t)ch * plane + (size_t)y * dw + x] = (v - mean[ch]) / dev[ch];
            }
        }
    }
}

void dav2o_bilinear_half_pixel(const float* in, int iw, int ih, int ow, int oh,
                               int channels, float* out) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < channels; ++c) {
        const float* src = in + (size_t)c * iw * ih;
        for (int y = 0; y < oh; ++y) {
            int y0, y1; float ly;
            hp_coord(y, ih, oh, &y0, &y1, &ly);
            for (int x = 0; x < ow; ++x) {
                int x0, x1; float lx;
                hp_coord(x, iw, ow, &x0, &x1, &lx);
                const float top = src[(size_t)y0 * iw + x0] * (1.0f - lx) + src[(size_t)y0 * iw + x1] * lx;
                const float bot = src[(size_t)y1 * iw + x0] * (1.0f - lx) + src[(size_t)y1 * iw + x1] * lx;
                out[((size_t)c * oh + y) * ow + x] = top * (1.0f - ly) + bot * ly;
            }
        }
    }
}

/* ------------------------------------------------------------ row ops */
/* layer_norm.glsl: 64 lanes accumulate strided partial sums of x and x^2,
 * tree-reduced; var = max(E[x^2]-mean^2, 0); out = (x-mean)*rsqrt*w + b. */
void dav2o_layer_norm(const float* input, const float* weight,
                      const float* bias, float* output, size_t rows,
                      int columns, float eps) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        const float* x = input + r * (size_t)columns;
        float ps[64], pq[64];
        for (int lane = 0; lane < 64; ++lane) {
            float s = 0.0f, q = 0.0f;
            for (int c = lane; c < columns; c += 64) { s += x[c]; q += x[c] * x[c]; }
            ps[lane] = s; pq[lane] = q;
        }
        for (int w = 32; w > 0; w >>= 1)
            for (int lane = 0; lane < w; ++lane) { ps[lane] += ps[lane + w]; pq[lane] += pq[lane + w]; }
        const float denom = fmaxf_((float)columns, 1.0f);
        const float mean = ps[0] / denom;
        const float var = fmaxf_(pq[0] / denom - mean * mean, 0.0f);
        const float inv = 1.0f / sqrtf(var + eps);
        float* y = output + r * (size_t)columns;
        for (int c = 0; c < columns; ++c) y[c] = (x[c] - mean) * inv * weight[c] + bias[c];
    }
}

static float gelu_nr(float value) {
    const float x = value * 0.7071067811865475f;
    const float m = fabsf(x);
    const float t = 1.0f / (1.0f + 0.5f * m);
    const float p = -1.26551223f + t * (1.00002368f + t * (0.37409196f + t * (0.09678418f +
        t * (-0.18628806f + t * (0.27886807f + t * (-1.13520398f + t * (1.48851587f +
        t * (-0.82215223f + t * 0.17087277f))))))));
    const float erfc_m = t * expf(-m * m + p);
    const float erf_v = x >= 0.0f ? 1.0f - erfc_m : erfc_m - 1.0f;
    return 0.5f * value * (1.0f + erf_v);
}

void dav2o_gelu(const float* input, float* output, size_t count) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < count; ++i) output[i] = gelu_nr(input[i]);
}

void dav2o_softmax_rows(const float* input, float* output, size_t rows,
                        int columns, float scale) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        const float* x = input + r * (size_t)columns;
        float* y = output + r * (size_t)columns;
        float m = -FLT_MAX;
        for (int c = 0; c < columns; ++c) { const float v = x[c] * scale; if (v > m) m = v; }
        float s = 0.0f;
        for (int c = 0; c < columns; ++c) { const float e = expf(x[c] * scale - m); y[c] = e; s += e; }
        const float inv = 1.0f / fmaxf_(s, 1.0e-20f);
        for (int c = 0; c < columns; ++c) y[c] *= inv;
    }
}

void dav2o_add_scaled(const float* residual, const float* addend,
                      const float* scale, float* output, size_t count,
                      int columns) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < count; ++i) {
        const float scaled = addend[i] * scale[i % (size_t)columns];
        output[i] = residual[i] + scaled;
    }
}

void dav2o_relu(const float* input, float* output, size_t count) {
    for (size_t i = 0; i < count; ++i) output[i] = input[i] > 0.0f ? input[i] : 0.0f;
}

void dav2o_add(const float* left, const float* right, float* output, size_t count) {
    for (size_t i = 0; i < count; ++i) output[i] = left[i] + right[i];
}

void dav2o_sigmoid_scale(const float* input, float* output, size_t count, float scale) {
    for (size_t i = 0; i < count; ++i) output[i] = scale / (1.0f + expf(-input[i]));
}

/* bilinear_align_true.glsl: src = (x*(in-1))/(out-1) in f32. */
void dav2o_bilinear_align_true(const float* input, int iw, int ih, int ow,
                               int oh, int channels, float* output) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < channels; ++c) {
        const float* src = input + (size_t)c * iw * ih;
        for (int y = 0; y < oh; ++y) {
            const float sy = oh > 1 ? (float)y * (float)(ih - 1) / (float)(oh - 1) : 0.0f;
            const int y0 = (int)floorf(sy);
            const int y1 = imin(y0 + 1, ih - 1);
            const float fy = sy - (float)y0;
            for (int x = 0; x < ow; ++x) {
                const float sx = ow > 1 ? (float)x * (float)(iw - 1) / (float)(ow - 1) : 0.0f;
                const int x0 = (int)floorf(sx);
                const int x1 = imin(x0 + 1, iw - 1);
                const float fx = sx - (float)x0;
                const float top = src[(size_t)y0 * iw + x0] * (1.0f - fx) + src[(size_t)y0 * iw + x1] * fx;
                const float bot = src[(size_t)y1 * iw + x0] * (1.0f - fx) + src[(size_t)y1 * iw + x1] * fx;
                output[((size_t)c * oh + y) * ow + x] = top * (1.0f - fy) + bot * fy;
            }
        }
    }
}

void dav2o_reduce_minmax(const float* input, size_t count, float* range) {
    float lo = INFINITY, hi = -INFINITY;
    for (size_t i = 0; i < count; ++i) {
        lo = fminf(lo, input[i]);
        hi = fmaxf(hi, input[i]);
    }
    range[0] = lo;
    range[1] = hi;
}

static float clamp01(float v) { return v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v); }

void dav2o_normalize_relative(float* depth, size_t count, const float* range) {
    const float lo = range[0];
    const float span = range[1] - lo;
    for (size_t i = 0; i < count; ++i)
        depth[i] = span > 1.0e-12f ? clamp01((depth[i] - lo) / span) : 0.0f;
}

void dav2o_normalize_metric(float* depth, size_t count, const float* range,
                            float maximum_depth) {
    const float lo = range[0];
    const float span = maximum_depth - lo;
    for (size_t i = 0; i < count; ++i)
        depth[i] = span > 1.0e-12f ? clamp01((depth[i] - lo) / span) : 0.0f;
}

/* --------------------------------------------------------------- int8 */
static uint32_t pack4(const int v[4]) {
    uint32_t w = 0;
    for (int j = 0; j < 4; ++j) w |= ((uint32_t)v[j] & 0xffu) << (8 * j);
    return w;
}

static float clamp127(float v) { return v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v); }

void dav2o_quantize_rows_s8(const float* input, size_t rows, int columns,
                            size_t input_offset, uint32_t* packed,
                            float* scales) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        const float* x = input + input_offset + r * (size_t)columns;
        float m = 0.0f;
        for (int c = 0; c < columns; ++c) m = fmaxf_(m, fabsf(x[c]));
        const float scale = fmaxf_(m / 127.0f, 1.0e-8f);
        scales[r] = scale;
        const int words = columns / 4;
        for (int w = 0; w < words; ++w) {
            int v[4];
            for (int j = 0; j < 4; ++j) v[j] = (int)rintf(clamp127(x[w * 4 + j] / scale));
            packed[r * (size_t)words + w] = pack4(v);
        }
    }
}

static float im2col_value(const float* in, int iw, int ih, int ow, int k,
                          int s, int pad, size_t row, int column) {
    const int ox = (int)(row % (size_t)ow), oy = (int)(row / (size_t)ow);
    const int area = k * k;
    const int ci = column / area, ki = column % area;
    const int kx = ki % k, ky = ki / k;
    const int ix = ox * s + kx - pad, iy = oy * s + ky - pad;
    if (ix < 0 || iy < 0 || ix >= iw || iy >= ih) return 0.0f;
    return in[((size_t)ci * ih + iy) * iw + ix];
}

void dav2o_im2col_quantize_s8(const float* input, int iw, int ih, int ic,
                              int ow, int oh, int k, int s, int pad,
                              uint32_t* packed, float* scales) {
    const size_t rows = (size_t)ow * oh;
    const int columns = ic * k * k;
    const int words = (columns + 3) / 4;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        float m = 0.0f;
        for (int c = 0; c < columns; ++c) m = fmaxf_(m, fabsf(im2col_value(input, iw, ih, ow, k, s, pad, r, c)));
        const float scale = fmaxf_(m / 127.0f, 1.0e-8f);
        scales[r] = scale;
        const float inv = 1.0f / scale;
        for (int w = 0; w < words; ++w) {
            int v[4];
            for (int j = 0; j < 4; ++j) {
                const int c = w * 4 + j;
                v[j] = c < columns ? (int)rintf(clamp127(im2col_value(input, iw, ih, ow, k, s, pad, r, c) * inv)) : 0;
            }
            packed[r * (size_t)words + w] = pack4(v);
        }
    }
}

static int32_t dot4(uint32_t a, uint32_t b) {
    int32_t s = 0;
    for (int j = 0; j < 4; ++j) s += (int32_t)(int8_t)(a >> (8 * j)) * (int32_t)(int8_t)(b >> (8 * j));
    return s;
}

void dav2o_linear_s8(const uint32_t* pin, const uint32_t* pw, const float* s_in,
                     const float* s_w, const float* bias, size_t rows,
                     int in_columns, int out_columns, size_t row_offset,
                     size_t row_stride, int transposed, int has_bias,
                     float* out) {
    const int words = in_columns / 4;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        for (int n = 0; n < out_columns; ++n) {
            int32_t acc = 0;
            for (int w = 0; w < words; ++w) acc += dot4(pin[r * (size_t)words + w], pw[(size_t)n * words + w]);
            const float v = (float)acc * s_in[r] * s_w[n] + (has_bias ? bias[n] : 0.0f);
            const size_t dr = r + row_offset;
            if (transposed) out[(size_t)n * row_stride + dr] = v;
            else out[dr * (size_t)out_columns + n] = v;
        }
    }
}

void dav2o_conv_transpose_s8(const uint32_t* pin, const uint32_t* pw,
                             const float* s_in, const float* s_w,
                             const float* bias, int iw, int ih, int ic,
                             int oc, int k, float* out) {
    const int words = ic / 4;
    const int ow = iw * k, oh = ih * k;
#pragma omp parallel for schedule(static)
    for (int co = 0; co < oc; ++co) {
        for (int y = 0; y < oh; ++y) {
            for (int x = 0; x < ow; ++x) {
                const int in_row = (y / k) * iw + (x / k);
                const int wrow = ((y % k) * k + (x % k)) * oc + co;
                int32_t acc = 0;
                for (int w = 0; w < words; ++w) acc += dot4(pin[(size_t)in_row * words + w], pw[(size_t)wrow * words + w]);
                out[((size_t)co * oh + y) * ow + x] = (float)acc * s_in[in_row] * s_w[wrow] + bias[co];
            }
        }
    }
}

void dav2o_pack_weight_s8(const float* weight, size_t rows, int columns,
                          int transposed_layout, int out_channels, int kernel,
                          uint32_t* packed, float* scales) {
    const int words = columns / 4;
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        float m = 0.0f;
        float* row = (float*)malloc(sizeof(float) * (size_t)columns);
        for (int c = 0; c < columns; ++c) {
            float v;
            if (!transposed_layout) {
                v = weight[r * (size_t)columns + c];
            } else {
                /* row = (ky*k+kx)*Cout + co, column = ci; source [Ci,Co,k,k] */
                const size_t ki = r / (size_t)out_channels, co = r % (size_t)out_channels;
                const size_t ky = ki / (size_t)kernel, kx = ki % (size_t)kernel;
                v = weight[(((size_t)c * out_channels + co) * kernel + ky) * kernel + kx];
            }
            row[c] = v;
            m = fmaxf_(m, fabsf(v));
        }
        const float scale = fmaxf_(m / 127.0f, 1.0e-8f);
        scales[r] = scale;
        for (int w = 0; w < words; ++w) {
            int v[4];
            for (int j = 0; j < 4; ++j) {
                float q = row[w * 4 + j] / scale;
                q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
                v[j] = (int)nearbyintf(q);
            }
            packed[r * (size_t)words + w] = pack4(v);
        }
        free(row);
    }
}

/* ----------------------------------------------------------- fp32 GEMM-ish */
void dav2o_linear_f32(const float* input, const float* weight,
                      const float* bias, size_t rows, int in_columns,
                      int out_columns, float* output) {
#pragma omp parallel for schedule(static)
    for (size_t r = 0; r < rows; ++r) {
        const float* x = input + r * (size_t)in_columns;
        for (int n = 0; n < out_columns; ++n) {
            const float* w = weight + (size_t)n * in_columns;
            float s = 0.0f;
            for (int k = 0; k < in_columns; ++k) s += x[k] * w[k];
            output[r * (size_t)out_columns + n] = s + (bias ? bias[n] : 0.0f);
        }
    }
}

void dav2o_conv2d_f32(const float* input, const float* weight,
                      const float* bias, int iw, int ih, int ic, int oc,
                      int k, int s, int pad, float* output) {
    const int ow = (iw + 2 * pad - k) / s + 1;
    const int oh = (ih + 2 * pad - k) / s + 1;
#pragma omp parallel for schedule(static)
    for (int co = 0; co < oc; ++co) {
        for (int y = 0; y < oh; ++y) {
            for (int x = 0; x < ow; ++x) {
                float acc = bias ? bias[co] : 0.0f;
                for (int ci = 0; ci < ic; ++ci) {
                    for (int ky = 0; ky < k; ++ky) {
                        const int iy = y * s + ky - pad;
                        if (iy < 0 || iy >= ih) continue;
                        for (int kx = 0; kx < k; ++kx) {
                            const int ix = x * s + kx - pad;
                            if (ix < 0 || ix >= iw) continue;
                            acc += input[((size_t)ci * ih + iy) * iw + ix] *
                                   weight[(((size_t)co * ic + ci) * k + ky) * k + kx];
                        }
                    }
                }
                output[((size_t)co * oh + y) * ow + x] = acc;
            }
        }
    }
}

void dav2o_conv_transpose_f32(const float* input, const float* weight,
                              const float* bias, int iw, int ih, int ic,
                              int oc, int k, float* output) {
    const int ow = iw * k, oh = ih * k;
#pragma omp parallel for schedule(static)
    for (int co = 0; co < oc; ++co) {
        for (int y = 0; y < oh; ++y) {
            for (int x = 0; x < ow; ++x) {
                float acc = 0.0f;
                for (int ci = 0; ci < ic; ++ci)
                    acc += input[((size_t)ci * ih + y / k) * iw + x / k] *
                           weight[(((size_t)ci * oc + co) * k + (y % k)) * k + (x % k)];
                output[((size_t)co * oh + y) * ow + x] = acc + bias[co];
            }
        }
    }
}

void dav2o_project_tokens_f32(const float* tokens, const float* weight,
                              const float* bias, int width, int height,
                              int embedding, int oc, float* output) {
    const size_t hw = (size_t)width * height;
#pragma omp parallel for schedule(static)
    for (size_t p = 0; p < hw; ++p) {
        const float* x = tokens + (p + 1) * (size_t)embedding;
        for (int co = 0; co < oc; ++co) {
            const float* w = weight + (size_t)co * embedding;
            float s = 0.0f;
            for (int k = 0; k < embedding; ++k) s += x[k] * w[k];
            output[(size_t)co * hw + p] = s + bias[co];
        }
    }
}

void dav2o_patch_embed_f32(const float* image, const float* weight,
                           const float* bias, const float* cls, int iw,
                           int ih, int embedding, float* tokens) {
    const int pw = iw / 14, ph = ih / 14;
    for (int f = 0; f < embedding; ++f) tokens[f] = cls[f];
#pragma omp parallel for schedule(static)
    for (int p = 0; p < pw * ph; ++p) {
        const int px = p % pw, py = p / pw;
        for (int f = 0; f < embedding; ++f) {
            float s = 0.0f;
            for (int c = 0; c < 3; ++c)
                for (int ky = 0; ky < 14; ++ky)
                    for (int kx = 0; kx < 14; ++kx)
                        s += image[((size_t)c * ih + py * 14 + ky) * iw + px * 14 + kx] *
                             weight[(((size_t)f * 3 + c) * 14 + ky) * 14 + kx];
            tokens[(size_t)(p + 1) * embedding + f] = s + bias[f];
        }
    }
}

static float cc1(float x, float a) { return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f; }
static float cc2(float x, float a) { return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a; }

static float cubic_interp(float x0, float x1, float x2, float x3, float t) {
    const float a = -0.75f;
    const float c0 = cc2(t + 1.0f, a), c1 = cc1(t, a), c2 = cc1(1.0f - t, a), c3 = cc2((1.0f - t) + 1.0f, a);
    return x0 * c0 + x1 * c1 + x2 * c2 + x3 * c3;
}

void dav2o_position_bicubic(const float* pos, int D, int pw, int ph,
                            float* planar) {
    const float sx = (pw == 37 && ph == 37) ? 1.0f : (float)(1.0 / (((double)pw + 0.1) / 37.0));
    const float sy = (pw == 37 && ph == 37) ? 1.0f : (float)(1.0 / (((double)ph + 0.1) / 37.0));
#pragma omp parallel for schedule(static)
    for (int f = 0; f < D; ++f) {
        for (int y = 0; y < ph; ++y) {
            for (int x = 0; x < pw; ++x) {
                const float src_x = ((float)x + 0.5f) * sx - 0.5f;
                const float src_y = ((float)y + 0.5f) * sy - 0.5f;
                const int bx = (int)floorf(src_x), by = (int)floorf(src_y);
                const float tx = src_x - (float)bx, ty = src_y - (float)by;
                float rows[4];
                for (int k = 0; k < 4; ++k) {
                    const int yy = imax(0, imin(by - 1 + k, 36));
                    float v[4];
                    for (int j = 0; j < 4; ++j) {
                        const int xx = imax(0, imin(bx - 1 + j, 36));
                        v[j] = pos[(size_t)(1 + yy * 37 + xx) * D + f];
                    }
                    rows[k] = cubic_interp(v[0], v[1], v[2], v[3], tx);
                }
                planar[((size_t)f * ph + y) * pw + x] = cubic_interp(rows[0], rows[1], rows[2], rows[3], ty);
            }
        }
    }
}

void dav2o_add_position(float* tokens, const float* planar, const float* pos,
                        int pw, int ph, int D) {
    const size_t hw = (size_t)pw * ph;
    for (int f = 0; f < D; ++f) tokens[f] = tokens[f] + pos[f];
    for (size_t p = 0; p < hw; ++p)
        for (int f = 0; f < D; ++f)
            tokens[(p + 1) * (size_t)D + f] = tokens[(p + 1) * (size_t)D + f] + planar[(size_t)f * hw + p];
}

void dav2o_attention_head64(const float* qkv, int N, int H, float* out) {
    const size_t E = (size_t)H * 64;
#pragma omp parallel for schedule(dynamic, 4)
    for (int t = 0; t < N; ++t) {
        float* scores = (float*)malloc(sizeof(float) * (size_t)N);
        for (int h = 0; h < H; ++h) {
            float m = -FLT_MAX;
            for (int s = 0; s < N; ++s) {
                float acc = 0.0f;
                for (int f = 0; f < 64; ++f)
                    acc += qkv[(size_t)t * E * 3 + (size_t)h * 64 + f] * 0.125f *
                           qkv[(size_t)s * E * 3 + E + (size_t)h * 64 + f];
                scores[s] = acc;
                if (acc > m) m = acc;
            }
            float den = 0.0f;
            for (int s = 0; s < N; ++s) { scores[s] = expf(scores[s] - m); den += scores[s]; }
            const float inv = 1.0f / fmaxf_(den, 1.0e-20f);
            for (int f = 0; f < 64; ++f) {
                float acc = 0.0f;
                for (int s = 0; s < N; ++s)
                    acc += scores[s] * inv * qkv[(size_t)s * E * 3 + 2 * E + (size_t)h * 64 + f];
                out[(size_t)t * E + (size_t)h * 64 + f] = acc;
            }
        }
        free(scores);
    }
}
