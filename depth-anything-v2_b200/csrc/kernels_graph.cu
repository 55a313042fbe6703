// Kernels the executor graph needs around the GEMMs: patch im2col, the
// bicubic positional-embedding resize, token initialisation, channels-last
// bilinear resize and im2col-quantize, and on-device weight preparation
// (per-output-row int8 codes, half conversion, reorders).
#include "kernels.cuh"

namespace dav2cuda {
namespace {

template <typename H>
__device__ __forceinline__ H cvt(float v);
template <>
__device__ __forceinline__ __half cvt<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <typename H>
__device__ __forceinline__ float tof(H v);
template <>
__device__ __forceinline__ float tof<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float tof<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float tof<float>(float v) { return v; }

unsigned gcap(uint64_t n) {
    const uint64_t g = (n + 255) / 256;
    return (unsigned)(g == 0 ? 1 : (g < 148 * 32 ? g : 148 * 32));
}

// Non-overlapping 14x14 patches of planar [B][3][H][W] images -> rows
// (img, py, px) with columns c*196 + ky*14 + kx (the Conv2d weight order),
// zero-padded to kp columns.
template <typename H>
__global__ void patch_im2col_kernel(H* __restrict__ out, const float* __restrict__ img, uint32_t h, uint32_t w,
                                    uint32_t kp, uint64_t rows) {
    const uint32_t pw = w / 14, ph = h / 14;
    const uint64_t n = rows * kp;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t r = i / kp;
        const uint32_t col = (uint32_t)(i % kp);
        float v = 0.f;
        if (col < 588) {
            const uint64_t b = r / ((uint64_t)pw * ph);
            const uint32_t p = (uint32_t)(r % ((uint64_t)pw * ph));
            const uint32_t py = p / pw, px = p % pw;
            const uint32_t c = col / 196, rem = col % 196;
            v = __ldg(img + ((b * 3 + c) * h + py * 14 + rem / 14) * w + px * 14 + rem % 14);
        }
        out[i] = cvt<H>(v);
    }
}

// position_bicubic.glsl:76-105 (a = -0.75, clamp to the 37x37 grid) with
// the scale rule of src/operators.cpp:1346-1364, written token-major:
// out[(py*pw + px)*D + f].
__device__ __forceinline__ float cc1(float x) {
    const float a = -0.75f;
    return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
}
__device__ __forceinline__ float cc2(float x) {
    const float a = -0.75f;
    return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a;
}
__device__ __forceinline__ float cubic_interp(float x0, float x1, float x2, float x3, float t) {
    return x0 * cc2(t + 1.0f) + x1 * cc1(t) + x2 * cc1(1.0f - t) + x3 * cc2((1.0f - t) + 1.0f);
}

__global__ void position_bicubic_kernel(float* __restrict__ out, const float* __restrict__ pos, uint32_t d,
                                        uint32_t pw, uint32_t ph, float sx, float sy) {
    const uint64_t n = (uint64_t)pw * ph * d;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t f = (uint32_t)(i % d);
        const uint32_t p = (uint32_t)(i / d);
        const uint32_t x = p % pw, y = p / pw;
        const float srcx = ((float)x + 0.5f) * sx - 0.5f;
        const float srcy = ((float)y + 0.5f) * sy - 0.5f;
        const int bx = (int)floorf(srcx), by = (int)floorf(srcy);
        const float tx = srcx - (float)bx, ty = srcy - (float)by;
        float rows[4];
        for (int k = 0; k < 4; ++k) {
            const int yy = min(max(by - 1 + k, 0), 36);
            float v[4];
            for (int j = 0; j < 4; ++j) {
                const int xx = min(max(bx - 1 + j, 0), 36);
                v[j] = __ldg(pos + (uint64_t)(1 + yy * 37 + xx) * d + f);
            }
            rows[k] = cubic_interp(v[0], v[1], v[2], v[3], tx);
        }
        out[i] = cubic_interp(rows[0], rows[1], rows[2], rows[3], ty);
    }
}

// tokens[img*T + 0] = cls + pos[0]; tokens[img*T + 1 + p] = pos_interp[p]
// (the patch GEMM then adds its result on top: add_position.glsl order).
__global__ void fill_tokens_kernel(float* __restrict__ x, const float* __restrict__ cls,
                                   const float* __restrict__ pos, const float* __restrict__ interp, uint32_t d,
                                   uint32_t tokens, uint64_t rows) {
    const uint64_t n = rows * d;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t f = (uint32_t)(i % d);
        const uint32_t t = (uint32_t)((i / d) % tokens);
        x[i] = t == 0 ? __ldg(cls + f) + __ldg(pos + f) : __ldg(interp + (uint64_t)(t - 1) * d + f);
    }
}

// Align-corners bilinear on channels-last 16-bit maps, 8 channels per thread,
// in the arithmetic of bilinear_align_true.glsl:27-63: source coordinate
// (x*(in-1))/(out-1), a*(1-f) + b*f with every product and sum rounded
// (horizontal first, then vertical), f32 math, the result rounded to the
// 16-bit type. A block per (image, source row pair k): it writes every output
// row whose top source row is k (the last pair also the rows on the last
// source row), so each horizontal lerp of the two source rows is computed
// once and shared by those rows (about oh/ih of them); the x table (source
// columns and weight) is computed once per block into shared memory; each
// thread keeps one 8-channel chunk and strides over the pixels (blockDim is a
// multiple of the chunk count).
__device__ __forceinline__ float nhwc_coord(uint32_t o, uint32_t in, uint32_t out) {
    return out > 1 ? __fdiv_rn(__fmul_rn((float)o, (float)(in - 1)), (float)(out - 1)) : 0.f;
}

// source row pair of output row y: its top source row, the last source row
// folded into the last pair (monotone in y)
__device__ __forceinline__ uint32_t nhwc_row_pair(uint32_t y, uint32_t ih, uint32_t oh, uint32_t pairs) {
    return min((uint32_t)floorf(nhwc_coord(y, ih, oh)), pairs - 1);
}

constexpr uint32_t kNhwcRowsMax = 4;  // output rows per pass over a staged pair

template <typename H>
__global__ void __launch_bounds__(256) bilinear_nhwc_kernel(H* __restrict__ out, const H* __restrict__ in,
                                                            uint32_t ih, uint32_t iw, uint32_t oh, uint32_t ow,
                                                            uint32_t c) {
    extern __shared__ uint32_t xtab[];  // [ow][3]: x0*c, x1*c, fx bits
    const uint32_t cv = c / 8;
    const uint32_t pairs = ih > 1 ? ih - 1 : 1;
    const uint32_t k = blockIdx.x % pairs, b = blockIdx.x / pairs;
    for (uint32_t x = threadIdx.x; x < ow; x += blockDim.x) {
        const float sxf = nhwc_coord(x, iw, ow);
        const uint32_t x0 = (uint32_t)floorf(sxf);
        const uint32_t x1 = min(x0 + 1, iw - 1);
        xtab[3 * x] = x0 * c;
        xtab[3 * x + 1] = x1 * c;
        xtab[3 * x + 2] = __float_as_uint(__fsub_rn(sxf, (float)x0));
    }
    // output rows of this pair: [y_lo, y_hi)
    const uint64_t y_est = (uint64_t)k * (oh - 1) / pairs;  // within a few rows of the first one
    uint32_t y_lo = (uint32_t)(y_est < oh ? y_est : oh - 1);
    while (y_lo > 0 && nhwc_row_pair(y_lo - 1, ih, oh, pairs) >= k) --y_lo;
    while (y_lo < oh && nhwc_row_pair(y_lo, ih, oh, pairs) < k) ++y_lo;
    uint32_t y_hi = y_lo;
    while (y_hi < oh && nhwc_row_pair(y_hi, ih, oh, pairs) == k) ++y_hi;
    const uint32_t r0 = k, r1 = min(k + 1, ih - 1);
    const H* s0 = in + ((uint64_t)b * ih + r0) * iw * c;
    const H* s1 = in + ((uint64_t)b * ih + r1) * iw * c;
    const uint32_t cc = (threadIdx.x % cv) * 8;
    const uint32_t step = blockDim.x / cv;
    __syncthreads();
    for (uint32_t yc = y_lo; yc < y_hi; yc += kNhwcRowsMax) {
        const uint32_t nr = min(kNhwcRowsMax, y_hi - yc);
        float fy[kNhwcRowsMax], gy[kNhwcRowsMax];
        bool top1[kNhwcRowsMax], bot1[kNhwcRowsMax];  // top / bottom source row is r1 (else r0)
#pragma unroll
        for (uint32_t j = 0; j < kNhwcRowsMax; ++j) {
            const float syf = nhwc_coord(yc + j, ih, oh);
            const uint32_t y0 = (uint32_t)floorf(syf), y1 = min(y0 + 1, ih - 1);
            fy[j] = __fsub_rn(syf, (float)y0);
            gy[j] = __fsub_rn(1.0f, fy[j]);
            top1[j] = y0 != r0;
            bot1[j] = y1 != r0;
        }
        bool plain = true;  // every row of the pass: top r0, bottom r1
#pragma unroll
        for (uint32_t j = 0; j < kNhwcRowsMax; ++j) plain = plain && (j >= nr || (!top1[j] && bot1[j]));
        H* o = out + ((uint64_t)b * oh + yc) * ow * c;
        for (uint32_t x = threadIdx.x / cv; x < ow; x += step) {
            const uint32_t o0 = xtab[3 * x] + cc, o1 = xtab[3 * x + 1] + cc;
            const float fx = __uint_as_float(xtab[3 * x + 2]), gx = __fsub_rn(1.0f, fx);
            const uint4 a00 = *reinterpret_cast<const uint4*>(s0 + o0);
            const uint4 a01 = *reinterpret_cast<const uint4*>(s0 + o1);
            const uint4 a10 = *reinterpret_cast<const uint4*>(s1 + o0);
            const uint4 a11 = *reinterpret_cast<const uint4*>(s1 + o1);
            const H* h00 = reinterpret_cast<const H*>(&a00);
            const H* h01 = reinterpret_cast<const H*>(&a01);
            const H* h10 = reinterpret_cast<const H*>(&a10);
            const H* h11 = reinterpret_cast<const H*>(&a11);
            float hz0[8], hz1[8];  // horizontal lerps of source rows r0 and r1
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                hz0[j] = __fadd_rn(__fmul_rn(tof(h00[j]), gx), __fmul_rn(tof(h01[j]), fx));
                hz1[j] = __fadd_rn(__fmul_rn(tof(h10[j]), gx), __fmul_rn(tof(h11[j]), fx));
            }
#pragma unroll
            for (uint32_t r = 0; r < kNhwcRowsMax; ++r) {
                if (r < nr) {
                    uint4 res;
                    H* rr = reinterpret_cast<H*>(&res);
                    if (plain) {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            rr[j] = cvt<H>(__fadd_rn(__fmul_rn(hz0[j], gy[r]), __fmul_rn(hz1[j], fy[r])));
                    } else {
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float top = top1[r] ? hz1[j] : hz0[j], bot = bot1[r] ? hz1[j] : hz0[j];
                            rr[j] = cvt<H>(__fadd_rn(__fmul_rn(top, gy[r]), __fmul_rn(bot, fy[r])));
                        }
                    }
                    *reinterpret_cast<uint4*>(o + ((uint64_t)r * ow + x) * c + cc) = res;
                }
            }
        }
    }
}

// im2col-quantize of a channels-last half map (the stride-2 resize layer in
// the int8 path): row = output pixel, columns in (ky, kx, c) order — the
// reference's (c, ky, kx) order with the weight columns permuted alike, which
// leaves every row scale, every code and every integer dot product
// unchanged. Row scale = max(absmax/127, 1e-8), code = rint(x*(1/scale)).
template <typename H>
__global__ void __launch_bounds__(256) im2col_quantize_nhwc_kernel(uint8_t* __restrict__ out,
                                                                   float* __restrict__ scales,
                                                                   const H* __restrict__ in, uint32_t h,
                                                                   uint32_t w, uint32_t c, uint32_t ldc,
                                                                   uint32_t k, uint32_t s, uint32_t pad,
                                                                   uint32_t oh, uint32_t ow, uint32_t kp) {
    __shared__ float red[8];
    const uint64_t r = blockIdx.x;
    const uint64_t b = r / ((uint64_t)oh * ow);
    const uint32_t pp = (uint32_t)(r % ((uint64_t)oh * ow));
    const uint32_t oy = pp / ow, ox = pp % ow;
    const uint32_t cols = k * k * c;
    auto value = [&](uint32_t col) -> float {
        const uint32_t tap = col / c, ch = col % c;
        const int iy = (int)(oy * s + tap / k) - (int)pad, ix = (int)(ox * s + tap % k) - (int)pad;
        if (iy < 0 || ix < 0 || iy >= (int)h || ix >= (int)w) return 0.f;
        return tof(in[((b * h + iy) * w + ix) * ldc + ch]);
    };
    float m = 0.f;
    for (uint32_t col = threadIdx.x; col < cols; col += 256) m = fmaxf(m, fabsf(value(col)));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t = fmaxf(t, red[i]);
        red[0] = fmaxf(t / 127.0f, 1.0e-8f);
        scales[r] = red[0];
    }
    __syncthreads();
    const float inv = 1.0f / red[0];
    for (uint32_t col = threadIdx.x; col < kp; col += 256)
        out[r * kp + col] = col < cols ? (uint8_t)q8(__fmul_rn(value(col), inv)) : 0;
}

// Eight consecutive channels as floats: one 16-byte load for half maps, two
// for f32 maps.
template <typename H>
__device__ __forceinline__ void load8(const H* p, float (&f)[8]) {
    const uint4 q = *reinterpret_cast<const uint4*>(p);
    const H* hv = reinterpret_cast<const H*>(&q);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = tof(hv[j]);
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float (&f)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Vectorised form of the same for 8-aligned channels: each thread holds up to
// VEC groups of 8 channels of one tap in registers, so the row is gathered
// once; codes and padding as above.
template <typename H, int VEC>
__global__ void __launch_bounds__(256) im2col_quantize_nhwc_vec_kernel(uint8_t* __restrict__ out,
                                                                       float* __restrict__ scales,
                                                                       const H* __restrict__ in, uint32_t h,
                                                                       uint32_t w, uint32_t c, uint32_t ldc,
                                                                       uint32_t k, uint32_t s, uint32_t pad,
                                                                       uint32_t oh, uint32_t ow, uint32_t kp) {
    __shared__ float red[8];
    const uint64_t r = blockIdx.x;
    const uint64_t b = r / ((uint64_t)oh * ow);
    const uint32_t pp = (uint32_t)(r % ((uint64_t)oh * ow));
    const uint32_t oy = pp / ow, ox = pp % ow;
    const uint32_t cg = c / 8, groups = k * k * cg;
    float v[VEC][8];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        const uint32_t g = threadIdx.x + 256u * i;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
        if (g < groups) {
            const uint32_t tap = g / cg, ch = (g % cg) * 8;
            const int iy = (int)(oy * s + tap / k) - (int)pad, ix = (int)(ox * s + tap % k) - (int)pad;
            if (iy >= 0 && ix >= 0 && iy < (int)h && ix < (int)w) load8(in + ((b * h + iy) * w + ix) * ldc + ch, v[i]);
#pragma unroll
            for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[i][j]));
        }
    }
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t = fmaxf(t, red[i]);
    const float scale = fmaxf(t / 127.0f, 1.0e-8f);
    if (threadIdx.x == 0) scales[r] = scale;
    const float inv = 1.0f / scale;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        const uint32_t g = threadIdx.x + 256u * i;
        if (g < groups) {
            uint32_t q[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) q[j] = q8(__fmul_rn(v[i][j], inv));
            *reinterpret_cast<uint2*>(out + r * kp + 8ull * g) =
                make_uint2(q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24), q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24));
        }
    }
    for (uint32_t col = groups * 8 + threadIdx.x; col < kp; col += 256) out[r * kp + col] = 0;
}

// Per-output-row int8 weight codes (src/gpu_model.cpp:207-284): scale =
// max(absmax/127, 1e-8), code = nearbyint(clamp(w/scale)). Source element
// of (row, col) per layout:
//   kind 0: w[row*K + col]                          (linear / conv, c-major)
//   kind 1: conv-transpose [Ci][Co][k][k]: row = (ky*k+kx)*Co + co, col = ci
//   kind 2: conv [Co][Ci][k][k] with columns reordered to (ky, kx, ci)
__device__ __forceinline__ float weight_at(const float* w, int kind, uint64_t row, uint32_t col, uint32_t K,
                                           uint32_t co, uint32_t k, uint32_t ci) {
    if (kind == 0) return w[row * K + col];
    if (kind == 1) {
        const uint32_t kk = (uint32_t)(row / co), o = (uint32_t)(row % co);
        return w[(((uint64_t)col * co + o) * k + kk / k) * k + kk % k];
    }
    const uint32_t tap = col / ci, c = col % ci;
    return w[((row * ci + c) * k + tap / k) * k + tap % k];
}

__global__ void __launch_bounds__(256) pack_weight_s8_kernel(uint8_t* __restrict__ out, float* __restrict__ scales,
                                                             const float* __restrict__ w, int kind, uint32_t K,
                                                             uint32_t kp, uint32_t co, uint32_t k, uint32_t ci) {
    __shared__ float red[8];
    const uint64_t row = blockIdx.x;
    float m = 0.f;
    for (uint32_t col = threadIdx.x; col < K; col += 256) m = fmaxf(m, fabsf(weight_at(w, kind, row, col, K, co, k, ci)));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < 8; ++i) t = fmaxf(t, red[i]);
        red[0] = fmaxf(t / 127.0f, 1.0e-8f);
        scales[row] = red[0];
    }
    __syncthreads();
    const float scale = red[0];
    for (uint32_t col = threadIdx.x; col < kp; col += 256)
        out[row * kp + col] = col < K ? (uint8_t)q8(weight_at(w, kind, row, col, K, co, k, ci) / scale) : 0;
}

// Half weights in the same three layouts (kind 2 pads channels to cip).
template <typename H>
__global__ void half_weight_kernel(H* __restrict__ out, const float* __restrict__ w, int kind, uint64_t rows,
                                   uint32_t K, uint32_t kp, uint32_t co, uint32_t k, uint32_t ci, uint32_t cip) {
    const uint64_t n = rows * kp;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t row = i / kp;
        const uint32_t col = (uint32_t)(i % kp);
        float v = 0.f;
        if (kind == 2) {
            const uint32_t tap = col / cip, c = col % cip;
            if (tap < k * k && c < ci) v = w[((row * ci + c) * k + tap / k) * k + tap % k];
        } else if (col < K) {
            v = weight_at(w, kind, row, col, K, co, k, ci);
        }
        out[i] = cvt<H>(v);
    }
}

__global__ void expand_bias_kernel(float* __restrict__ out, const float* __restrict__ bias, uint32_t co,
                                   uint32_t reps) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < co * reps) out[i] = bias[i % co];
}

__global__ void store_pointer_kernel(void** slot, void* value) { *slot = value; }

}  // namespace

int launch_store_pointer(void** slot, void* value, cudaStream_t st) {
    store_pointer_kernel<<<1, 1, 0, st>>>(slot, value);
    return check_launch("store_pointer");
}

template <typename H>
int launch_patch_im2col(H* out, const float* img, uint32_t batch, uint32_t h, uint32_t w, uint32_t kp,
                        cudaStream_t st) {
    const uint64_t rows = (uint64_t)batch * (h / 14) * (w / 14);
    patch_im2col_kernel<H><<<gcap(rows * kp), 256, 0, st>>>(out, img, h, w, kp, rows);
    return check_launch("patch_im2col");
}

int launch_position_bicubic(float* out, const float* pos, uint32_t d, uint32_t pw, uint32_t ph, cudaStream_t st) {
    const bool same = pw == 37 && ph == 37;
    const float sx = same ? 1.0f : (float)(1.0 / (((double)pw + 0.1) / 37.0));
    const float sy = same ? 1.0f : (float)(1.0 / (((double)ph + 0.1) / 37.0));
    position_bicubic_kernel<<<gcap((uint64_t)pw * ph * d), 256, 0, st>>>(out, pos, d, pw, ph, sx, sy);
    return check_launch("position_bicubic");
}

int launch_fill_tokens(float* x, const float* cls, const float* pos, const float* interp, uint32_t d,
                       uint32_t tokens, uint32_t batch, cudaStream_t st) {
    const uint64_t rows = (uint64_t)batch * tokens;
    fill_tokens_kernel<<<gcap(rows * d), 256, 0, st>>>(x, cls, pos, interp, d, tokens, rows);
    return check_launch("fill_tokens");
}

template <typename H>
int launch_bilinear_nhwc(H* out, const H* in, uint32_t batch, uint32_t ih, uint32_t iw, uint32_t oh, uint32_t ow,
                         uint32_t c, cudaStream_t st) {
    if (c % 8) return set_error(DAV2CUDA_INVALID_ARGUMENT, "bilinear_nhwc: channels % 8");
    const uint32_t cv = c / 8;
    if (cv == 0 || cv > 256) return set_error(DAV2CUDA_INVALID_ARGUMENT, "bilinear_nhwc: channels must be 8..2048");
    const size_t tab = (size_t)ow * 3 * sizeof(uint32_t);
    if (tab > 48 * 1024) return set_error(DAV2CUDA_INVALID_ARGUMENT, "bilinear_nhwc: output row too wide");
    const uint64_t blocks = (uint64_t)batch * (ih > 1 ? ih - 1 : 1);
    if (blocks > 0x7fffffffull) return set_error(DAV2CUDA_INVALID_ARGUMENT, "bilinear_nhwc: grid too large");
    bilinear_nhwc_kernel<H><<<(unsigned)blocks, (256 / cv) * cv, tab, st>>>(out, in, ih, iw, oh, ow, c);
    return check_launch("bilinear_nhwc");
}

template <typename H>
int launch_im2col_quantize_nhwc(uint8_t* out, float* scales, const H* in, uint32_t batch, uint32_t h, uint32_t w,
                                uint32_t c, uint32_t ldc, uint32_t k, uint32_t s, uint32_t pad, uint32_t oh,
                                uint32_t ow, uint32_t kp, cudaStream_t st) {
    const uint64_t rows = (uint64_t)batch * oh * ow;
    const uint32_t groups = k * k * (c / 8);
    if (c % 8 == 0 && ldc % 8 == 0 && kp % 8 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0 &&
        reinterpret_cast<uintptr_t>(out) % 8 == 0 && groups <= 8 * 256) {
        const int vec = (int)((groups + 255) / 256);
#define DAV2_IM2COL_VEC(V)                                                                                   \
    case V:                                                                                                  \
        im2col_quantize_nhwc_vec_kernel<H, V><<<(unsigned)rows, 256, 0, st>>>(out, scales, in, h, w, c, ldc, k, s, \
                                                                              pad, oh, ow, kp);              \
        break;
        switch (vec) {
            DAV2_IM2COL_VEC(1)
            DAV2_IM2COL_VEC(2)
            DAV2_IM2COL_VEC(3)
            DAV2_IM2COL_VEC(4)
            DAV2_IM2COL_VEC(5)
            DAV2_IM2COL_VEC(6)
            DAV2_IM2COL_VEC(7)
            default: DAV2_IM2COL_VEC(8)
        }
#undef DAV2_IM2COL_VEC
        return check_launch("im2col_quantize_nhwc");
    }
    im2col_quantize_nhwc_kernel<H><<<(unsigned)rows, 256, 0, st>>>(out, scales, in, h, w, c, ldc, k, s, pad, oh, ow,
                                                                    kp);
    return check_launch("im2col_quantize_nhwc");
}

int launch_pack_weight_s8(uint8_t* out, float* scales, const float* w, int kind, uint64_t rows, uint32_t K,
                          uint32_t kp, uint32_t co, uint32_t k, uint32_t ci, cudaStream_t st) {
    pack_weight_s8_kernel<<<(unsigned)rows, 256, 0, st>>>(out, scales, w, kind, K, kp, co, k, ci);
    return check_launch("pack_weight_s8");
}

template <typename H>
int launch_half_weight(H* out, const float* w, int kind, uint64_t rows, uint32_t K, uint32_t kp, uint32_t co,
                       uint32_t k, uint32_t ci, uint32_t cip, cudaStream_t st) {
    half_weight_kernel<H><<<gcap(rows * kp), 256, 0, st>>>(out, w, kind, rows, K, kp, co, k, ci, cip);
    return check_launch("half_weight");
}

int launch_expand_bias(float* out, const float* bias, uint32_t co, uint32_t reps, cudaStream_t st) {
    expand_bias_kernel<<<(co * reps + 255) / 256, 256, 0, st>>>(out, bias, co, reps);
    return check_launch("expand_bias");
}

#define DAV2_INST(H)                                                                                            \
    template int launch_patch_im2col<H>(H*, const float*, uint32_t, uint32_t, uint32_t, uint32_t, cudaStream_t); \
    template int launch_bilinear_nhwc<H>(H*, const H*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,       \
                                         uint32_t, cudaStream_t);                                               \
    template int launch_im2col_quantize_nhwc<H>(uint8_t*, float*, const H*, uint32_t, uint32_t, uint32_t,      \
                                                uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,     \
                                                uint32_t, uint32_t, cudaStream_t);                              \
    template int launch_half_weight<H>(H*, const float*, int, uint64_t, uint32_t, uint32_t, uint32_t, uint32_t, \
                                       uint32_t, uint32_t, cudaStream_t);
DAV2_INST(__half)
DAV2_INST(__nv_bfloat16)
#undef DAV2_INST
template int launch_im2col_quantize_nhwc<float>(uint8_t*, float*, const float*, uint32_t, uint32_t, uint32_t,
                                                uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                                                uint32_t, uint32_t, cudaStream_t);

}  // namespace dav2cuda
