// Bandwidth-bound kernels of the operator layer: LayerNorm (plain and fused
// with row quantization), exact GELU, row softmax, LayerScale/residual adds,
// align-corners bilinear, min-max normalization, image preprocessing and the
// int8 row / im2col quantizers. Layouts follow the reference operators
// (src/operators.cpp); each kernel names the shader whose arithmetic it
// reproduces.
#include "kernels.cuh"

#include <algorithm>
#include <cfloat>

namespace dav2cuda {

namespace {

constexpr int kBlock = 256;

__device__ __forceinline__ float gelu_erf(float v) {
    // torch.nn.GELU (exact erf), which gelu.glsl approximates to ~1.2e-7.
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ------------------------------------------------------------- LayerNorm
// layer_norm.glsl:27-67: mean = sum/n; var = max(sumsq/n - mean^2, 0);
// y = (x - mean) * rsqrt(var + eps) * w + b. One warp per row; the row is
// held in registers (VPL float4 per lane) so the input is read once.
// Output row o reads input row (o / out_group) * in_group + in_offset +
// o % out_group, which lets the encoder taps drop the class-token row.
// Output kinds: f32, f16 or bf16 values, or int8 codes + per-row scale
// (the fused form of layer_norm followed by quantize_rows_int8_fused.glsl).
enum LnOut { kLnF32 = 0, kLnF16 = 1, kLnBF16 = 2, kLnS8 = 3 };

template <int VPL, int OUT>
__global__ void __launch_bounds__(256) layer_norm_warp_kernel(
    void* __restrict__ out, float* __restrict__ out_scales, const float* __restrict__ in,
    const float* __restrict__ w, const float* __restrict__ b, uint32_t rows, uint32_t cols, float eps,
    uint32_t out_group, uint32_t in_group, uint32_t in_offset) {
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const uint64_t in_row = (uint64_t)(warp / out_group) * in_group + in_offset + warp % out_group;
    const float4* x4 = reinterpret_cast<const float4*>(in + in_row * cols);
    const uint32_t n4 = cols >> 2;
    float4 v[VPL];
    float s = 0.f, q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < n4) {
            v[i] = __ldg(x4 + c);
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
            q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
        } else {
            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    s = warp_sum(s);
    q = warp_sum(q);
    const float n = fmaxf((float)cols, 1.0f);
    const float mean = s / n;
    const float var = fmaxf(q / n - mean * mean, 0.0f);
    const float inv = 1.0f / sqrtf(var + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < n4) {
            const float4 ww = __ldg(w4 + c), bb = __ldg(b4 + c);
            v[i].x = (v[i].x - mean) * inv * ww.x + bb.x;
            v[i].y = (v[i].y - mean) * inv * ww.y + bb.y;
            v[i].z = (v[i].z - mean) * inv * ww.z + bb.z;
            v[i].w = (v[i].w - mean) * inv * ww.w + bb.w;
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
        }
    }
    const uint64_t orow = warp;
    if constexpr (OUT == kLnS8) {
        amax = warp_max(amax);
        const float scale = fmaxf(amax / 127.0f, 1.0e-8f);
        const float rs = __frcp_rn(scale);
        if (lane == 0) out_scales[orow] = scale;
        uint32_t* o = reinterpret_cast<uint32_t*>(out) + orow * n4;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint32_t c = lane + 32u * i;
            if (c < n4)
                o[c] = q8x4_quot(v[i].x, v[i].y, v[i].z, v[i].w, scale, rs);
        }
    } else if constexpr (OUT == kLnF32) {
        float4* o = reinterpret_cast<float4*>(out) + orow * n4;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint32_t c = lane + 32u * i;
            if (c < n4) o[c] = v[i];
        }
    } else {
        using H = typename std::conditional<OUT == kLnF16, __half, __nv_bfloat16>::type;
        uint2* o = reinterpret_cast<uint2*>(out) + orow * n4;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const uint32_t c = lane + 32u * i;
            if (c < n4) {
                H h[4] = {from_f<H>(v[i].x), from_f<H>(v[i].y), from_f<H>(v[i].z), from_f<H>(v[i].w)};
                o[c] = *reinterpret_cast<uint2*>(h);
            }
        }
    }
}

// Generic LayerNorm for column counts the register path does not cover:
// one 64-thread block per row, lane-strided partial sums exactly as the
// shader, two reads of the row.
__global__ void layer_norm_generic_kernel(float* __restrict__ out, const float* __restrict__ in,
                                          const float* __restrict__ w, const float* __restrict__ b,
                                          uint32_t cols, float eps) {
    __shared__ float ps[64], pq[64];
    const uint64_t row = blockIdx.x;
    const float* x = in + row * cols;
    float s = 0.f, q = 0.f;
    for (uint32_t c = threadIdx.x; c < cols; c += 64) {
        const float v = x[c];
        s += v;
        q += v * v;
    }
    ps[threadIdx.x] = s;
    pq[threadIdx.x] = q;
    __syncthreads();
    for (int width = 32; width > 0; width >>= 1) {
        if ((int)threadIdx.x < width) {
            ps[threadIdx.x] += ps[threadIdx.x + width];
            pq[threadIdx.x] += pq[threadIdx.x + width];
        }
        __syncthreads();
    }
    const float n = fmaxf((float)cols, 1.0f);
    const float mean = ps[0] / n;
    const float var = fmaxf(pq[0] / n - mean * mean, 0.0f);
    const float inv = 1.0f / sqrtf(var + eps);
    for (uint32_t c = threadIdx.x; c < cols; c += 64) out[row * cols + c] = (x[c] - mean) * inv * w[c] + b[c];
}

// ------------------------------------------------------------ elementwise
__global__ void gelu_kernel(float* __restrict__ out, const float* __restrict__ in, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t n4 = n >> 2;
    const float4* i4 = reinterpret_cast<const float4*>(in);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 v = __ldcs(i4 + i);
        v.x = gelu_erf(v.x);
        v.y = gelu_erf(v.y);
        v.z = gelu_erf(v.z);
        v.w = gelu_erf(v.w);
        __stcs(o4 + i, v);
    }
    for (uint64_t i = (n4 << 2) + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = gelu_erf(in[i]);
}

// add_scaled.glsl is declared `precise`: product and sum are rounded
// separately (no FMA contraction).
__global__ void add_scaled_kernel(float* __restrict__ out, const float* __restrict__ res,
                                  const float* __restrict__ add, const float* __restrict__ scale, uint64_t n,
                                  uint32_t cols) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __fadd_rn(res[i], __fmul_rn(add[i], __ldg(scale + i % cols)));
}

__global__ void relu_kernel(float* __restrict__ out, const float* __restrict__ in, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = fmaxf(in[i], 0.0f);
}

__global__ void add_kernel(float* __restrict__ out, const float* __restrict__ a, const float* __restrict__ b,
                           uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = a[i] + b[i];
}

__global__ void sigmoid_scale_kernel(float* __restrict__ out, const float* __restrict__ in, uint64_t n,
                                     float s) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = s / (1.0f + expf(-in[i]));
}

// ---------------------------------------------------------------- softmax
// softmax_lastdim.glsl:19-69 on input*scale: max, exp(v - max), sum,
// multiply by 1/max(sum, 1e-20). One warp per row, the row kept in
// registers (MAXV float2 per lane), so each element is read and written
// exactly once.
// exp(x) as 2^(x*log2e) on the exponential unit (relative error ~2^-22).
__device__ __forceinline__ float exp_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
    return y;
}

// softmax_lastdim.glsl:19-69: row max of x*scale, exp(x*scale - max), sum,
// normalize. One warp per row, the row held in registers (read once,
// written once); the register budget is capped at three 256-thread blocks
// per SM so that 24 warps (24 rows) per SM keep loads in flight.
template <int MAXV>
__global__ void __launch_bounds__(256, MAXV <= 24 ? 3 : 1) softmax_warp_kernel(float* __restrict__ out, const float* __restrict__ in,
                                                              uint64_t rows, uint32_t cols, float scale) {
    const uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float2* x2 = reinterpret_cast<const float2*>(in + warp * cols);
    float2* y2 = reinterpret_cast<float2*>(out + warp * cols);
    const uint32_t n2 = cols >> 1;
    float2 v[MAXV];
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < n2) {
            v[i] = __ldcs(x2 + c);
            v[i].x *= scale;
            v[i].y *= scale;
            m = fmaxf(m, fmaxf(v[i].x, v[i].y));
        }
    }
    float tail = 0.f;
    const bool odd = (cols & 1u) && lane == 0;
    if (odd) {
        tail = in[warp * cols + cols - 1] * scale;
        m = fmaxf(m, tail);
    }
    m = warp_max(m);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < n2) {
            v[i].x = exp_fast(v[i].x - m);
            v[i].y = exp_fast(v[i].y - m);
            s += v[i].x + v[i].y;
        }
    }
    if (odd) {
        tail = exp_fast(tail - m);
        s += tail;
    }
    s = warp_sum(s);
    const float inv = 1.0f / fmaxf(s, 1.0e-20f);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const uint32_t c = lane + 32u * i;
        if (c < n2) __stcs(y2 + c, make_float2(v[i].x * inv, v[i].y * inv));
    }
    if (odd) out[warp * cols + cols - 1] = tail * inv;
}

// Generic row softmax (any width): one block per row, three passes.
__global__ void softmax_generic_kernel(float* __restrict__ out, const float* __restrict__ in, uint32_t cols,
                                       float scale) {
    __shared__ float red[32];
    const uint64_t row = blockIdx.x;
    const float* x = in + row * cols;
    float* y = out + row * cols;
    float m = -FLT_MAX;
    for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, x[c] * scale);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -FLT_MAX;
        t = warp_max(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    m = red[0];
    __syncthreads();
    float s = 0.f;
    for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) {
        const float e = expf(x[c] * scale - m);
        y[c] = e;
        s += e;
    }
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = 1.0f / fmaxf(red[0], 1.0e-20f);
    for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) y[c] *= inv;
}

// --------------------------------------------------------------- bilinear
// bilinear_align_true.glsl:27-63: src = (x*(in-1))/(out-1) in f32,
// x1 = min(x0+1, in-1), top/bottom lerps. Products and sums are rounded
// separately so the result equals the shader's written order.
__device__ __forceinline__ void align_coord(uint32_t o, uint32_t in, uint32_t out, uint32_t& i0, uint32_t& i1,
                                            float& f) {
    const float s = out > 1 ? __fdiv_rn(__fmul_rn((float)o, (float)(in - 1)), (float)(out - 1)) : 0.0f;
    i0 = (uint32_t)floorf(s);
    i1 = min(i0 + 1, in - 1);
    f = __fsub_rn(s, (float)i0);
}

__device__ __forceinline__ float lerp_rn(float a, float b, float f) {
    return __fadd_rn(__fmul_rn(a, __fsub_rn(1.0f, f)), __fmul_rn(b, f));
}

// Planar form for many planes: a thread per output column of one row walks
// a chunk of kPlanesPerBlock planes with its source columns and weights
// computed once, so the per-element work is four loads, the three lerps and
// one store with pointer increments.
constexpr uint32_t kPlanesPerBlock = 16;

template <typename TI, typename TO>
__global__ void __launch_bounds__(1024) bilinear_align_rows_kernel(TO* __restrict__ out, const TI* __restrict__ in,
                                                                   uint32_t iw, uint32_t ih, uint32_t ow, uint32_t oh,
                                                                   uint32_t planes) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y;
    if (x >= ow) return;
    uint32_t x0, x1, y0, y1;
    float fx, fy;
    align_coord(x, iw, ow, x0, x1, fx);
    align_coord(y, ih, oh, y0, y1, fy);
    const float gx = __fsub_rn(1.0f, fx), gy = __fsub_rn(1.0f, fy);
    const uint32_t c0 = blockIdx.z * kPlanesPerBlock;
    const uint32_t c1 = min(c0 + kPlanesPerBlock, planes);
    const uint64_t in_plane = (uint64_t)iw * ih, out_plane = (uint64_t)ow * oh;
    const TI* r0 = in + c0 * in_plane + (uint64_t)y0 * iw;
    const TI* r1 = in + c0 * in_plane + (uint64_t)y1 * iw;
    TO* o = out + c0 * out_plane + (uint64_t)y * ow + x;
#pragma unroll 4
    for (uint32_t c = c0; c < c1; ++c, r0 += in_plane, r1 += in_plane, o += out_plane) {
        // the shader's order: a*(1-f) + b*f, each product and sum rounded
        const float top = __fadd_rn(__fmul_rn(to_f(__ldg(r0 + x0)), gx), __fmul_rn(to_f(__ldg(r0 + x1)), fx));
        const float bot = __fadd_rn(__fmul_rn(to_f(__ldg(r1 + x0)), gx), __fmul_rn(to_f(__ldg(r1 + x1)), fx));
        *o = from_f<TO>(__fadd_rn(__fmul_rn(top, gy), __fmul_rn(bot, fy)));
    }
}

// Channels-last f32 [B][ih][iw][C] -> planar f32 [B][C][oh][ow] with the same
// align-corners arithmetic. A block per (image, 32 channels, source row pair
// k): it stages source rows k and k+1 of its channels ([2][iw][32] floats,
// each pixel one 128-byte line read as float4 by 8 lanes, every load of a
// thread issued before its first store) in shared memory with a 33-word
// pixel stride (conflict-free staging stores and reads), then writes every
// output row whose top source row is k (the last block also the rows on the
// last source row). Each horizontal lerp of a staged row is computed once and
// shared by all those output rows (about oh/ih of them), which halves the
// shared-memory reads of a 2x upsample. Warps take channels, lanes output
// columns: every output row leaves as coalesced stores from registers.
constexpr uint32_t kNhwcPixelWords = 33;
constexpr uint32_t kNhwcMaxSmem = 200 * 1024;
constexpr uint32_t kNhwcStageLoads = 8;  // float4 loads in flight per thread while staging

// block (source row pair) of output row y: its top source row, the last
// source row folded into the last pair
__device__ __forceinline__ uint32_t nhwc_pair_of(uint32_t y, uint32_t ih, uint32_t oh, uint32_t pairs) {
    uint32_t y0, y1;
    float fy;
    align_coord(y, ih, oh, y0, y1, fy);
    return min(y0, pairs - 1);
}

__global__ void __launch_bounds__(256, 4) bilinear_nhwc_to_planar_kernel(float* __restrict__ out,
                                                                         const float* __restrict__ in, uint32_t ih,
                                                                         uint32_t iw, uint32_t c, uint32_t oh,
                                                                         uint32_t ow) {
    extern __shared__ float src_rows[];  // [2][iw][kNhwcPixelWords]
    const uint32_t groups = c / 32, pairs = ih > 1 ? ih - 1 : 1;
    // consecutive blocks take consecutive row pairs of one channel group:
    // the blocks in flight write long runs of the same planes
    const uint32_t k = blockIdx.x % pairs;
    const uint32_t g = (blockIdx.x / pairs) % groups;
    const uint64_t b = blockIdx.x / ((uint64_t)groups * pairs);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t r0 = k, r1 = min(k + 1, ih - 1);
    // output rows of this pair: [y_lo, y_hi) (the pair index is monotone in y)
    const uint64_t y_est = (uint64_t)k * (oh - 1) / pairs;  // within a few rows of the first one
    uint32_t y_lo = (uint32_t)(y_est < oh ? y_est : oh - 1);
    while (y_lo > 0 && nhwc_pair_of(y_lo - 1, ih, oh, pairs) >= k) --y_lo;
    while (y_lo < oh && nhwc_pair_of(y_lo, ih, oh, pairs) < k) ++y_lo;
    uint32_t y_hi = y_lo;
    while (y_hi < oh && nhwc_pair_of(y_hi, ih, oh, pairs) == k) ++y_hi;
    if (y_lo >= y_hi) return;  // no output row on this pair (downsampling)

    const uint32_t per_row = iw * 8;  // float4s per staged row
    const float* base0 = in + ((b * ih + r0) * iw) * c + 32u * g;
    const float* base1 = in + ((b * ih + r1) * iw) * c + 32u * g;
    for (uint32_t i0 = threadIdx.x; i0 < 2 * per_row; i0 += kNhwcStageLoads * 256) {
        float4 v[kNhwcStageLoads];
#pragma unroll
        for (uint32_t j = 0; j < kNhwcStageLoads; ++j) {
            const uint32_t i = i0 + j * 256;
            if (i < 2 * per_row) {
                const uint32_t r = i >= per_row, rem = i - r * per_row;
                v[j] = __ldg(reinterpret_cast<const float4*>((r ? base1 : base0) + (uint64_t)(rem >> 3) * c) +
                             (rem & 7));
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < kNhwcStageLoads; ++j) {
            const uint32_t i = i0 + j * 256;
            if (i < 2 * per_row) {
                const uint32_t r = i >= per_row, rem = i - r * per_row;
                float* d = src_rows + (r * iw + (rem >> 3)) * kNhwcPixelWords + 4 * (rem & 7);
                d[0] = v[j].x;
                d[1] = v[j].y;
                d[2] = v[j].z;
                d[3] = v[j].w;
            }
        }
    }
    // x coordinates of the output columns, once per block
    uint32_t* tab_x = reinterpret_cast<uint32_t*>(src_rows + 2 * iw * kNhwcPixelWords);  // x0 | x1 << 16
    float* tab_f = reinterpret_cast<float*>(tab_x + ow);
    for (uint32_t x = threadIdx.x; x < ow; x += blockDim.x) {
        uint32_t x0, x1;
        float fx;
        align_coord(x, iw, ow, x0, x1, fx);
        tab_x[x] = x0 | (x1 << 16);
        tab_f[x] = fx;
    }
    __syncthreads();
    const float* s0 = src_rows;
    const float* s1 = src_rows + iw * kNhwcPixelWords;
    const uint64_t plane = (uint64_t)oh * ow;
    for (uint32_t yc = y_lo; yc < y_hi; yc += 2) {
        // two output rows per pass: vertical weights, and which staged row is
        // each one's top / bottom (rows 0 / 1 for all but the last pair)
        const bool two = yc + 1 < y_hi;
        uint32_t ya0, ya1, yb0 = r0, yb1 = r1;
        float fa, fb = 0.f;
        align_coord(yc, ih, oh, ya0, ya1, fa);
        if (two) align_coord(yc + 1, ih, oh, yb0, yb1, fb);
        const float ga = __fsub_rn(1.0f, fa), gb = __fsub_rn(1.0f, fb);
        const bool plain = ya0 == r0 && ya1 != r0 && yb0 == r0 && yb1 != r0;
        const bool ta = ya0 != r0, ba = ya1 != r0, tb = yb0 != r0, bb = yb1 != r0;
        // row pointers of the warp's four channels (warp + 8q)
        float* oa[4];
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) oa[q] = out + (b * c + 32u * g + warp + 8 * q) * plane + (uint64_t)yc * ow;
        const float* w0 = s0 + warp;
        const float* w1 = s1 + warp;
        for (uint32_t x = lane; x < ow; x += 32) {
            const uint32_t t = tab_x[x], o0 = (t & 0xffffu) * kNhwcPixelWords, o1 = (t >> 16) * kNhwcPixelWords;
            const float fx = tab_f[x], gx = __fsub_rn(1.0f, fx);
#pragma unroll
            for (uint32_t q = 0; q < 4; ++q) {
                // the shader's order: a*(1-f) + b*f, each product and sum rounded
                const float h0 = __fadd_rn(__fmul_rn(w0[o0 + 8 * q], gx), __fmul_rn(w0[o1 + 8 * q], fx));
                const float h1 = __fadd_rn(__fmul_rn(w1[o0 + 8 * q], gx), __fmul_rn(w1[o1 + 8 * q], fx));
                if (plain) {
                    oa[q][x] = __fadd_rn(__fmul_rn(h0, ga), __fmul_rn(h1, fa));
                    if (two) oa[q][x + ow] = __fadd_rn(__fmul_rn(h0, gb), __fmul_rn(h1, fb));
                } else {
                    oa[q][x] = __fadd_rn(__fmul_rn(ta ? h1 : h0, ga), __fmul_rn(ba ? h1 : h0, fa));
                    if (two) oa[q][x + ow] = __fadd_rn(__fmul_rn(tb ? h1 : h0, gb), __fmul_rn(bb ? h1 : h0, fb));
                }
            }
        }
    }
}

template <typename TI, typename TO>
__global__ void bilinear_align_kernel(TO* __restrict__ out, const TI* __restrict__ in, uint32_t iw, uint32_t ih,
                                      uint32_t ow, uint32_t oh, uint32_t planes) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y;
    if (x >= ow) return;
    uint32_t x0, x1, y0, y1;
    float fx, fy;
    align_coord(x, iw, ow, x0, x1, fx);
    align_coord(y, ih, oh, y0, y1, fy);
    for (uint32_t c = blockIdx.z; c < planes; c += gridDim.z) {
        const TI* src = in + (uint64_t)c * iw * ih;
        const float top = lerp_rn(to_f(src[(uint64_t)y0 * iw + x0]), to_f(src[(uint64_t)y0 * iw + x1]), fx);
        const float bot = lerp_rn(to_f(src[(uint64_t)y1 * iw + x0]), to_f(src[(uint64_t)y1 * iw + x1]), fx);
        out[((uint64_t)c * oh + y) * ow + x] = from_f<TO>(lerp_rn(top, bot, fy));
    }
}

// ---------------------------------------------------------------- min/max
__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Batched forms: image z (blockIdx.y of the reduction and normalization)
// covers in[z*n, z*n + n) and owns range slots [2z, 2z + 1].
__global__ void minmax_init_kernel(uint32_t* keys, uint32_t batch) {
    const uint32_t z = blockIdx.x * blockDim.x + threadIdx.x;
    if (z >= batch) return;
    keys[2 * z] = 0xffffffffu;  // +max key
    keys[2 * z + 1] = 0u;       // -max key
}

// reduce_minmax.glsl:10-33 as a grid-wide reduction: per-block warp
// reductions, then order-preserving integer atomics on the two range slots.
__global__ void minmax_reduce_kernel(uint32_t* keys, const float* __restrict__ in, uint64_t n) {
    in += (uint64_t)blockIdx.y * n;
    keys += 2u * blockIdx.y;
    float lo = INFINITY, hi = -INFINITY;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = __ldg(in + i);
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
    }
    lo = warp_min(lo);
    hi = warp_max(hi);
    if ((threadIdx.x & 31) == 0) {
        atomicMin(keys, order_key(lo));
        atomicMax(keys + 1, order_key(hi));
    }
}

__global__ void minmax_finish_kernel(uint32_t* keys, uint32_t batch) {
    const uint32_t z = blockIdx.x * blockDim.x + threadIdx.x;
    if (z >= batch) return;
    const float lo = order_value(keys[2 * z]);
    const float hi = order_value(keys[2 * z + 1]);
    reinterpret_cast<float*>(keys)[2 * z] = lo;
    reinterpret_cast<float*>(keys)[2 * z + 1] = hi;
}

// normalize_relative.glsl / normalize_metric.glsl (metric: maximum > 0).
__global__ void normalize_kernel(float* __restrict__ d, const float* __restrict__ range, uint64_t n,
                                 float maximum) {
    d += (uint64_t)blockIdx.y * n;
    range += 2u * blockIdx.y;
    const float lo = range[0];
    const float span = (maximum > 0.0f ? maximum : range[1]) - lo;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        d[i] = span > 1.0e-12f ? fminf(fmaxf((d[i] - lo) / span, 0.0f), 1.0f) : 0.0f;
}

// -------------------------------------------------------------- preprocess
__device__ __forceinline__ float cubic_w(int tap, float t) {
    const float a = -0.75f;
    float x;
    switch (tap) {
        case 0: x = t + 1.0f; return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a;
        case 1: x = t; return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
        case 2: x = 1.0f - t; return ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
        default: x = 2.0f - t; return ((a * x - 5.0f * a) * x + 8.0f * a) * x - 4.0f * a;
    }
}

__constant__ float c_mean[3] = {0.485f, 0.456f, 0.406f};
__constant__ float c_dev[3] = {0.229f, 0.224f, 0.225f};

// preprocess_rgba.glsl:53-108 (per output pixel, 16 taps per channel).
// Batched: image z = blockIdx.z reads px + z * img_stride and writes its own
// three planes.
__global__ void preprocess_u32_kernel(float* __restrict__ out, const uint32_t* __restrict__ px, uint32_t sw,
                                      uint32_t sh, uint32_t stride, uint32_t rgba, uint32_t dw, uint32_t dh,
                                      uint64_t img_stride) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y;
    if (x >= dw) return;
    px += (uint64_t)blockIdx.z * img_stride;
    out += (uint64_t)blockIdx.z * 3u * dw * dh;
    const float sx = ((float)x + 0.5f) * (float)sw / (float)dw - 0.5f;
    const float sy = ((float)y + 0.5f) * (float)sh / (float)dh - 0.5f;
    const int bx = (int)floorf(sx), by = (int)floorf(sy);
    const float fx = sx - (float)bx, fy = sy - (float)by;
    const uint64_t plane = (uint64_t)dw * dh;
    for (int ch = 0; ch < 3; ++ch) {
        const uint32_t shift = ch == 1 ? 8u : (rgba ? (ch == 0 ? 0u : 16u) : (ch == 0 ? 16u : 0u));
        float r = 0.0f;
        for (int ty = 0; ty < 4; ++ty) {
            const int iy = min(max(by - 1 + ty, 0), (int)sh - 1);
            float row = 0.0f;
            for (int tx = 0; tx < 4; ++tx) {
                const int ix = min(max(bx - 1 + tx, 0), (int)sw - 1);
                const uint32_t p = __ldg(px + (uint64_t)iy * stride + ix);
                row += (float)((p >> shift) & 255u) / 255.0f * cubic_w(tx, fx);
            }
            r += row * cubic_w(ty, fy);
        }
        out[ch * plane + (uint64_t)y * dw + x] = (r - c_mean[ch]) / c_dev[ch];
    }
}

// OpenCV-style bicubic of src/image.cpp:163-269 for BGR8 (float
// coefficients; the reference accumulates in double, here in float: the
// difference is far below the fp32 operator tolerance).
__device__ __forceinline__ void cv_coeffs(float x, float c[4]) {
    const float a = -0.75f;
    c[0] = ((a * (x + 1.0f) - 5.0f * a) * (x + 1.0f) + 8.0f * a) * (x + 1.0f) - 4.0f * a;
    c[1] = ((a + 2.0f) * x - (a + 3.0f)) * x * x + 1.0f;
    const float o = 1.0f - x;
    c[2] = ((a + 2.0f) * o - (a + 3.0f)) * o * o + 1.0f;
    c[3] = 1.0f - c[0] - c[1] - c[2];
}

__global__ void preprocess_bgr8_kernel(float* __restrict__ out, const uint8_t* __restrict__ bgr, uint32_t sw,
                                       uint32_t sh, uint64_t row_stride, uint64_t img_stride, uint32_t dw,
                                       uint32_t dh) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y;
    const uint32_t img = blockIdx.z;
    if (x >= dw) return;
    const double scale_x = (double)sw / dw, scale_y = (double)sh / dh;
    const float cx = (float)((x + 0.5) * scale_x - 0.5);
    const float cy = (float)((y + 0.5) * scale_y - 0.5);
    const int bx = (int)floorf(cx), by = (int)floorf(cy);
    float ax[4], ay[4];
    cv_coeffs(cx - (float)bx, ax);
    cv_coeffs(cy - (float)by, ay);
    const uint8_t* src = bgr + img * img_stride;
    float acc[3] = {0.f, 0.f, 0.f};
    for (int ty = 0; ty < 4; ++ty) {
        const int iy = min(max(by - 1 + ty, 0), (int)sh - 1);
        const uint8_t* row = src + (uint64_t)iy * row_stride;
        float h[3] = {0.f, 0.f, 0.f};
        for (int tx = 0; tx < 4; ++tx) {
            const int ix = min(max(bx - 1 + tx, 0), (int)sw - 1);
            const uint8_t* p = row + 3 * ix;
            h[0] += ((float)__ldg(p + 2) / 255.0f) * ax[tx];
            h[1] += ((float)__ldg(p + 1) / 255.0f) * ax[tx];
            h[2] += ((float)__ldg(p + 0) / 255.0f) * ax[tx];
        }
        acc[0] += h[0] * ay[ty];
        acc[1] += h[1] * ay[ty];
        acc[2] += h[2] * ay[ty];
    }
    const uint64_t plane = (uint64_t)dw * dh;
    float* o = out + (uint64_t)img * 3 * plane + (uint64_t)y * dw + x;
    for (int ch = 0; ch < 3; ++ch) o[ch * plane] = (acc[ch] - c_mean[ch]) / c_dev[ch];
}

// Bilinear (align_corners=False) square resize of BGR8 frames.
__device__ __forceinline__ void hp_coord(uint32_t d, uint32_t in, uint32_t out, uint32_t& i0, uint32_t& i1,
                                         float& l) {
    const float scale = (float)in / (float)out;
    float src = scale * ((float)d + 0.5f) - 0.5f;
    src = fmaxf(src, 0.0f);
    uint32_t a = (uint32_t)src;
    a = min(a, in - 1);
    i0 = a;
    i1 = a + (a < in - 1 ? 1u : 0u);
    l = src - (float)a;
}

__global__ void preprocess_bgr8_bilinear_kernel(float* __restrict__ out, const uint8_t* __restrict__ bgr,
                                                uint32_t sw, uint32_t sh, uint64_t row_stride,
                                                uint64_t img_stride, uint32_t dw, uint32_t dh) {
    const uint32_t x = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t y = blockIdx.y;
    const uint32_t img = blockIdx.z;
    if (x >= dw) return;
    uint32_t x0, x1, y0, y1;
    float lx, ly;
    hp_coord(x, sw, dw, x0, x1, lx);
    hp_coord(y, sh, dh, y0, y1, ly);
    const uint8_t* src = bgr + img * img_stride;
    const uint8_t* r0 = src + (uint64_t)y0 * row_stride;
    const uint8_t* r1 = src + (uint64_t)y1 * row_stride;
    const uint64_t plane = (uint64_t)dw * dh;
    float* o = out + (uint64_t)img * 3 * plane + (uint64_t)y * dw + x;
    for (int ch = 0; ch < 3; ++ch) {
        const int b = 2 - ch;
        const float v00 = __ldg(r0 + 3 * x0 + b) / 255.0f, v01 = __ldg(r0 + 3 * x1 + b) / 255.0f;
        const float v10 = __ldg(r1 + 3 * x0 + b) / 255.0f, v11 = __ldg(r1 + 3 * x1 + b) / 255.0f;
        const float top = v00 * (1.0f - lx) + v01 * lx;
        const float bot = v10 * (1.0f - lx) + v11 * lx;
        o[ch * plane] = ((top * (1.0f - ly) + bot * ly) - c_mean[ch]) / c_dev[ch];
    }
}

// ------------------------------------------------------------ quantizers
__device__ __forceinline__ float block_max_128(float v, float* red) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    const float r = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    __syncthreads();
    return r;
}

// quantize_rows_int8_fused.glsl:20-55: scale = max(absmax/127, 1e-8);
// code = rint(clamp(x/scale, -127, 127)). One 128-thread block per row.
// The input row o starts at input_offset + (o / group) * group_stride +
// (o % group) * row_stride, so token matrices can skip their class row and
// channel-padded maps can be read in place.
template <typename T>
__global__ void __launch_bounds__(128) quantize_rows_kernel(uint32_t* __restrict__ packed,
                                                            float* __restrict__ scales,
                                                            const T* __restrict__ in, uint32_t cols,
                                                            uint64_t offset, uint32_t group,
                                                            uint64_t group_stride, uint32_t row_stride,
                                                            uint32_t out_words) {
    __shared__ float red[4];
    const uint64_t row = blockIdx.x;
    const T* x = in + offset + (row / group) * group_stride + (row % group) * (uint64_t)row_stride;
    float m = 0.f;
    for (uint32_t c = threadIdx.x; c < cols; c += 128) m = fmaxf(m, fabsf(to_f(x[c])));
    m = block_max_128(m, red);
    const float scale = fmaxf(m / 127.0f, 1.0e-8f);
    const float rs = __frcp_rn(scale);
    if (threadIdx.x == 0) scales[row] = scale;
    const uint32_t words = cols >> 2;
    uint32_t* o = packed + row * out_words;
    for (uint32_t w = threadIdx.x; w < out_words; w += 128) {
        uint32_t word = 0;
        if (w < words) {
            word = q8x4_quot(to_f(x[4 * w]), to_f(x[4 * w + 1]), to_f(x[4 * w + 2]), to_f(x[4 * w + 3]), scale, rs);
        }
        o[w] = word;
    }
}

// Eight consecutive row elements (one 16-byte load for half rows, two for
// f32 rows) as floats; streaming loads (each row is read once).
template <typename T>
__device__ __forceinline__ void load8_cs(const T* p, float (&f)[8]);
template <>
__device__ __forceinline__ void load8_cs<__half>(const __half* p, float (&f)[8]) {
    const uint4 q = __ldcs(reinterpret_cast<const uint4*>(p));
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 t = __half22float2(h[j]);
        f[2 * j] = t.x;
        f[2 * j + 1] = t.y;
    }
}
template <>
__device__ __forceinline__ void load8_cs<float>(const float* p, float (&f)[8]) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
    const float4 b = __ldcs(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Register-resident form of the same quantizer for f16 or f32 rows whose
// width is a multiple of 1024: each of the 128 threads holds VEC groups of 8
// values (16- or 32-byte loads), so the row is read from HBM once and its
// codes written once.
template <typename T, int VEC>
__global__ void __launch_bounds__(128) quantize_rows_vec_kernel(uint32_t* __restrict__ packed,
                                                                float* __restrict__ scales,
                                                                const T* __restrict__ in, uint32_t cols,
                                                                uint32_t row_stride, uint32_t out_words) {
    __shared__ float red[4];
    const uint64_t row = blockIdx.x;
    const T* x = in + row * (uint64_t)row_stride;
    float v[VEC][8];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        load8_cs<T>(x + 8u * (threadIdx.x + 128u * i), v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[i][j]));
    }
    m = block_max_128(m, red);
    const float scale = fmaxf(m / 127.0f, 1.0e-8f);
    const float rs = __frcp_rn(scale);
    if (threadIdx.x == 0) scales[row] = scale;
    uint2* o = reinterpret_cast<uint2*>(packed + row * out_words);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
        uint2 w;
        w.x = q8x4_quot(v[i][0], v[i][1], v[i][2], v[i][3], scale, rs);
        w.y = q8x4_quot(v[i][4], v[i][5], v[i][6], v[i][7], scale, rs);
        o[threadIdx.x + 128 * i] = w;
    }
}

// Warp-per-row form for f16 / f32 rows of 256*VPL columns (VPL <= 8): each
// lane holds VPL groups of 8 values, the row maximum is a shuffle reduction,
// and a 128-thread block quantizes four rows (no block barrier).
template <typename T, int VPL>
__global__ void __launch_bounds__(128) quantize_rows_warp_kernel(uint32_t* __restrict__ packed,
                                                                 float* __restrict__ scales,
                                                                 const T* __restrict__ in, uint64_t rows,
                                                                 uint32_t row_stride, uint32_t out_words) {
    const uint64_t row = (uint64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const uint32_t lane = threadIdx.x & 31;
    if (row >= rows) return;
    const T* x = in + row * (uint64_t)row_stride;
    float v[VPL][8];
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        load8_cs<T>(x + 8u * (lane + 32u * i), v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[i][j]));
    }
    m = warp_max(m);
    const float scale = fmaxf(m / 127.0f, 1.0e-8f);
    const float rs = __frcp_rn(scale);
    if (lane == 0) scales[row] = scale;
    uint2* o = reinterpret_cast<uint2*>(packed + row * out_words);
#pragma unroll
    for (int i = 0; i < VPL; ++i)
        o[lane + 32 * i] = make_uint2(q8x4_quot(v[i][0], v[i][1], v[i][2], v[i][3], scale, rs),
                                      q8x4_quot(v[i][4], v[i][5], v[i][6], v[i][7], scale, rs));
}

// im2col_quantize_int8.glsl:26-84 on planar [C,H,W] input: row = output
// pixel, column = c*k*k + ky*k + kx, zero padding; code = rint(clamp(x *
// (1/scale))). Rows are written out_words words apart (>= ceil(K/4));
// words past the im2col width are zero.
__global__ void __launch_bounds__(128) im2col_quantize_kernel(
    uint32_t* __restrict__ packed, float* __restrict__ scales, const float* __restrict__ in, uint32_t iw,
    uint32_t ih, uint32_t ic, uint32_t ow, uint32_t oh, uint32_t k, uint32_t s, int pad, uint32_t out_words,
    uint64_t image_stride, uint64_t rows_per_image) {
    __shared__ float red[4];
    const uint64_t row_global = blockIdx.x;
    const uint64_t img = row_global / rows_per_image;
    const uint32_t row = (uint32_t)(row_global % rows_per_image);
    const float* src = in + img * image_stride;
    const uint32_t ox = row % ow, oy = row / ow;
    const uint32_t area = k * k;
    const uint32_t cols = ic * area;
    auto value = [&](uint32_t c) -> float {
        const uint32_t ci = c / area, ki = c % area;
        const int ix = (int)(ox * s + ki % k) - pad;
        const int iy = (int)(oy * s + ki / k) - pad;
        if (ix < 0 || iy < 0 || ix >= (int)iw || iy >= (int)ih) return 0.0f;
        return __ldg(src + ((uint64_t)ci * ih + iy) * iw + ix);
    };
    float m = 0.f;
    for (uint32_t c = threadIdx.x; c < cols; c += 128) m = fmaxf(m, fabsf(value(c)));
    m = block_max_128(m, red);
    const float scale = fmaxf(m / 127.0f, 1.0e-8f);
    if (threadIdx.x == 0) scales[row_global] = scale;
    const float inv = 1.0f / scale;
    uint32_t* o = packed + row_global * out_words;
    for (uint32_t w = threadIdx.x; w < out_words; w += 128) {
        uint32_t word = 0;
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t c = 4 * w + j;
            if (c < cols) word |= q8(__fmul_rn(value(c), inv)) << (8 * j);
        }
        o[w] = word;
    }
}

// Four codes q8(x * inv) (x * inv rounded once, clamped to +-127, rounded to
// the nearest integer, ties to even) packed little-endian: the rounding is
// the f32 addition of 1.5*2^23, whose low mantissa byte is the code. For the
// exact row abs-max m, inv = 1/max(m/127, 1e-8) gives |x * inv| <= 127 *
// (1 + 3 * 2^-24) < 127.5, so only the lower clamp can act (on NaN: -127,
// as fmaxf returns the other operand). It also must stay: with nothing
// between them, the packed product and rounding addition were contracted
// into one fused multiply-add, which rounds once and moves codes at
// half-integers.
__device__ __forceinline__ uint32_t q8x4_mul(float v0, float v1, float v2, float v3, float inv) {
    constexpr float C = 12582912.0f;
    float q0, q1, q2, q3, t0, t1, t2, t3;
    f2_mul(q0, q1, v0, v1, inv, inv);  // the same IEEE products, two per instruction
    f2_mul(q2, q3, v2, v3, inv, inv);
    q0 = fmaxf(q0, -127.0f);
    q1 = fmaxf(q1, -127.0f);
    q2 = fmaxf(q2, -127.0f);
    q3 = fmaxf(q3, -127.0f);
    f2_add(t0, t1, q0, q1, C, C);
    f2_add(t2, t3, q2, q3, C, C);
    const uint32_t lo = __byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(t2), __float_as_uint(t3), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
}

// Per-pixel channel abs-max of planar [B][C][HW] maps -> [B][HW]. A block covers kAbsmaxPixels consecutive pixels; each pixel's channels are
// split over kAbsmaxSplit threads (channel j goes to thread j % kAbsmaxSplit),
// lanes walk pixels (coalesced plane reads), partial maxima meet in shared
// memory.
constexpr uint32_t kAbsmaxPixels = 64, kAbsmaxSplit = 4;

__global__ void __launch_bounds__(kAbsmaxPixels * kAbsmaxSplit) pixel_absmax_kernel(
    float* __restrict__ out, const float* __restrict__ in, uint32_t c, uint32_t hw, uint64_t pixels) {
    __shared__ float part[kAbsmaxSplit][kAbsmaxPixels];
    const uint32_t lp = threadIdx.x % kAbsmaxPixels, q = threadIdx.x / kAbsmaxPixels;
    const uint64_t i = (uint64_t)blockIdx.x * kAbsmaxPixels + lp;
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
    if (i < pixels) {
        const uint64_t img = i / hw, px = i % hw;
        const float* src = in + img * c * hw + px + (uint64_t)q * hw;
        const uint64_t step = (uint64_t)kAbsmaxSplit * hw;
        uint32_t ch = q;
#pragma unroll 2
        for (; ch + 3 * kAbsmaxSplit < c; ch += 4 * kAbsmaxSplit, src += 4 * step) {
            m0 = fmaxf(m0, fabsf(__ldg(src)));
            m1 = fmaxf(m1, fabsf(__ldg(src + step)));
            m2 = fmaxf(m2, fabsf(__ldg(src + 2 * step)));
            m3 = fmaxf(m3, fabsf(__ldg(src + 3 * step)));
        }
        for (; ch < c; ch += kAbsmaxSplit, src += step) m0 = fmaxf(m0, fabsf(__ldg(src)));
    }
    part[q][lp] = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
    __syncthreads();
    if (q == 0 && i < pixels) {
        float m = part[0][lp];
#pragma unroll
        for (uint32_t k = 1; k < kAbsmaxSplit; ++k) m = fmaxf(m, part[k][lp]);
        out[i] = m;
    }
}

// im2col_quantize_int8.glsl:26-84 for a 3x3, stride-1, pad-1 convolution of
// planar [B][C][H][W] maps, without materialising floats: the row (output
// pixel) abs-max over its C*9 im2col values is the maximum of the per-pixel
// channel abs-maxima over the 3x3 neighbourhood (padding contributes 0), so
// the exact row scale max(absmax/127, 1e-8) is known before any code is
// formed. A block (8 warps) quantizes kIm2colPixels consecutive pixels of one
// image row, kIm2colChunk channels at a time: the chunk's 3-row x
// (kIm2colPixels+2)-pixel halo is staged channel-fastest in shared memory
// (lanes walk the pixels, so every plane read is coalesced; one float4 store
// per 4 channels), then kIm2colChunk/4 lanes take a pixel (a lane 4
// channels) and walk the 9 taps: one float4 shared read, x*(1/scale) for each
// value, one 4-code word, the pixel's words one contiguous store into its
// GEMM row at column tap*C + channel ((ky, kx, c) order). Columns [9C, kp)
// are written zero. A small chunk keeps 5 blocks per SM in flight, so one
// block's staging loads overlap the others' code phases.
constexpr uint32_t kIm2colPixels = 32;
constexpr uint32_t kIm2colChunk = 64;  // 27.7 KB of halo
constexpr uint32_t kIm2colLanesPerPixel = kIm2colChunk / 4;
constexpr uint32_t kIm2colPixelsPerWarp = 32 / kIm2colLanesPerPixel;
constexpr uint32_t kIm2colHalo = kIm2colPixels + 2;
constexpr uint32_t kIm2colPixelWords = kIm2colChunk + 4;  // 16-byte rows; conflict-free float4 staging stores
constexpr uint32_t kIm2colStageItems = 6;                  // (group, row) pairs in flight per warp while staging

__global__ void __launch_bounds__(256, 5) im2col_quantize_3x3_planar_kernel(
    uint8_t* __restrict__ codes, float* __restrict__ scales, const float* __restrict__ in,
    const float* __restrict__ pix_absmax, uint32_t c, uint32_t h, uint32_t w, uint32_t kp) {
    extern __shared__ float4 im2col_smem[];  // halo [3][kIm2colHalo][kIm2colPixelWords], then inv_s
    float* halo = reinterpret_cast<float*>(im2col_smem);
    float* inv_s = halo + 3 * kIm2colHalo * kIm2colPixelWords;
    const uint32_t tiles_x = (w + kIm2colPixels - 1) / kIm2colPixels;
    const uint32_t y = (blockIdx.x / tiles_x) % h;
    const uint64_t img = (uint64_t)blockIdx.x / ((uint64_t)tiles_x * h);
    const uint32_t x0 = (blockIdx.x % tiles_x) * kIm2colPixels;
    const uint32_t np = min(kIm2colPixels, w - x0);
    const uint64_t row0 = (img * h + y) * w + x0;  // GEMM row of the tile's first pixel
    if (threadIdx.x < kIm2colPixels) {
        float m = 0.f;
        const uint32_t x = x0 + threadIdx.x;
        if (threadIdx.x < np) {
            for (int dy = -1; dy <= 1; ++dy)
                for (int dx = -1; dx <= 1; ++dx) {
                    const int yy = (int)y + dy, xx = (int)x + dx;
                    if (yy >= 0 && yy < (int)h && xx >= 0 && xx < (int)w)
                        m = fmaxf(m, pix_absmax[(img * h + yy) * w + xx]);
                }
            const float scale = fmaxf(m / 127.0f, 1.0e-8f);
            scales[row0 + threadIdx.x] = scale;
            inv_s[threadIdx.x] = 1.0f / scale;
        } else {
            inv_s[threadIdx.x] = 0.f;
        }
    }
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const uint64_t hw = (uint64_t)h * w;
    const float* plane0 = in + img * (uint64_t)c * hw;
    for (uint32_t ch0 = 0; ch0 < c; ch0 += kIm2colChunk) {
        const uint32_t groups = min(kIm2colChunk, c - ch0) / 4;  // 4-channel groups in this chunk
        __syncthreads();  // inv_s written; the previous chunk's halo consumed
        const uint32_t prs = groups * 3;  // (4-channel group, halo row) pairs, pair = 3 * group + row
        // stage, halo pixels 0..31: lanes walk the pixels (coalesced plane
        // reads), warps the pairs, kIm2colStageItems pairs' loads in flight
        {
            const int xx = (int)(x0 + lane) - 1;
            const bool x_in = xx >= 0 && xx < (int)w;
            for (uint32_t pr0 = warp; pr0 < prs; pr0 += kIm2colStageItems * 8) {
                float4 v[kIm2colStageItems];
#pragma unroll
                for (uint32_t k = 0; k < kIm2colStageItems; ++k) {
                    const uint32_t pr = pr0 + 8 * k, grp = pr / 3;
                    const int yy = (int)y + (int)(pr - 3 * grp) - 1;
                    v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (pr < prs && x_in && yy >= 0 && yy < (int)h) {
                        const float* q = plane0 + (uint64_t)(ch0 + 4 * grp) * hw + (uint64_t)yy * w + xx;
                        v[k].x = __ldg(q);
                        v[k].y = __ldg(q + hw);
                        v[k].z = __ldg(q + 2 * hw);
                        v[k].w = __ldg(q + 3 * hw);
                    }
                }
#pragma unroll
                for (uint32_t k = 0; k < kIm2colStageItems; ++k) {
                    const uint32_t pr = pr0 + 8 * k, grp = pr / 3;
                    if (pr < prs)
                        *reinterpret_cast<float4*>(halo + ((pr - 3 * grp) * kIm2colHalo + lane) * kIm2colPixelWords +
                                                   4 * grp) = v[k];
                }
            }
        }
        // stage, halo pixels 32 and 33 of every pair
        for (uint32_t i = threadIdx.x; i < 2 * prs; i += blockDim.x) {
            const uint32_t pr = i >> 1, px = kIm2colPixels + (i & 1), grp = pr / 3, r = pr - 3 * grp;
            const int yy = (int)y + (int)r - 1, xx = (int)(x0 + px) - 1;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (yy >= 0 && yy < (int)h && xx >= 0 && xx < (int)w) {
                const float* q = plane0 + (uint64_t)(ch0 + 4 * grp) * hw + (uint64_t)yy * w + xx;
                v.x = __ldg(q);
                v.y = __ldg(q + hw);
                v.z = __ldg(q + 2 * hw);
                v.w = __ldg(q + 3 * hw);
            }
            *reinterpret_cast<float4*>(halo + (r * kIm2colHalo + px) * kIm2colPixelWords + 4 * grp) = v;
        }
        __syncthreads();
        // codes: kIm2colLanesPerPixel lanes per pixel (a lane per 4 channels),
        // kIm2colPixelsPerWarp pixels per warp step, the 9 taps unrolled
        // (constant shared offsets)
        const uint32_t gl = lane % kIm2colLanesPerPixel, sub = lane / kIm2colLanesPerPixel;
        if (gl < groups) {
            const uint32_t tap_words = c / 4;
            for (uint32_t p = warp * kIm2colPixelsPerWarp + sub; p < np; p += nwarps * kIm2colPixelsPerWarp) {
                const float inv = inv_s[p];
                const float* hp = halo + p * kIm2colPixelWords + 4 * gl;
                uint32_t* o = reinterpret_cast<uint32_t*>(codes + (row0 + p) * kp + ch0) + gl;
#pragma unroll
                for (uint32_t tap = 0; tap < 9; ++tap, o += tap_words) {
                    const float4 v = *reinterpret_cast<const float4*>(
                        hp + ((tap / 3) * kIm2colHalo + tap % 3) * kIm2colPixelWords);
                    *o = q8x4_mul(v.x, v.y, v.z, v.w, inv);
                }
            }
        }
    }
    // zero columns beyond 9*c, a warp per row
    const uint32_t words = kp / 4, used = 9 * c / 4;
    if (used < words)
        for (uint32_t r = warp; r < np; r += nwarps) {
            uint32_t* o = reinterpret_cast<uint32_t*>(codes + (row0 + r) * kp);
            for (uint32_t wd = used + lane; wd < words; wd += 32) o[wd] = 0u;
        }
}

}  // namespace

int launch_im2col_quantize_3x3_planar(uint8_t* codes, float* scales, float* pix_absmax, const float* in,
                                      uint32_t batch, uint32_t c, uint32_t h, uint32_t w, uint32_t kp,
                                      cudaStream_t st) {
    if (kp % 4 || kp < 9 * c) return set_error(DAV2CUDA_INVALID_ARGUMENT, "im2col 3x3: row width");
    const uint64_t pixels = (uint64_t)batch * h * w;
    pixel_absmax_kernel<<<(unsigned)((pixels + kAbsmaxPixels - 1) / kAbsmaxPixels), kAbsmaxPixels * kAbsmaxSplit, 0,
                          st>>>(pix_absmax, in, c, h * w, pixels);
    if (c % 4) return set_error(DAV2CUDA_INVALID_ARGUMENT, "im2col 3x3: channels % 4");
    const uint64_t blocks = (uint64_t)batch * h * ((w + kIm2colPixels - 1) / kIm2colPixels);
    if (blocks > 0x7fffffffull) return set_error(DAV2CUDA_INVALID_ARGUMENT, "im2col 3x3: grid too large");
    const size_t smem = (3 * kIm2colHalo * kIm2colPixelWords + kIm2colPixels) * sizeof(float);
    if (cudaFuncSetAttribute(im2col_quantize_3x3_planar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return set_error(DAV2CUDA_LAUNCH_FAILED, "im2col 3x3: cannot set shared memory size");
    im2col_quantize_3x3_planar_kernel<<<(unsigned)blocks, 256, smem, st>>>(codes, scales, in, pix_absmax, c, h, w,
                                                                           kp);
    return check_launch("im2col_quantize_3x3_planar");
}

// ============================================================ launchers
static unsigned grid_for(uint64_t n, unsigned block = kBlock) {
    const uint64_t g = (n + block - 1) / block;
    const uint64_t cap = 148ull * 16;
    return (unsigned)(g < cap ? (g == 0 ? 1 : g) : cap);
}

int launch_layer_norm(void* out, float* out_scales, const float* in, const float* w, const float* b,
                      uint32_t rows, uint32_t cols, float eps, int out_kind, uint32_t out_group,
                      uint32_t in_group, uint32_t in_offset, cudaStream_t st) {
    const bool vec = (cols % 4 == 0) && cols <= 32 * 4 * 8 && (reinterpret_cast<uintptr_t>(in) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (reinterpret_cast<uintptr_t>(b) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(out) % 16 == 0);
    if (!vec) {
        if (out_kind != kLnF32 || out_group != in_group || in_offset != 0)
            return set_error(DAV2CUDA_INVALID_ARGUMENT, "layer_norm: this output form needs columns % 4 == 0 and <= 1024");
        layer_norm_generic_kernel<<<rows, 64, 0, st>>>(static_cast<float*>(out), in, w, b, cols, eps);
        return check_launch("layer_norm_generic");
    }
    const unsigned grid = (unsigned)(((uint64_t)rows * 32 + 127) / 128);  // 4 rows per block
    const int vpl = (int)((cols / 4 + 31) / 32);
#define LN_CASE(V)                                                                                         \
    case V:                                                                                                \
        switch (out_kind) {                                                                                \
            case kLnF32: layer_norm_warp_kernel<V, kLnF32><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break; \
            case kLnF16: layer_norm_warp_kernel<V, kLnF16><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break; \
            case kLnBF16: layer_norm_warp_kernel<V, kLnBF16><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break; \
            default: layer_norm_warp_kernel<V, kLnS8><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break; \
        }                                                                                                  \
        break;
    switch (vpl) {
        LN_CASE(1)
        LN_CASE(2)
        LN_CASE(3)
        LN_CASE(4)
        LN_CASE(6)
        LN_CASE(8)
        case 5:
        case 7:
            switch (out_kind) {
                case kLnF32: layer_norm_warp_kernel<8, kLnF32><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break;
                case kLnF16: layer_norm_warp_kernel<8, kLnF16><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break;
                case kLnBF16: layer_norm_warp_kernel<8, kLnBF16><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break;
                default: layer_norm_warp_kernel<8, kLnS8><<<grid, 128, 0, st>>>(out, out_scales, in, w, b, rows, cols, eps, out_group, in_group, in_offset); break;
            }
            break;
        default: return set_error(DAV2CUDA_INVALID_ARGUMENT, "layer_norm: unsupported width");
    }
#undef LN_CASE
    return check_launch("layer_norm");
}

int launch_gelu(float* out, const float* in, uint64_t n, cudaStream_t st) {
    gelu_kernel<<<grid_for((n + 3) / 4), kBlock, 0, st>>>(out, in, n);
    return check_launch("gelu");
}

int launch_softmax(float* out, const float* in, uint64_t rows, uint32_t cols, float scale, cudaStream_t st) {
    const bool aligned = (reinterpret_cast<uintptr_t>(in) % 8 == 0) && (reinterpret_cast<uintptr_t>(out) % 8 == 0) &&
                         (cols % 2 == 0);
    const unsigned grid = (unsigned)((rows * 32 + 255) / 256);
    if (aligned && cols <= 2 * 32 * 24) {
        softmax_warp_kernel<24><<<grid, 256, 0, st>>>(out, in, rows, cols, scale);
    } else if (aligned && cols <= 2 * 32 * 48) {
        softmax_warp_kernel<48><<<grid, 256, 0, st>>>(out, in, rows, cols, scale);
    } else {
        softmax_generic_kernel<<<(unsigned)rows, 256, 0, st>>>(out, in, cols, scale);
    }
    return check_launch("softmax");
}

int launch_add_scaled(float* out, const float* res, const float* add, const float* scale, uint64_t n,
                      uint32_t cols, cudaStream_t st) {
    add_scaled_kernel<<<grid_for(n), kBlock, 0, st>>>(out, res, add, scale, n, cols);
    return check_launch("add_scaled");
}

int launch_relu(float* out, const float* in, uint64_t n, cudaStream_t st) {
    relu_kernel<<<grid_for(n), kBlock, 0, st>>>(out, in, n);
    return check_launch("relu");
}

int launch_add(float* out, const float* a, const float* b, uint64_t n, cudaStream_t st) {
    add_kernel<<<grid_for(n), kBlock, 0, st>>>(out, a, b, n);
    return check_launch("add");
}

int launch_sigmoid_scale(float* out, const float* in, uint64_t n, float s, cudaStream_t st) {
    sigmoid_scale_kernel<<<grid_for(n), kBlock, 0, st>>>(out, in, n, s);
    return check_launch("sigmoid_scale");
}

template <typename TI, typename TO>
int launch_bilinear_align(TO* out, const TI* in, uint32_t iw, uint32_t ih, uint32_t ow, uint32_t oh,
                          uint32_t planes, cudaStream_t st) {
    if (planes >= kPlanesPerBlock && (planes + kPlanesPerBlock - 1) / kPlanesPerBlock <= 65535 && oh <= 65535) {
        const uint32_t threads = std::min<uint32_t>((ow + 31) / 32 * 32, 1024u);
        dim3 grid((ow + threads - 1) / threads, oh, (planes + kPlanesPerBlock - 1) / kPlanesPerBlock);
        bilinear_align_rows_kernel<TI, TO><<<grid, threads, 0, st>>>(out, in, iw, ih, ow, oh, planes);
        return check_launch("bilinear_align_true");
    }
    dim3 grid((ow + 127) / 128, oh, planes < 65535 ? planes : 65535);
    bilinear_align_kernel<TI, TO><<<grid, 128, 0, st>>>(out, in, iw, ih, ow, oh, planes);
    return check_launch("bilinear_align_true");
}
template int launch_bilinear_align<float, float>(float*, const float*, uint32_t, uint32_t, uint32_t, uint32_t,
                                                 uint32_t, cudaStream_t);

bool bilinear_nhwc_to_planar_supported(uint32_t iw, uint32_t c, uint32_t ow) {
    return c && c % 32 == 0 && iw && ((uint64_t)2 * iw * kNhwcPixelWords + 2ull * ow) * sizeof(float) <= kNhwcMaxSmem;
}

int launch_bilinear_nhwc_to_planar(float* out, const float* in, uint32_t batch, uint32_t ih, uint32_t iw, uint32_t c,
                                   uint32_t oh, uint32_t ow, cudaStream_t st) {
    if (!bilinear_nhwc_to_planar_supported(iw, c, ow) || !batch || !ih || !oh || !ow ||
        reinterpret_cast<uintptr_t>(in) % 16)
        return set_error(DAV2CUDA_INVALID_ARGUMENT,
                         "bilinear_nhwc_to_planar: channels % 32, source width fitting shared memory, 16-byte source");
    const uint64_t blocks = (uint64_t)batch * (ih > 1 ? ih - 1 : 1) * (c / 32);
    if (blocks > 0x7fffffffull) return set_error(DAV2CUDA_INVALID_ARGUMENT, "bilinear_nhwc_to_planar: grid too large");
    const size_t smem = ((size_t)2 * iw * kNhwcPixelWords + 2 * (size_t)ow) * sizeof(float);
    if (cudaFuncSetAttribute(bilinear_nhwc_to_planar_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return set_error(DAV2CUDA_LAUNCH_FAILED, "bilinear_nhwc_to_planar: cannot set shared memory size");
    bilinear_nhwc_to_planar_kernel<<<(unsigned)blocks, 256, smem, st>>>(out, in, ih, iw, c, oh, ow);
    return check_launch("bilinear_nhwc_to_planar");
}

int launch_minmax_batched(const float* in, float* ranges, uint64_t n, uint32_t batch, cudaStream_t st) {
    if (batch == 0 || batch > 65535) return set_error(DAV2CUDA_INVALID_ARGUMENT, "reduce_minmax: batch out of range");
    uint32_t* keys = reinterpret_cast<uint32_t*>(ranges);
    minmax_init_kernel<<<(batch + 127) / 128, 128, 0, st>>>(keys, batch);
    const unsigned gx = (unsigned)std::max<uint64_t>(1, grid_for(n) / batch);
    minmax_reduce_kernel<<<dim3(gx, batch), kBlock, 0, st>>>(keys, in, n);
    minmax_finish_kernel<<<(batch + 127) / 128, 128, 0, st>>>(keys, batch);
    return check_launch("reduce_minmax");
}

int launch_minmax(const float* in, float* range, uint64_t n, cudaStream_t st) {
    return launch_minmax_batched(in, range, n, 1, st);
}

int launch_normalize_batched(float* d, const float* ranges, uint64_t n, uint32_t batch, float maximum,
                             cudaStream_t st) {
    if (batch == 0 || batch > 65535) return set_error(DAV2CUDA_INVALID_ARGUMENT, "normalize: batch out of range");
    const unsigned gx = (unsigned)std::max<uint64_t>(1, grid_for(n) / batch);
    normalize_kernel<<<dim3(gx, batch), kBlock, 0, st>>>(d, ranges, n, maximum);
    return check_launch("normalize");
}

int launch_normalize(float* d, const float* range, uint64_t n, float maximum, cudaStream_t st) {
    return launch_normalize_batched(d, range, n, 1, maximum, st);
}

int launch_preprocess_u32_batched(float* out, const uint32_t* px, uint32_t batch, uint32_t sw, uint32_t sh,
                                  uint32_t stride, uint64_t img_stride, uint32_t rgba, uint32_t dw, uint32_t dh,
                                  cudaStream_t st) {
    if (batch == 0 || batch > 65535) return set_error(DAV2CUDA_INVALID_ARGUMENT, "preprocess_u32: batch out of range");
    dim3 grid((dw + 127) / 128, dh, batch);
    preprocess_u32_kernel<<<grid, 128, 0, st>>>(out, px, sw, sh, stride, rgba, dw, dh, img_stride);
    return check_launch("preprocess_u32");
}

int launch_preprocess_u32(float* out, const uint32_t* px, uint32_t sw, uint32_t sh, uint32_t stride,
                          uint32_t rgba, uint32_t dw, uint32_t dh, cudaStream_t st) {
    return launch_preprocess_u32_batched(out, px, 1, sw, sh, stride, 0, rgba, dw, dh, st);
}

int launch_preprocess_bgr8(float* out, const uint8_t* bgr, uint32_t batch, uint32_t sw, uint32_t sh,
                           uint64_t row_stride, uint64_t img_stride, uint32_t dw, uint32_t dh, int bilinear,
                           cudaStream_t st) {
    dim3 grid((dw + 127) / 128, dh, batch);
    if (bilinear)
        preprocess_bgr8_bilinear_kernel<<<grid, 128, 0, st>>>(out, bgr, sw, sh, row_stride, img_stride, dw, dh);
    else
        preprocess_bgr8_kernel<<<grid, 128, 0, st>>>(out, bgr, sw, sh, row_stride, img_stride, dw, dh);
    return check_launch("preprocess_bgr8");
}

template <typename T>
int launch_quantize_rows(uint32_t* packed, float* scales, const T* in, uint64_t rows, uint32_t cols,
                         uint64_t offset, uint32_t group, uint64_t group_stride, uint32_t row_stride,
                         uint32_t out_words, cudaStream_t st) {
    if (rows == 0) return DAV2CUDA_OK;
    if constexpr (std::is_same<T, __half>::value || std::is_same<T, float>::value) {
        constexpr uint32_t kAlign = 8;  // 8-element groups start on 16-byte boundaries
        const bool plain = offset == 0 && (group == rows || group_stride == (uint64_t)group * row_stride);
        const bool aligned = (reinterpret_cast<uintptr_t>(in) % 16 == 0) && (row_stride % kAlign == 0) &&
                             (reinterpret_cast<uintptr_t>(packed) % 8 == 0) && out_words == cols / 4;
        if (plain && aligned && cols % 256 == 0 && cols <= 2048) {
            const unsigned grid = (unsigned)((rows + 3) / 4);
#define DAV2_QWARP(V)                                                                                        \
    case V:                                                                                                  \
        quantize_rows_warp_kernel<T, V><<<grid, 128, 0, st>>>(packed, scales, in, rows, row_stride, out_words); \
        break;
            switch (cols / 256) {
                DAV2_QWARP(1) DAV2_QWARP(2) DAV2_QWARP(3) DAV2_QWARP(4) DAV2_QWARP(5) DAV2_QWARP(6) DAV2_QWARP(7)
                default: DAV2_QWARP(8)
            }
#undef DAV2_QWARP
            return check_launch("quantize_rows_warp");
        }
        if (plain && aligned && cols % 1024 == 0 && cols <= 8192) {
#define DAV2_QVEC(V)                                                                                          \
    case V:                                                                                                   \
        quantize_rows_vec_kernel<T, V><<<(unsigned)rows, 128, 0, st>>>(packed, scales, in, cols, row_stride,  \
                                                                       out_words);                            \
        break;
            switch (cols / 1024) {
                DAV2_QVEC(1) DAV2_QVEC(2) DAV2_QVEC(3) DAV2_QVEC(4) DAV2_QVEC(6) DAV2_QVEC(8)
                default: goto generic;
            }
#undef DAV2_QVEC
            return check_launch("quantize_rows_vec");
        }
    }
generic:
    quantize_rows_kernel<T><<<(unsigned)rows, 128, 0, st>>>(packed, scales, in, cols, offset, group, group_stride,
                                                            row_stride, out_words);
    return check_launch("quantize_rows");
}
template int launch_quantize_rows<float>(uint32_t*, float*, const float*, uint64_t, uint32_t, uint64_t,
                                         uint32_t, uint64_t, uint32_t, uint32_t, cudaStream_t);
template int launch_quantize_rows<__half>(uint32_t*, float*, const __half*, uint64_t, uint32_t, uint64_t,
                                          uint32_t, uint64_t, uint32_t, uint32_t, cudaStream_t);

int launch_im2col_quantize(uint32_t* packed, float* scales, const float* in, uint32_t batch, uint32_t iw,
                           uint32_t ih, uint32_t ic, uint32_t ow, uint32_t oh, uint32_t k, uint32_t s, int pad,
                           uint32_t out_words, cudaStream_t st) {
    const uint64_t rows = (uint64_t)ow * oh;
    im2col_quantize_kernel<<<(unsigned)(rows * batch), 128, 0, st>>>(packed, scales, in, iw, ih, ic, ow, oh, k, s,
                                                                      pad, out_words, (uint64_t)ic * iw * ih, rows);
    return check_launch("im2col_quantize");
}

}  // namespace dav2cuda
