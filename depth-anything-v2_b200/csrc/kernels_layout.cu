// Layout conversions feeding the tensor-core GEMM: planar f32 -> channels-
// last half, f32 -> half, row padding to 16-byte multiples, explicit im2col
// of channels-last maps (strided convolutions) and convolution weight
// reorders to the K-major [Cout][ky][kx][Cin] operand layout.
#include "kernels.cuh"

namespace dav2cuda {
namespace {

template <typename H>
__device__ __forceinline__ H cvt(float v);
template <>
__device__ __forceinline__ __half cvt<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ float cvt<float>(float v) { return v; }

// [B][C][H][W] f32 -> [B][H][W][Cp] half via a 32x32 shared-memory transpose
// per (image, 32 channels, 32 pixels).
template <typename H>
__global__ void nchw_to_nhwc_kernel(H* __restrict__ out, const float* __restrict__ in, uint32_t c, uint32_t hw,
                                    uint32_t cp) {
    __shared__ float tile[32][33];
    const uint64_t img = blockIdx.z;
    const uint32_t p0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const float* src = in + img * (uint64_t)c * hw;
    for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y) {
        const uint32_t ch = c0 + i, px = p0 + threadIdx.x;
        tile[i][threadIdx.x] = (ch < c && px < hw) ? __ldg(src + (uint64_t)ch * hw + px) : 0.0f;
    }
    __syncthreads();
    H* dst = out + img * (uint64_t)hw * cp;
    for (uint32_t i = threadIdx.y; i < 32; i += blockDim.y) {
        const uint32_t px = p0 + i, ch = c0 + threadIdx.x;
        if (px < hw && ch < cp) dst[(uint64_t)px * cp + ch] = cvt<H>(tile[threadIdx.x][i]);
    }
}

template <typename H>
__global__ void to_half_kernel(H* __restrict__ out, const float* __restrict__ in, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = cvt<H>(in[i]);
}

template <typename H>
__global__ void pad_rows_kernel(H* __restrict__ out, const float* __restrict__ in, uint64_t rows, uint32_t cols,
                                uint32_t cols_p) {
    const uint64_t n = rows * cols_p;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t r = i / cols_p;
        const uint32_t c = (uint32_t)(i % cols_p);
        out[i] = cvt<H>(c < cols ? in[r * cols + c] : 0.0f);
    }
}

// Channels-last im2col: row = (img, oy, ox), column = (ky*k + kx)*C + c,
// padded with zeros to kp columns. 8 channels (16 bytes) per thread.
template <typename H>
__global__ void im2col_nhwc_kernel(H* __restrict__ out, const H* __restrict__ in, uint32_t h, uint32_t w,
                                   uint32_t c, uint32_t k, uint32_t s, uint32_t pad, uint32_t oh, uint32_t ow,
                                   uint32_t kp, uint64_t rows) {
    const uint32_t vec_per_row = kp / 8;
    const uint64_t total = rows * vec_per_row;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const uint64_t r = i / vec_per_row;
        const uint32_t col = (uint32_t)(i % vec_per_row) * 8;
        const uint64_t img = r / ((uint64_t)oh * ow);
        const uint32_t pp = (uint32_t)(r % ((uint64_t)oh * ow));
        const uint32_t oy = pp / ow, ox = pp % ow;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (col < k * k * c) {
            const uint32_t tap = col / c, ch = col % c;
            const int iy = (int)(oy * s + tap / k) - (int)pad;
            const int ix = (int)(ox * s + tap % k) - (int)pad;
            if (iy >= 0 && ix >= 0 && iy < (int)h && ix < (int)w)
                v = *reinterpret_cast<const uint4*>(in + ((img * h + iy) * w + ix) * c + ch);
        }
        *reinterpret_cast<uint4*>(out + r * kp + col) = v;
    }
}

template <typename H>
__global__ void conv_weight_kernel(H* __restrict__ out, const float* __restrict__ w, uint32_t co, uint32_t ci,
                                   uint32_t k, uint32_t cip) {
    const uint64_t n = (uint64_t)co * k * k * cip;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t c = (uint32_t)(i % cip);
        const uint64_t t = i / cip;
        const uint32_t tap = (uint32_t)(t % (k * k));
        const uint32_t o = (uint32_t)(t / (k * k));
        out[i] = cvt<H>(c < ci ? w[(((uint64_t)o * ci + c) * k + tap / k) * k + tap % k] : 0.0f);
    }
}

// int8 convolution weight codes [Co][K] (K = Ci*k*k in the reference's
// (ci, ky, kx) column order, rows k_in bytes apart) -> (ky, kx, ci) column
// order with rows padded to kp bytes: the order of a channels-last im2col.
// A permutation of each row's codes, so every dot product is unchanged.
__global__ void conv_codes_tap_major_kernel(uint8_t* __restrict__ out, const uint8_t* __restrict__ in, uint32_t co,
                                            uint32_t ci, uint32_t kk, uint32_t k_in, uint32_t kp) {
    const uint64_t n = (uint64_t)co * kp;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t o = i / kp;
        const uint32_t col = (uint32_t)(i % kp);
        uint8_t v = 0;
        if (col < ci * kk) v = in[o * k_in + (uint64_t)(col % ci) * kk + col / ci];
        out[i] = v;
    }
}

unsigned grid_cap(uint64_t n) {
    const uint64_t g = (n + 255) / 256;
    return (unsigned)(g == 0 ? 1 : (g < 148 * 16 ? g : 148 * 16));
}

}  // namespace

template <typename H>
int launch_nchw_to_nhwc(H* out, const float* in, uint32_t batch, uint32_t c, uint32_t h, uint32_t w, uint32_t cp,
                        cudaStream_t st) {
    const uint32_t hw = h * w;
    dim3 grid((hw + 31) / 32, (cp + 31) / 32, batch);
    nchw_to_nhwc_kernel<H><<<grid, dim3(32, 8), 0, st>>>(out, in, c, hw, cp);
    return check_launch("nchw_to_nhwc");
}

template <typename H>
int launch_to_half(H* out, const float* in, uint64_t n, cudaStream_t st) {
    to_half_kernel<H><<<grid_cap(n), 256, 0, st>>>(out, in, n);
    return check_launch("to_half");
}

template <typename H>
int launch_pad_rows_half(H* out, const float* in, uint64_t rows, uint32_t cols, uint32_t cols_p, cudaStream_t st) {
    pad_rows_kernel<H><<<grid_cap(rows * cols_p), 256, 0, st>>>(out, in, rows, cols, cols_p);
    return check_launch("pad_rows");
}

template <typename H>
int launch_im2col_nhwc(H* out, const H* in, uint32_t batch, uint32_t h, uint32_t w, uint32_t c, uint32_t k,
                       uint32_t s, uint32_t pad, uint32_t oh, uint32_t ow, uint32_t kp, cudaStream_t st) {
    if (c % 8 || kp % 8) return set_error(DAV2CUDA_INVALID_ARGUMENT, "im2col_nhwc: channels must be multiples of 8");
    const uint64_t rows = (uint64_t)batch * oh * ow;
    im2col_nhwc_kernel<H><<<grid_cap(rows * (kp / 8)), 256, 0, st>>>(out, in, h, w, c, k, s, pad, oh, ow, kp, rows);
    return check_launch("im2col_nhwc");
}

template <typename H>
int launch_conv_weight_to_half(H* out, const float* w, uint32_t co, uint32_t ci, uint32_t k, uint32_t cip,
                               cudaStream_t st) {
    conv_weight_kernel<H><<<grid_cap((uint64_t)co * k * k * cip), 256, 0, st>>>(out, w, co, ci, k, cip);
    return check_launch("conv_weight");
}

int launch_conv_codes_tap_major(uint8_t* out, const uint8_t* in, uint32_t co, uint32_t ci, uint32_t kk, uint32_t k_in,
                                uint32_t kp, cudaStream_t st) {
    conv_codes_tap_major_kernel<<<grid_cap((uint64_t)co * kp), 256, 0, st>>>(out, in, co, ci, kk, k_in, kp);
    return check_launch("conv_codes_tap_major");
}

template int launch_nchw_to_nhwc<float>(float*, const float*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,
                                        cudaStream_t);

#define DAV2_INST(H)                                                                                           \
    template int launch_nchw_to_nhwc<H>(H*, const float*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,    \
                                        cudaStream_t);                                                          \
    template int launch_to_half<H>(H*, const float*, uint64_t, cudaStream_t);                                  \
    template int launch_pad_rows_half<H>(H*, const float*, uint64_t, uint32_t, uint32_t, cudaStream_t);        \
    template int launch_im2col_nhwc<H>(H*, const H*, uint32_t, uint32_t, uint32_t, uint32_t, uint32_t,         \
                                       uint32_t, uint32_t, uint32_t, uint32_t, uint32_t, cudaStream_t);        \
    template int launch_conv_weight_to_half<H>(H*, const float*, uint32_t, uint32_t, uint32_t, uint32_t,       \
                                               cudaStream_t);
DAV2_INST(__half)
DAV2_INST(__nv_bfloat16)
#undef DAV2_INST

}  // namespace dav2cuda
