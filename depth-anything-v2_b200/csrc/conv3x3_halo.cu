// 3x3 convolution (pad 1) to 128 output channels on channels-last 16-bit
// maps, + bias, 16-bit channels-last output — the DPT head's output_conv1
// (src/dpt.cpp:830-840; conv2d_common.glsl:55-139 in the reference) — as a
// halo-loading tcgen05 kernel.
//
// A tile is two image rows x 128 output pixels (M = 256: two M=128 MMAs that
// share every weight tile). Per 64-channel chunk one TMA box brings the tile's
// 4 x 130-pixel halo into shared memory as 128-byte-swizzled pixel rows; tap
// (dy, dx) of output row r is the same rows seen from pixel (r + dy)*130 + dx,
// an operand descriptor started there (the MMA undoes the swizzle from the
// absolute address bits, as TMA applied it). Weight tiles (128 output
// channels x 64 input channels, one per (chunk, tap)) stream through their own
// ring. Against one shifted A tile per tap (the generic implicit GEMM), each
// input pixel crosses L2 once per chunk instead of nine times, and each weight
// tile serves 256 pixels instead of 128.
//
// Roles (persistent, one CTA per SM): warp 0 TMA (halo ring and weight ring),
// warp 1 the MMA issuer (8 MMAs per weight tile into two 128-column TMEM
// accumulators, double-buffered across tiles: all 512 columns), warps 2..5
// the epilogue (one TMEM lane quarter each: + bias, rounded to 16 bits, stored
// as 256-byte channels-last pixel rows). Every wait is bounded; a timeout sets
// the device error word and the kernel drains and returns.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>

namespace dav2cuda {
namespace {

constexpr uint32_t kHaloPixels = 130;
constexpr uint32_t kHaloRows = 4;                            // two output rows + the rows above and below
constexpr uint32_t kHaloBytes = kHaloRows * kHaloPixels * 128;  // 66560 = 65 KB
constexpr uint32_t kAStages = 2;
constexpr uint32_t kBBytes = 128 * 128;                      // 128 output channels x 64 input channels
constexpr uint32_t kBStages = 5;
constexpr uint32_t kCout = 128;
constexpr uint32_t kThreads = 6 * 32;
constexpr uint32_t kSmem = kAStages * kHaloBytes + kBStages * kBBytes + 1024 + 1024;  // + barriers + slack
static_assert(kHaloBytes % 1024 == 0, "halo stages must keep the 1 KB swizzle period");
static_assert(kSmem <= 232448, "shared memory above the per-block limit");

struct ConvParams {
    uint32_t batch, h, w, cin;  // input [batch][h][w][cin] -> output [batch][h][w][128]
    uint32_t tiles_x, tiles_y, tiles;
    const float* bias;          // [128]
    void* out;
    int* err;
};

__device__ __forceinline__ uint64_t desc_sw128_at(uint32_t saddr) {
    // K-major, 128-byte rows, 128-byte swizzle, 8-row groups 1 KB apart; the
    // start may be any row of a 1 KB-aligned swizzled region (base offset 0)
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    conv3x3_halo_kernel(const __grid_constant__ CUtensorMap tm_in, const __grid_constant__ CUtensorMap tm_w,
                        const ConvParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* sA = smem;                               // [stage][4 x 130 pixels][128 B, swizzled]
    uint8_t* sB = smem + kAStages * kHaloBytes;       // [stage][128 rows][128 B, swizzled]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kBStages * kBBytes);
    uint64_t* a_full = bars;                          // [A stage]
    uint64_t* a_empty = a_full + kAStages;
    uint64_t* b_full = a_empty + kAStages;            // [B stage]
    uint64_t* b_empty = b_full + kBStages;
    uint64_t* tfull = b_empty + kBStages;             // [accumulator pair]
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t chunks = p.cin / 64;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_in);
        tma_prefetch_desc(&tm_w);
        for (uint32_t s = 0; s < kAStages; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        for (uint32_t s = 0; s < kBStages; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t ga = 0, gb = 0;  // halo and weight stages filled (all tiles)
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
                const uint32_t xt = t % p.tiles_x, rest = t / p.tiles_x;
                const uint32_t yt = rest % p.tiles_y, img = rest / p.tiles_y;
                for (uint32_t c = 0; ok && c < chunks; ++c, ++ga) {
                    const uint32_t sa = ga % kAStages;
                    if (!mbar_wait(&a_empty[sa], ((ga / kAStages) & 1u) ^ 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&a_full[sa], kHaloBytes);
                    tma_load_4d(sA + sa * kHaloBytes, &tm_in, &a_full[sa], (int)(c * 64u), (int)(xt * 128u) - 1,
                                (int)(yt * 2u) - 1, (int)img);
                    for (uint32_t tap = 0; tap < 9; ++tap, ++gb) {
                        const uint32_t sb = gb % kBStages;
                        if (!mbar_wait(&b_empty[sb], ((gb / kBStages) & 1u) ^ 1u, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive_expect_tx(&b_full[sb], kBBytes);
                        tma_load_2d(sB + sb * kBBytes, &tm_w, &b_full[sb], (int)(tap * p.cin + c * 64u), 0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc(1u, kBF16 ? 1u : 0u, 128u, kCout);
            const uint32_t a0 = smem_addr(sA), b0 = smem_addr(sB);
            uint32_t ga = 0, gb = 0, local = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++local) {
                const uint32_t buf = local & 1u;
                // the epilogue has read this accumulator pair's previous tile
                if (!mbar_wait(&tempty[buf], ((local >> 1) & 1u) ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t acc0 = tmem + buf * 2u * kCout;  // output rows 0 and 1 at +0, +kCout
                for (uint32_t c = 0; ok && c < chunks; ++c, ++ga) {
                    const uint32_t sa = ga % kAStages;
                    if (!mbar_wait(&a_full[sa], (ga / kAStages) & 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    const uint32_t halo = a0 + sa * kHaloBytes;
                    for (uint32_t tap = 0; tap < 9; ++tap, ++gb) {
                        const uint32_t sb = gb % kBStages;
                        if (!mbar_wait(&b_full[sb], (gb / kBStages) & 1u, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t brow = b0 + sb * kBBytes;
#pragma unroll
                        for (uint32_t r = 0; r < 2; ++r) {
                            const uint32_t arow = halo + ((r + tap / 3) * kHaloPixels + tap % 3) * 128u;
#pragma unroll
                            for (uint32_t kk = 0; kk < 4; ++kk)  // 16 channels per MMA
                                umma<false>(acc0 + r * kCout, desc_sw128_at(arow + 32u * kk),
                                            desc_sw128_at(brow + 32u * kk), idesc, (c | tap | kk) ? 1u : 0u);
                        }
                        umma_commit(&b_empty[sb]);
                        mma_issued = true;
                    }
                    if (ok) umma_commit(&a_empty[sa]);
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (pixels of the tile)
        const uint32_t quarter = warp & 3u;
        uint32_t local = 0;
        for (uint32_t t = blockIdx.x; t < p.tiles; t += gridDim.x, ++local) {
            const uint32_t buf = local & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (local >> 1) & 1u, abort_flag, p.err))) break;
            tc_fence_after();
            const uint32_t xt = t % p.tiles_x, rest = t / p.tiles_x;
            const uint32_t yt = rest % p.tiles_y, img = rest / p.tiles_y;
            const uint32_t x = xt * 128u + quarter * 32u + lane;
#pragma unroll 1
            for (uint32_t r = 0; r < 2; ++r) {
                const uint32_t y = yt * 2u + r;
                const bool live = x < p.w && y < p.h;
                uint16_t* orow = static_cast<uint16_t*>(p.out) + (((uint64_t)img * p.h + y) * p.w + x) * kCout;
#pragma unroll 1
                for (uint32_t c0 = 0; c0 < kCout; c0 += 32) {
                    uint32_t acc[32];
                    tmem_ld_32x32b_x32(tmem + ((quarter * 32u) << 16) + buf * 2u * kCout + r * kCout + c0, acc);
                    tmem_ld_wait();
                    if (live) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const float4 b0 = __ldg(reinterpret_cast<const float4*>(p.bias + c0) + 2 * q);
                            const float4 b1 = __ldg(reinterpret_cast<const float4*>(p.bias + c0) + 2 * q + 1);
                            const float bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
                            uint32_t packed[4];
#pragma unroll
                            for (int k = 0; k < 4; ++k) {
                                const float v0 = __fadd_rn(__uint_as_float(acc[8 * q + 2 * k]), bs[2 * k]);
                                const float v1 = __fadd_rn(__uint_as_float(acc[8 * q + 2 * k + 1]), bs[2 * k + 1]);
                                if constexpr (kBF16) {
                                    __nv_bfloat162 h2 = __floats2bfloat162_rn(v0, v1);
                                    packed[k] = *reinterpret_cast<uint32_t*>(&h2);
                                } else {
                                    __half2 h2 = __floats2half2_rn(v0, v1);
                                    packed[k] = *reinterpret_cast<uint32_t*>(&h2);
                                }
                            }
                            *reinterpret_cast<uint4*>(orow + c0 + 8 * q) =
                                make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }

    __syncthreads();
    if (*abort_flag) {
        if (warp == 1 && lane == 0 && mma_issued) {
            umma_commit(drain);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(smem_addr(drain), 0) && globaltimer() - t0 < 100000000ull) {
            }
        }
        if (threadIdx.x == 0) {
            const unsigned long long t0 = globaltimer();
            while (globaltimer() - t0 < 2000000ull) {
            }
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_conv_enc = nullptr;
std::once_flag g_conv_enc_once;

}  // namespace

bool conv3x3_halo_supported(uint32_t cin, uint32_t cout, uint32_t ldo) {
    return cout == kCout && ldo == kCout && cin && cin % 64 == 0 && cin <= 4096;
}

int launch_conv3x3_halo(void* out, const void* in, const void* weight, const float* bias, bool bf16, uint32_t batch,
                        uint32_t h, uint32_t w, uint32_t cin, cudaStream_t st) {
    if (!conv3x3_halo_supported(cin, kCout, kCout) || !batch || !h || !w)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv3x3_halo: input channels must be a multiple of 64");
    if (reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(weight) % 16 ||
        reinterpret_cast<uintptr_t>(bias) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv3x3_halo: buffers must be 16-byte aligned");
    std::call_once(g_conv_enc_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_conv_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_conv_enc) return set_error(DAV2CUDA_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
    const CUtensorMapDataType dt = bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    // input [batch][h][w][cin]: box = 64 channels x 130 pixels x 4 rows x 1 image
    CUtensorMap tm_in, tm_w;
    const cuuint64_t dims_in[4] = {cin, w, h, batch};
    const cuuint64_t str_in[3] = {(cuuint64_t)cin * 2, (cuuint64_t)w * cin * 2, (cuuint64_t)h * w * cin * 2};
    const cuuint32_t box_in[4] = {64, kHaloPixels, kHaloRows, 1};
    // weights [128][9 * cin]: box = 64 input channels x 128 output channels
    const cuuint64_t dims_w[2] = {(cuuint64_t)9 * cin, kCout};
    const cuuint64_t str_w[1] = {(cuuint64_t)9 * cin * 2};
    const cuuint32_t box_w[2] = {64, kCout};
    if (g_conv_enc(&tm_in, dt, 4, const_cast<void*>(in), dims_in, str_in, box_in, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        g_conv_enc(&tm_w, dt, 2, const_cast<void*>(weight), dims_w, str_w, box_w, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv3x3_halo: tensor map encoding failed");
    auto kernel = bf16 ? conv3x3_halo_kernel<true> : conv3x3_halo_kernel<false>;
    static std::atomic<uint64_t> configured[2];  // one bit per device ordinal, per operand type
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured_on(configured[bf16], dev)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess)
            return set_error(DAV2CUDA_LAUNCH_FAILED, "conv3x3_halo: cannot set shared memory size");
        mark_configured(configured[bf16], dev);
    }
    ConvParams p;
    p.batch = batch;
    p.h = h;
    p.w = w;
    p.cin = cin;
    p.tiles_x = (w + 127) / 128;
    p.tiles_y = (h + 1) / 2;
    const uint64_t tiles = (uint64_t)batch * p.tiles_y * p.tiles_x;
    if (tiles > 0xFFFFFFFFull) return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv3x3_halo: too many tiles");
    p.tiles = (uint32_t)tiles;
    p.bias = bias;
    p.out = out;
    p.err = device_error_word();
    if (!p.err) return set_error(DAV2CUDA_INTERNAL_ERROR, "conv3x3_halo: no device error word");
    const int sms = sm_count(dev);
    if (sms <= 0) return set_error(DAV2CUDA_LAUNCH_FAILED, "conv3x3_halo: cannot query the SM count");
    const uint32_t grid = p.tiles < (uint32_t)sms ? p.tiles : (uint32_t)sms;
    kernel<<<grid, kThreads, kSmem, st>>>(tm_in, tm_w, p);
    return check_launch("conv3x3_halo");
}

}  // namespace dav2cuda
