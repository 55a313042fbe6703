// The DPT output head's last two layers as one tcgen05 kernel (src/dpt.cpp:
// 830-854): output_conv2.0 (3x3, pad 1, Cp -> 32 channels, + bias), ReLU,
// output_conv2.2 (1x1, 32 -> 1, + bias), then ReLU (relative depth) or
// sigmoid * max_depth (metric), on channels-last 16-bit maps.
//
// With 32 output channels each MMA (M=128, N=32, K=16) reads as many A bytes
// as an N=256 one but does an eighth of the work, so the implicit-GEMM kernel
// that loads one shifted A tile per tap spends its time waiting on those
// loads. This kernel loads each input pixel once per tile instead: a tile is
// 128 consecutive output pixels of one image row, and per 64-channel chunk
// one TMA box brings the 3 x 130-pixel halo of the tile into shared memory as
// 128-byte pixel rows [row][pixel][64 channels] with the 128-byte swizzle
// (the K-major layout the MMA reads). Tap (dy, dx) is then the same rows seen
// from a base dy*130 + dx pixels further: an operand descriptor whose start is
// that pixel's row. The weights, packed in the same layout once per CTA, stay
// in shared memory.
//
// Roles (persistent, one CTA per SM): warp 0 TMA (halo planes into a ring of
// kStages chunk stages), warp 1 the MMA issuer (36 MMAs per chunk, two chunks
// per tile at Cp = 128, into one of two 32-column TMEM accumulators), warps
// 2..5 the head (one TMEM lane quarter each: relu(acc + b) . w + head_b per
// pixel, written to the depth map). Every wait is bounded; a timeout sets the
// device error word and the kernel drains and returns.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>

namespace dav2cuda {
namespace {

constexpr uint32_t kHaloPixels = 130;                    // 128 output pixels + left and right halo
constexpr uint32_t kHaloRows = 3;
constexpr uint32_t kChunkChannels = 64;                  // channels per stage: one 128-byte row per pixel
constexpr uint32_t kHaloBytes = kHaloRows * kHaloPixels * 128;  // 49920 per stage
constexpr uint32_t kStageBytes = 50176;                  // rounded to 1 KB (the swizzle pattern's period)
constexpr uint32_t kStages = 3;
constexpr uint32_t kCout = 32;
constexpr uint32_t kThreads = 6 * 32;
constexpr uint32_t kMaxCp = 128;                         // weights resident: 9 x Cp x 32 x 2 B
constexpr uint32_t kWeightBytes = 9 * kMaxCp * kCout * 2;  // 73728
constexpr uint32_t kSmem = kWeightBytes + kStages * kStageBytes + 1024 + 1024;  // + barriers + alignment slack
static_assert(kSmem <= 232448, "shared memory above the per-block limit");
static_assert(kStageBytes % 1024 == 0 && kStageBytes >= kHaloBytes, "stage size");

struct HeadParams {
    uint32_t batch, h, w, cp;  // input / output maps [batch][h][w][cp] -> [batch][h][w]
    uint32_t tiles_x, tiles;
    const uint16_t* weight;    // [32][9 * cp], column (ky*3 + kx)*cp + c
    const float* bias;         // [32]
    const float* head_w;       // [32]
    float head_b, head_max;
    uint32_t metric;
    float* out;
    float* const* out_slot;    // destination read from this device slot when set
    int* err;
};

// Shared-memory operand descriptor, K-major, 128-byte rows with the 128-byte
// swizzle (8-row groups 1 KB apart), for an operand that may start at any
// row of a 1 KB-aligned swizzled region: the MMA undoes the swizzle from the
// absolute address bits of each row, as TMA applied it, so the start needs no
// phase correction (base-offset field 0; a start row's phase written there
// was measured to misplace the rows).
__device__ __forceinline__ uint64_t desc_sw128_at(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    conv_head_halo_kernel(const __grid_constant__ CUtensorMap tm, const HeadParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 1 KB-aligned working area (the dynamic allocation carries 1 KB of slack)
    uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* sW = smem;                          // [tap][chunk][32 rows][128 B, swizzled]
    uint8_t* sA = smem + kWeightBytes;           // [stage][3 x 130 pixels][128 B, swizzled]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kStages * kStageBytes);
    uint64_t* full = bars;                       // [stage]
    uint64_t* empty = full + kStages;            // [stage]
    uint64_t* tfull = empty + kStages;           // [accumulator]
    uint64_t* tempty = tfull + 2;                // [accumulator]
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t chunks = p.cp / kChunkChannels;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm);
        for (uint32_t s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    // weights into the swizzled K-major layout: a 4 KB tile per (tap, chunk),
    // 16-byte unit j of row r at r*128 + ((j ^ (r & 7)) << 4)
    for (uint32_t u = threadIdx.x; u < 9 * chunks * kCout * 8; u += blockDim.x) {
        const uint32_t j = u & 7u, row = (u >> 3) % kCout, tc = (u >> 3) / kCout, c = tc % chunks, tap = tc / chunks;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(p.weight + (uint64_t)row * 9 * p.cp + tap * p.cp +
                                                             c * kChunkChannels + j * 8));
        *reinterpret_cast<uint4*>(sW + (size_t)(tc * kCout + row) * 128 + ((j ^ (row & 7u)) << 4)) = v;
    }
    fence_async_smem();
    if (warp == 1) tmem_alloc(tmem_slot, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t g = 0;  // chunk stages filled (all tiles)
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
                const uint32_t xt = t % p.tiles_x, row = t / p.tiles_x;
                const uint32_t y = row % p.h, img = row / p.h;
                for (uint32_t c = 0; c < chunks; ++c, ++g) {
                    const uint32_t s = g % kStages;
                    if (!mbar_wait(&empty[s], ((g / kStages) & 1u) ^ 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kHaloBytes);
                    tma_load_4d(sA + s * kStageBytes, &tm, &full[s], (int)(c * kChunkChannels), (int)(xt * 128u) - 1,
                                (int)y - 1, (int)img);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc(1u, kBF16 ? 1u : 0u, 128u, kCout);
            const uint32_t a0 = smem_addr(sA), w0 = smem_addr(sW);
            uint32_t g = 0, local = 0;
            bool ok = true;
            for (uint32_t t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++local) {
                const uint32_t buf = local & 1u;
                // the head has read this accumulator's previous tile
                if (!mbar_wait(&tempty[buf], ((local >> 1) & 1u) ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                for (uint32_t c = 0; c < chunks; ++c, ++g) {
                    const uint32_t s = g % kStages;
                    if (!mbar_wait(&full[s], (g / kStages) & 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t stage = a0 + s * kStageBytes;
#pragma unroll
                    for (uint32_t tap = 0; tap < 9; ++tap) {
                        // A: the tap's base pixel row of the stage; B: the (tap, chunk) weight tile
                        const uint32_t arow = stage + ((tap / 3) * kHaloPixels + tap % 3) * 128u;
                        const uint32_t brow = w0 + (tap * chunks + c) * (kCout * 128u);
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; ++kk)  // 16 channels per MMA
                            umma<false>(tmem + buf * kCout, desc_sw128_at(arow + 32u * kk),
                                        desc_sw128_at(brow + 32u * kk), idesc, (c | tap | kk) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);
                    mma_issued = true;
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else {
        // head: warp w reads TMEM lanes 32*(w%4) .. +31 (pixels of the tile)
        const uint32_t quarter = warp & 3u;
        const bool metric = p.metric != 0;
        float* dst = nullptr;
        uint32_t local = 0;
        for (uint32_t t = blockIdx.x; t < p.tiles; t += gridDim.x, ++local) {
            const uint32_t buf = local & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], (local >> 1) & 1u, abort_flag, p.err))) break;
            tc_fence_after();
            uint32_t acc[32];
            tmem_ld_32x32b_x32(tmem + ((quarter * 32u) << 16) + buf * kCout, acc);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            if (dst == nullptr) dst = p.out_slot ? *p.out_slot : p.out;
            const uint32_t xt = t % p.tiles_x, row = t / p.tiles_x;
            const uint32_t x = xt * 128u + quarter * 32u + lane;
            float d = 0.f;
#pragma unroll
            for (int g4 = 0; g4 < 8; ++g4) {
                const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.bias) + g4);
                const float4 w4 = __ldg(reinterpret_cast<const float4*>(p.head_w) + g4);
                const float bs[4] = {b4.x, b4.y, b4.z, b4.w}, ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float v = __fadd_rn(__uint_as_float(acc[4 * g4 + k]), bs[k]);
                    d = fmaf(fmaxf(v, 0.0f), ws[k], d);
                }
            }
            d += p.head_b;
            d = metric ? p.head_max / (1.0f + expf(-d)) : fmaxf(d, 0.0f);
            if (x < p.w) dst[(uint64_t)row * p.w + x] = d;
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
        tmem_dealloc(tmem, 64);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_head_enc = nullptr;
std::once_flag g_head_enc_once;

}  // namespace

bool conv_head_halo_supported(uint32_t cp, uint32_t cout) {
    return cout == kCout && cp && cp % kChunkChannels == 0 && cp <= kMaxCp;
}

int launch_conv_head_halo(float* out, float* const* out_slot, const void* in, const void* weight, const float* bias,
                          const float* head_w, float head_b, float head_max, bool metric, bool bf16, uint32_t batch,
                          uint32_t h, uint32_t w, uint32_t cp, cudaStream_t st) {
    if (!conv_head_halo_supported(cp, kCout) || !batch || !h || !w)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv_head_halo: channels must be 64 or 128");
    if (reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(weight) % 16 ||
        reinterpret_cast<uintptr_t>(bias) % 16 || reinterpret_cast<uintptr_t>(head_w) % 16)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv_head_halo: buffers must be 16-byte aligned");
    std::call_once(g_head_enc_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_head_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_head_enc) return set_error(DAV2CUDA_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
    // [batch][h][w][cp] 16-bit, box = 64 channels x 130 pixels x 3 rows x 1 image,
    // 128-byte swizzle: the box lands as [row][pixel][64 channels]
    CUtensorMap tm;
    const cuuint64_t dims[4] = {cp, w, h, batch};
    const cuuint64_t strides[3] = {(cuuint64_t)cp * 2, (cuuint64_t)w * cp * 2, (cuuint64_t)h * w * cp * 2};
    const cuuint32_t box[4] = {kChunkChannels, kHaloPixels, kHaloRows, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (g_head_enc(&tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(in), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv_head_halo: tensor map encoding failed");
    auto kernel = bf16 ? conv_head_halo_kernel<true> : conv_head_halo_kernel<false>;
    static std::atomic<uint64_t> configured[2];  // one bit per device ordinal, per operand type
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured_on(configured[bf16], dev)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess)
            return set_error(DAV2CUDA_LAUNCH_FAILED, "conv_head_halo: cannot set shared memory size");
        mark_configured(configured[bf16], dev);
    }
    HeadParams p;
    p.batch = batch;
    p.h = h;
    p.w = w;
    p.cp = cp;
    p.tiles_x = (w + 127) / 128;
    const uint64_t tiles = (uint64_t)batch * h * p.tiles_x;
    if (tiles > 0xFFFFFFFFull) return set_error(DAV2CUDA_INVALID_ARGUMENT, "conv_head_halo: too many tiles");
    p.tiles = (uint32_t)tiles;
    p.weight = static_cast<const uint16_t*>(weight);
    p.bias = bias;
    p.head_w = head_w;
    p.head_b = head_b;
    p.head_max = head_max;
    p.metric = metric ? 1u : 0u;
    p.out = out;
    p.out_slot = out_slot;
    p.err = device_error_word();
    if (!p.err) return set_error(DAV2CUDA_INTERNAL_ERROR, "conv_head_halo: no device error word");
    const int sms = sm_count(dev);
    if (sms <= 0) return set_error(DAV2CUDA_LAUNCH_FAILED, "conv_head_halo: cannot query the SM count");
    const uint32_t grid = p.tiles < (uint32_t)sms ? p.tiles : (uint32_t)sms;
    kernel<<<grid, kThreads, kSmem, st>>>(tm, p);
    return check_launch("conv_head_halo");
}

}  // namespace dav2cuda
