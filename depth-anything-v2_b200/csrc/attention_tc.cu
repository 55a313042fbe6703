// Flash attention on tcgen05 tensor cores (head dim 64, f16 operands, f32
// accumulation) — attention_head64 of the reference (src/operators.cpp:
// 1098-1209: QK^T*0.125 -> softmax_lastdim.glsl -> PV) without materialising
// the [heads, T, T] scores.
//
// One CTA = one (image, head, 256-query block) = two 128-query tiles that
// share every K/V block; 576 threads, one CTA per SM (a kernel that allocates
// tensor memory is resident once per SM), all 512 TMEM columns:
// tile t uses columns 256t + [0,128) for S and 256t + 128 + 64*(j%2) for O_j.
//   warp 0       TMA: the Q tiles once, then K_j / V_j (128 keys x 64 dims
//                each) into a 3-stage ring. The 3-D tensor map over qkv
//                [B][T][3E] zero-fills rows past T.
//   warp 1       MMA issuer, alternating the tiles: S = Q K_j^T (M=128, N=128,
//                K=64); once tile t has published P_j it queues S_{j+1} of that
//                tile first, then O_j = P_j V_j (M=128, N=64, K=128; V read as an
//                MN-major operand). While one tile's softmax runs, the tensor
//                core works for the other.
//   warps 2..9   softmax of tile 0, warps 10..17 of tile 1: two warps per
//                query row (TMEM lane), 64 keys each (row maxima combined
//                through shared memory): pass 1 over S for the row maximum,
//                pass 2 for exp2(s*c - m) -> P_j (f16) written to a 128-byte-
//                swizzled shared tile, row sum l; then O_{j-1} (complete by
//                then) is read from TMEM and accumulated in registers with the
//                running correction o = o*exp2(m_old - m_new) + O. Full key
//                blocks skip the key-range mask. Finally o / l.
// Ordering between the roles uses mbarriers; every wait is bounded and a
// timeout sets the device error word instead of hanging.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>
#include <type_traits>

namespace dav2cuda {
namespace {

struct AttnParams {
    uint32_t tokens, heads, num_kb;
    uint64_t out_ld;
    __half* out;
    int* err;
};

constexpr uint32_t kQTiles = 2;       // 128-query tiles per CTA
constexpr uint32_t kQ = 128 * kQTiles;  // queries per CTA
constexpr uint32_t kKV = 128;         // keys per block
constexpr uint32_t kStages = 3;       // K/V ring depth
constexpr uint32_t kTile = 128 * 128; // bytes of a 128 x 64 f16 tile
constexpr uint32_t kThreads = 64 + 256 * kQTiles;
// Q[2], K[3], V[3], P[2 tiles][2 atoms], 1 KB barriers, 1 KB maxima exchange
constexpr uint32_t kSmem = kTile * (kQTiles + 2 * kStages + 2 * kQTiles) + 2048;

__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr) {
    // MN-major operand, 128-byte swizzle: 8-row (K) groups 1024 B apart.
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm, const AttnParams p) {
    extern __shared__ uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if ((smem_addr(smem) & 1023u) != 0) {  // the 128-byte swizzle needs 1 KB aligned tiles
        if (threadIdx.x == 0) atomicExch(p.err, 2);
        return;
    }
    uint8_t* sQ = smem;                                // [tile]
    uint8_t* sK = smem + kQTiles * kTile;              // [stage]
    uint8_t* sV = sK + kStages * kTile;                // [stage]
    uint8_t* sP = sV + kStages * kTile;                // [tile][2 atoms]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kQTiles * kTile);
    uint64_t* q_full = bars + 0;     // [tile]
    uint64_t* kv_full = bars + 2;    // [stage]
    uint64_t* kv_empty = bars + 5;   // [stage]
    uint64_t* s_full = bars + 8;     // [tile]
    uint64_t* p_full = bars + 10;    // [tile]
    uint64_t* p_empty = bars + 12;   // [tile]
    uint64_t* o_full = bars + 14;    // [tile][2]
    uint64_t* o_empty = bars + 18;   // [tile][2]
    uint64_t* drain = bars + 22;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 24);
    __half* red = reinterpret_cast<__half*>(bars + 128);  // [tile][half][128 rows] row maxima (f16, rounded up)

    const uint32_t q0 = blockIdx.x * kQ, head = blockIdx.y, img = blockIdx.z;
    const uint32_t E = p.heads * 64u;
    const uint32_t ntiles = (p.tokens - q0 + 127u) / 128u >= kQTiles ? kQTiles : (p.tokens - q0 + 127u) / 128u;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm);
        for (uint32_t t = 0; t < kQTiles; ++t) {
            mbar_init(&q_full[t], 1);
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 8);
            mbar_init(&p_empty[t], 1);
            mbar_init(&o_full[2 * t], 1);
            mbar_init(&o_full[2 * t + 1], 1);
            mbar_init(&o_empty[2 * t], 8);
            mbar_init(&o_empty[2 * t + 1], 8);
        }
        for (uint32_t st = 0; st < kStages; ++st) {
            mbar_init(&kv_full[st], 1);
            mbar_init(&kv_empty[st], 1);
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
    const uint32_t nkb = p.num_kb;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            for (uint32_t t = 0; t < ntiles; ++t) {
                mbar_arrive_expect_tx(&q_full[t], kTile);
                tma_load_3d(sQ + t * kTile, &tm, &q_full[t], (int)(head * 64u), (int)(q0 + 128u * t), (int)img);
            }
            for (uint32_t j = 0; j < nkb && !*abort_flag; ++j) {
                const uint32_t st = j % kStages;
                if (!mbar_wait(&kv_empty[st], ((j / kStages) & 1u) ^ 1u, abort_flag, p.err)) break;
                mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
                tma_load_3d(sK + st * kTile, &tm, &kv_full[st], (int)(E + head * 64u), (int)(j * kKV), (int)img);
                tma_load_3d(sV + st * kTile, &tm, &kv_full[st], (int)(2 * E + head * 64u), (int)(j * kKV), (int)img);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = make_idesc(1u, 0u, 128u, 128u);
            constexpr uint32_t idesc_o = make_idesc(1u, 0u, 128u, 64u) | (1u << 16);  // B (V) MN-major
            auto issue_s = [&](uint32_t t, uint32_t j) {
                const uint32_t q_addr = smem_addr(sQ + t * kTile);
                const uint32_t k_addr = smem_addr(sK + (j % kStages) * kTile);
#pragma unroll
                for (uint32_t kk = 0; kk < 4; ++kk)
                    umma<false>(tmem + 256u * t, smem_desc_sw128(q_addr + 32u * kk), smem_desc_sw128(k_addr + 32u * kk),
                                idesc_s, kk ? 1u : 0u);
                umma_commit(&s_full[t]);
            };
            auto issue_o = [&](uint32_t t, uint32_t j) {
                const uint32_t p_addr = smem_addr(sP + 2u * t * kTile);
                const uint32_t v_addr = smem_addr(sV + (j % kStages) * kTile);
#pragma unroll
                for (uint32_t kk = 0; kk < 8; ++kk)
                    umma<false>(tmem + 256u * t + 128u + 64u * (j & 1u),
                                smem_desc_sw128(p_addr + (kk >> 2) * kTile + 32u * (kk & 3u)),
                                desc_mn_sw128(v_addr + kk * 2048u), idesc_o, kk ? 1u : 0u);
                umma_commit(&o_full[2 * t + (j & 1u)]);
                umma_commit(&p_empty[t]);
            };
            bool ok = mbar_wait(&kv_full[0], 0, abort_flag, p.err);
            for (uint32_t t = 0; ok && t < ntiles; ++t) {
                ok = mbar_wait(&q_full[t], 0, abort_flag, p.err);
                if (!ok) break;
                tc_fence_after();
                issue_s(t, 0);
                mma_issued = true;
            }
            for (uint32_t j = 0; ok && j < nkb; ++j) {
                if (j + 1 < nkb) {
                    ok = mbar_wait(&kv_full[(j + 1) % kStages], ((j + 1) / kStages) & 1u, abort_flag, p.err);
                    if (!ok) break;
                }
                for (uint32_t t = 0; ok && t < ntiles; ++t) {
                    // P_j of tile t ready (its softmax has also finished reading S_j):
                    // queue S_{j+1} first so that softmax can start on it, then O_j.
                    ok = mbar_wait(&p_full[t], j & 1u, abort_flag, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    if (j + 1 < nkb) issue_s(t, j + 1);
                    // O buffer j%2 of tile t was last used by block j-2
                    ok = mbar_wait(&o_empty[2 * t + (j & 1u)], ((j >> 1) & 1u) ^ 1u, abort_flag, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    issue_o(t, j);
                }
                if (ok) umma_commit(&kv_empty[j % kStages]);
            }
        }
    } else if ((warp - 2u) / 8u < ntiles) {
        // softmax: two warps per TMEM lane quarter of tile t; `half` selects keys
        // [64*half, 64*half+64) of S and dims [32*half, 32*half+32) of O.
        const uint32_t t = (warp - 2u) / 8u;
        const uint32_t quarter = warp & 3u;
        const uint32_t half = ((warp - 2u) >> 2) & 1u;
        const uint32_t row = quarter * 32u + lane;
        const uint32_t tb = tmem + 256u * t + ((quarter * 32u) << 16);
        const uint32_t pair_id = t * 4u + quarter;  // named barrier 1 + pair_id, shared by the two warps
        const float c = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        __half* my_red = red + (2u * t + half) * 128u + row;
        __half* partner_red = red + (2u * t + (half ^ 1u)) * 128u + row;
        uint8_t* atom = sP + (2u * t + half) * kTile + row * 128u;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
        float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
        bool ok = true;
        // literal barrier ids keep the CTA's named-barrier count small
        auto pair_sync = [&]() {
            switch (pair_id) {
                case 0: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
                case 1: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
                case 2: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
                case 3: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
                case 4: asm volatile("bar.sync 5, 64;" ::: "memory"); break;
                case 5: asm volatile("bar.sync 6, 64;" ::: "memory"); break;
                case 6: asm volatile("bar.sync 7, 64;" ::: "memory"); break;
                default: asm volatile("bar.sync 8, 64;" ::: "memory"); break;
            }
        };
        auto accumulate = [&](uint32_t b, float alpha_b) -> bool {
            if (!mbar_wait(&o_full[2 * t + (b & 1u)], (b >> 1) & 1u, abort_flag, p.err)) return false;
            tc_fence_after();
            float ov[32];
            tmem_ld_x32(tb + 128u + 64u * (b & 1u) + 32u * half, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], alpha_b, ov[i]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_empty[2 * t + (b & 1u)]);
            return true;
        };
        // pass 1 / pass 2 over this warp's 64 keys; kMask limits them to keys < T
        auto row_max = [&](auto mask_tag, uint32_t kbase, float mx) -> float {
            constexpr bool kMask = decltype(mask_tag)::value;
#pragma unroll 1
            for (uint32_t cc = 0; cc < 2; ++cc) {
                float s[32];
                tmem_ld_x32(tb + 64u * half + cc * 32u, s);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (!kMask || kbase + cc * 32u + i < p.tokens) mx = fmaxf(mx, s[i]);
            }
            return mx;
        };
        auto exp_pass = [&](auto mask_tag, uint32_t kbase, float mc) -> float {
            constexpr bool kMask = decltype(mask_tag)::value;
            float ls = 0.f;
#pragma unroll 1
            for (uint32_t cc = 0; cc < 2; ++cc) {
                float s[32];
                tmem_ld_x32(tb + 64u * half + cc * 32u, s);
                uint32_t h[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    float p0 = ex2_approx(fmaf(s[i], c, -mc));
                    float p1 = ex2_approx(fmaf(s[i + 1], c, -mc));
                    if (kMask) {
                        if (kbase + cc * 32u + i >= p.tokens) p0 = 0.f;
                        if (kbase + cc * 32u + i + 1 >= p.tokens) p1 = 0.f;
                    }
                    ls += p0 + p1;
                    __half2 hh = __floats2half2_rn(p0, p1);
                    h[i >> 1] = *reinterpret_cast<uint32_t*>(&hh);
                }
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t chunk = cc * 4u + q;
                    *reinterpret_cast<uint4*>(atom + ((chunk ^ (row & 7u)) << 4)) =
                        make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
                }
            }
            return ls;
        };
        for (uint32_t j = 0; j < nkb; ++j) {
            if (!mbar_wait(&s_full[t], j & 1u, abort_flag, p.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t kbase = j * kKV + 64u * half;
            const bool full = kbase + 64u <= p.tokens;
            float mx = full ? row_max(std::false_type{}, kbase, m) : row_max(std::true_type{}, kbase, m);
            // common row maximum: both warps round their partial maximum up to
            // f16, exchange it and take the larger, so they use the identical
            // value (>= the true maximum: every exp2 argument stays <= 0)
            const __half mine = __float2half_ru(mx);
            *my_red = mine;
            pair_sync();
            mx = __half2float(__hmax(mine, *partner_red));
            pair_sync();  // both have read before the next block overwrites
            const float alpha = ex2_approx((m - mx) * c);  // 0 on the first block
            m = mx;
            const float mc = m * c;
            // P of the previous block must have been consumed by its MMA
            if (!mbar_wait(&p_empty[t], (j & 1u) ^ 1u, abort_flag, p.err)) {
                ok = false;
                break;
            }
            const float ls = full ? exp_pass(std::false_type{}, kbase, mc) : exp_pass(std::true_type{}, kbase, mc);
            l = l * alpha + ls;
            tc_fence_before();
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[t]);
            // the previous block's O is complete by now (its P was released)
            if (j > 0 && !accumulate(j - 1, alpha_prev)) {
                ok = false;
                break;
            }
            alpha_prev = alpha;
        }
        if (ok && nkb > 0) ok = accumulate(nkb - 1, alpha_prev);
        // row sum = both halves' partial sums (same maximum); the tile's P
        // region is free once its last O MMA has completed
        float* lx = reinterpret_cast<float*>(sP + 2u * t * kTile);
        lx[half * 128u + row] = l;
        pair_sync();
        l += lx[(half ^ 1u) * 128u + row];
        const uint32_t qrow = q0 + 128u * t + row;
        if (ok && qrow < p.tokens) {
            const float inv = 1.0f / fmaxf(l, 1.0e-20f);
            __half* dst = p.out + ((uint64_t)img * p.tokens + qrow) * p.out_ld + head * 64u + half * 32u;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
                uint4 w;
                __half2 a = __floats2half2_rn(o[i] * inv, o[i + 1] * inv);
                __half2 b = __floats2half2_rn(o[i + 2] * inv, o[i + 3] * inv);
                __half2 cc2 = __floats2half2_rn(o[i + 4] * inv, o[i + 5] * inv);
                __half2 d = __floats2half2_rn(o[i + 6] * inv, o[i + 7] * inv);
                w.x = *reinterpret_cast<uint32_t*>(&a);
                w.y = *reinterpret_cast<uint32_t*>(&b);
                w.z = *reinterpret_cast<uint32_t*>(&cc2);
                w.w = *reinterpret_cast<uint32_t*>(&d);
                *reinterpret_cast<uint4*>(dst + i) = w;
            }
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

PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;
std::once_flag g_enc_once;

}  // namespace

int launch_attention_tc(__half* out, const __half* qkv, uint32_t batch, uint32_t tokens, uint32_t heads,
                        uint64_t qkv_ld, uint64_t out_ld, cudaStream_t st) {
    if (!tokens || !heads || !batch) return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: empty");
    if (qkv_ld != 3ull * heads * 64 || (qkv_ld * 2) % 16 || reinterpret_cast<uintptr_t>(qkv) % 16 || out_ld % 8 ||
        reinterpret_cast<uintptr_t>(out) % 16)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: misaligned or non-interleaved rows");
    std::call_once(g_enc_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_enc) return set_error(DAV2CUDA_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
    CUtensorMap tm;
    const cuuint64_t dims[3] = {qkv_ld, tokens, batch};
    const cuuint64_t strides[2] = {qkv_ld * 2, (cuuint64_t)tokens * qkv_ld * 2};
    const cuuint32_t box[3] = {64, 128, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult rc = g_enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(qkv), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: tensor map encoding failed");
    static uint64_t configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured >> (dev & 63) & 1ull)) {
        if (cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
                cudaSuccess ||
            cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return set_error(DAV2CUDA_LAUNCH_FAILED, "attention: cannot set shared memory size");
        configured |= 1ull << (dev & 63);
    }
    AttnParams p;
    p.tokens = tokens;
    p.heads = heads;
    p.num_kb = (tokens + kKV - 1) / kKV;
    p.out_ld = out_ld;
    p.out = out;
    p.err = device_error_word();
    if (!p.err) return set_error(DAV2CUDA_INTERNAL_ERROR, "attention: no device error word");
    dim3 grid((tokens + kQ - 1) / kQ, heads, batch);
    attention_tc_kernel<<<grid, kThreads, kSmem, st>>>(tm, p);
    return check_launch("attention_tc");
}

}  // namespace dav2cuda
