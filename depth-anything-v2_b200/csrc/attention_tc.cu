// Flash attention on tcgen05 tensor cores (head dim 64, f16 operands, f32
// accumulation) — attention_head64 of the reference (src/operators.cpp:
// 1098-1209: QK^T*0.125 -> softmax_lastdim.glsl -> PV) without materialising
// the [heads, T, T] scores.
//
// One CTA = one (image, head, 128-query tile), 320 threads; two CTAs share
// an SM.
//   warp 0      TMA: Q tile once, then K_j / V_j (128 keys x 64 dims each) into
//               a 2-stage ring. The 3-D tensor map over qkv [B][T][3E] zero-
//               fills rows past T.
//   warp 1      MMA issuer: S = Q K_j^T (M=128, N=128, K=64) into TMEM columns
//               0..127; once P_j is published it queues S_{j+1} first, then
//               O_j = P_j V_j (M=128, N=64, K=128; V read as an MN-major
//               operand) into TMEM columns 128 + 64*(j%2).
//   warps 2..9  softmax, two warps per query row (TMEM lane), 64 keys each
//               (maxima and sums combined through shared memory): pass 1 over S for
//               the row maximum, pass 2 for exp2(s*c - m) -> P_j (f16) written
//               to a 128-byte-swizzled shared tile, row sum l; then O_{j-1}
//               (complete by then) is read from TMEM and accumulated in
//               registers with the running correction
//               o = o*exp2(m_old - m_new) + O. Finally o / l.
// Ordering between the roles uses mbarriers; every wait is bounded and a
// timeout sets the device error word instead of hanging.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace dav2cuda {
namespace {

struct AttnParams {
    uint32_t tokens, heads, num_kb;
    uint64_t out_ld;
    __half* out;
    int* err;
};

constexpr uint32_t kQ = 128;          // queries per CTA
constexpr uint32_t kKV = 128;         // keys per block
constexpr uint32_t kTile = 128 * 128; // bytes of a 128 x 64 f16 tile
// Q, K[2], V[2], P (2 atoms), 16 barriers, 512 B maxima exchange. Two CTAs
// (each + 1 KB reserved) must fit the SM's 228 KB.
constexpr uint32_t kSmem = kTile * (1 + 2 + 2 + 2) + 128 + 512;

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

__global__ void __launch_bounds__(320, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm, const AttnParams p) {
    extern __shared__ uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if ((smem_addr(smem) & 1023u) != 0) {  // the 128-byte swizzle needs 1 KB aligned tiles
        if (threadIdx.x == 0) atomicExch(p.err, 2);
        return;
    }
    uint8_t* sQ = smem;
    uint8_t* sK = smem + kTile;
    uint8_t* sV = smem + 3 * kTile;
    uint8_t* sP = smem + 5 * kTile;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * kTile);
    uint64_t* q_full = bars + 0;
    uint64_t* kv_full = bars + 1;   // [2]
    uint64_t* kv_empty = bars + 3;  // [2]
    uint64_t* s_full = bars + 5;
    uint64_t* s_empty = bars + 6;
    uint64_t* p_full = bars + 7;
    uint64_t* p_empty = bars + 8;
    uint64_t* o_full = bars + 9;    // [2]
    uint64_t* o_empty = bars + 11;  // [2]
    uint64_t* drain = bars + 13;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bars + 15);
    __half* red = reinterpret_cast<__half*>(bars + 16);  // [2 halves][128 rows] row maxima (f16, rounded up)

    const uint32_t q0 = blockIdx.x * kQ, head = blockIdx.y, img = blockIdx.z;
    const uint32_t E = p.heads * 64u;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm);
        mbar_init(q_full, 1);
        mbar_init(&kv_full[0], 1);
        mbar_init(&kv_full[1], 1);
        mbar_init(&kv_empty[0], 1);
        mbar_init(&kv_empty[1], 1);
        mbar_init(s_full, 1);
        mbar_init(s_empty, 8);
        mbar_init(p_full, 8);
        mbar_init(p_empty, 1);
        mbar_init(&o_full[0], 1);
        mbar_init(&o_full[1], 1);
        mbar_init(&o_empty[0], 8);
        mbar_init(&o_empty[1], 8);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t nkb = p.num_kb;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, kTile);
            tma_load_3d(sQ, &tm, q_full, (int)(head * 64u), (int)q0, (int)img);
            for (uint32_t j = 0; j < nkb && !*abort_flag; ++j) {
                const uint32_t st = j & 1u;
                if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1u) ^ 1u, abort_flag, p.err)) break;
                mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
                tma_load_3d(sK + st * kTile, &tm, &kv_full[st], (int)(E + head * 64u), (int)(j * kKV), (int)img);
                tma_load_3d(sV + st * kTile, &tm, &kv_full[st], (int)(2 * E + head * 64u), (int)(j * kKV), (int)img);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = make_idesc(1u, 0u, 128u, 128u);
            constexpr uint32_t idesc_o = make_idesc(1u, 0u, 128u, 64u) | (1u << 16);  // B (V) MN-major
            const uint32_t q_addr = smem_addr(sQ), p_addr = smem_addr(sP);
            auto issue_s = [&](uint32_t j) {
                const uint32_t k_addr = smem_addr(sK + (j & 1u) * kTile);
#pragma unroll
                for (uint32_t kk = 0; kk < 4; ++kk)
                    umma<false>(tmem, smem_desc_sw128(q_addr + 32u * kk), smem_desc_sw128(k_addr + 32u * kk), idesc_s,
                                kk ? 1u : 0u);
                umma_commit(s_full);
            };
            bool ok = mbar_wait(q_full, 0, abort_flag, p.err) && mbar_wait(&kv_full[0], 0, abort_flag, p.err);
            if (ok) {
                tc_fence_after();
                issue_s(0);
                mma_issued = true;
            }
            for (uint32_t j = 0; ok && j < nkb; ++j) {
                // P_j ready (softmax also released S_j): queue S_{j+1} first so
                // the softmax warps can start on it, then O_j = P_j V_j.
                ok = mbar_wait(p_full, j & 1u, abort_flag, p.err);
                if (!ok) break;
                if (j + 1 < nkb) {
                    ok = mbar_wait(&kv_full[(j + 1) & 1u], ((j + 1) >> 1) & 1u, abort_flag, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                // O buffer j%2 was last used by block j-2
                ok = mbar_wait(&o_empty[j & 1u], ((j >> 1) & 1u) ^ 1u, abort_flag, p.err);
                if (!ok) break;
                tc_fence_after();
                const uint32_t v_addr = smem_addr(sV + (j & 1u) * kTile);
#pragma unroll
                for (uint32_t kk = 0; kk < 8; ++kk)
                    umma<false>(tmem + 128u + 64u * (j & 1u),
                                smem_desc_sw128(p_addr + (kk >> 2) * kTile + 32u * (kk & 3u)),
                                desc_mn_sw128(v_addr + kk * 2048u), idesc_o, kk ? 1u : 0u);
                umma_commit(&o_full[j & 1u]);
                umma_commit(p_empty);
                umma_commit(&kv_empty[j & 1u]);
            }
        }
    } else {
        // softmax: two warps per TMEM lane quarter; `half` selects keys
        // [64*half, 64*half+64) of S and dims [32*half, 32*half+32) of O.
        const uint32_t quarter = warp & 3u;
        const uint32_t half = (warp - 2u) >> 2;
        const uint32_t row = quarter * 32u + lane;
        const uint32_t lane_base = (quarter * 32u) << 16;
        const uint32_t bar_id = 1u + quarter;  // named barrier shared by the two warps of a quarter
        const float c = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
        float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
        bool ok = true;
        // literal barrier ids (1..4) keep the CTA's named-barrier count small
        auto pair_sync = [&]() {
            switch (bar_id) {
                case 1: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
                case 2: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
                case 3: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
                default: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
            }
        };
        auto accumulate = [&](uint32_t b, float alpha_b) -> bool {
            if (!mbar_wait(&o_full[b & 1u], (b >> 1) & 1u, abort_flag, p.err)) return false;
            tc_fence_after();
            float ov[32];
            tmem_ld_x32(tmem + lane_base + 128u + 64u * (b & 1u) + 32u * half, ov);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = fmaf(o[i], alpha_b, ov[i]);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_empty[b & 1u]);
            return true;
        };
        for (uint32_t j = 0; j < nkb; ++j) {
            if (!mbar_wait(s_full, j & 1u, abort_flag, p.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t kbase = j * kKV + 64u * half;
            // pass 1: maximum over this warp's 64 keys, combined with the partner
            float mx = m;
#pragma unroll 1
            for (uint32_t cc = 0; cc < 2; ++cc) {
                float s[32];
                tmem_ld_x32(tmem + lane_base + 64u * half + cc * 32u, s);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (kbase + cc * 32u + i < p.tokens) mx = fmaxf(mx, s[i]);
            }
            // common row maximum: both warps round their partial maximum up to
            // f16, exchange it and take the larger, so they use the identical
            // value (>= the true maximum: every exp2 argument stays <= 0)
            const __half mine = __float2half_ru(mx);
            red[half * 128u + row] = mine;
            pair_sync();
            mx = __half2float(__hmax(mine, red[(half ^ 1u) * 128u + row]));
            pair_sync();  // both have read before the next block overwrites
            const float alpha = ex2_approx((m - mx) * c);  // 0 on the first block
            m = mx;
            const float mc = m * c;
            if (!mbar_wait(p_empty, (j & 1u) ^ 1u, abort_flag, p.err)) {
                ok = false;
                break;
            }
            // pass 2: P = exp2(s*c - m*c) for the 64 keys (one swizzled atom)
            float ls = 0.f;
            uint8_t* atom = sP + half * kTile + row * 128u;
#pragma unroll 1
            for (uint32_t cc = 0; cc < 2; ++cc) {
                float s[32];
                tmem_ld_x32(tmem + lane_base + 64u * half + cc * 32u, s);
                uint32_t h[16];
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                    const float p0 = kbase + cc * 32u + i < p.tokens ? ex2_approx(fmaf(s[i], c, -mc)) : 0.f;
                    const float p1 = kbase + cc * 32u + i + 1 < p.tokens ? ex2_approx(fmaf(s[i + 1], c, -mc)) : 0.f;
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
            l = l * alpha + ls;
            tc_fence_before();
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(s_empty);
                mbar_arrive(p_full);
            }
            if (j > 0 && !accumulate(j - 1, alpha_prev)) {
                ok = false;
                break;
            }
            alpha_prev = alpha;
        }
        if (ok && nkb > 0) ok = accumulate(nkb - 1, alpha_prev);
        // row sum = both halves' partial sums (same maximum); the P tile is
        // free once the last O MMA has completed
        float* lx = reinterpret_cast<float*>(sP);
        lx[half * 128u + row] = l;
        pair_sync();
        l += lx[(half ^ 1u) * 128u + row];
        if (ok && q0 + row < p.tokens) {
            const float inv = 1.0f / fmaxf(l, 1.0e-20f);
            __half* dst = p.out + ((uint64_t)img * p.tokens + q0 + row) * p.out_ld + head * 64u + half * 32u;
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
        tmem_dealloc(tmem, 256);
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
        if (getenv("DAV2CUDA_VERBOSE")) {
            int blocks = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, attention_tc_kernel, 320, kSmem);
            fprintf(stderr, "[dav2cuda] attention_tc: %u B shared memory, %d CTAs per SM\n", kSmem, blocks);
        }
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
    attention_tc_kernel<<<grid, 320, kSmem, st>>>(tm, p);
    return check_launch("attention_tc");
}

}  // namespace dav2cuda
