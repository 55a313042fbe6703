// Fused multi-head attention for head_dim 64 (the reference's
// attention_head64: src/operators.cpp:1098-1209, bmm.glsl score/value modes
// and softmax_lastdim.glsl), written flash-style so the [heads, N, N] score
// matrix never reaches HBM:
//
//   for each 64-query block of one (image, head):
//     for each 64-key block: S = Q K^T (tensor cores, fp32 accumulate),
//       online softmax of S * 0.125 in registers (running max / sum),
//       O += P V (P re-used from the S registers as the A operand)
//     O /= sum
//
// Input is the interleaved QKV matrix [tokens, 3*heads*64] (q | k | v),
// output is token-major [tokens, heads*64] — the reference layouts. K/V
// tiles are double-buffered in shared memory with cp.async and an XOR
// swizzle of the 16-byte chunks so ldmatrix is bank-conflict free.
#include "kernels.cuh"

namespace dav2cuda {
namespace {

constexpr int kBM = 64;   // queries per CTA (4 warps x 16 rows)
constexpr int kBN = 64;   // keys per iteration
constexpr int kD = 64;    // head dim

__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
    const uint32_t n = pred ? 16u : 0u;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

template <bool kBF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (kBF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (kBF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

template <typename H>
__global__ void __launch_bounds__(128) attention_kernel(H* __restrict__ out, const H* __restrict__ qkv,
                                                        uint32_t tokens, uint32_t heads, uint64_t qkv_ld,
                                                        uint64_t out_ld) {
    constexpr bool kBF16 = std::is_same<H, __nv_bfloat16>::value;
    __shared__ __align__(128) uint8_t sQ[kBM * 128];
    __shared__ __align__(128) uint8_t sK[2][kBN * 128];
    __shared__ __align__(128) uint8_t sV[2][kBN * 128];

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t q0 = blockIdx.x * kBM;
    const uint32_t head = blockIdx.y;
    const uint64_t img = blockIdx.z;
    const uint64_t E = (uint64_t)heads * kD;
    const H* base = qkv + img * tokens * qkv_ld;
    const H* qb = base + head * kD;
    const H* kb = base + E + head * kD;
    const H* vb = base + 2 * E + head * kD;

    // Q tile: 64 rows x 8 chunks of 16 B; 128 threads x 4 chunks.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t idx = tid + 128u * i;
        const uint32_t row = idx >> 3, ch = idx & 7u;
        const uint32_t q = q0 + row;
        const bool ok = q < tokens;
        cp_async16(smem_addr(sQ) + swz(row, ch), qb + (uint64_t)(ok ? q : 0) * qkv_ld + ch * 8, ok);
    }
    auto load_kv = [&](int stage, uint32_t k0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t idx = tid + 128u * i;
            const uint32_t row = idx >> 3, ch = idx & 7u;
            const uint32_t kk = k0 + row;
            const bool ok = kk < tokens;
            const uint64_t off = (uint64_t)(ok ? kk : 0) * qkv_ld + ch * 8;
            cp_async16(smem_addr(sK[stage]) + swz(row, ch), kb + off, ok);
            cp_async16(smem_addr(sV[stage]) + swz(row, ch), vb + off, ok);
        }
    };
    load_kv(0, 0);
    cp_commit();

    const uint32_t num_kb = (tokens + kBN - 1) / kBN;
    const float scale_log2 = 0.125f * 1.4426950408889634f;

    uint32_t qf[4][4];  // Q fragments for the 4 k-steps of 16 dims
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};

    const uint32_t mi = lane >> 3, r8 = lane & 7u;

    for (uint32_t jb = 0; jb < num_kb; ++jb) {
        const int stage = jb & 1;
        if (jb + 1 < num_kb) {
            load_kv(stage ^ 1, (jb + 1) * kBN);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (jb == 0) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint32_t row = warp * 16u + r8 + (mi & 1u) * 8u;
                const uint32_t ch = ks * 2u + (mi >> 1);
                ldsm_x4(smem_addr(sQ) + swz(row, ch), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
            }
        }
        // S = Q K^T for 16 rows x 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-key n-tiles
                uint32_t b0, b1, b2, b3;
                const uint32_t krow = jp * 16u + r8 + (mi >> 1) * 8u;
                const uint32_t ch = ks * 2u + (mi & 1u);
                ldsm_x4(smem_addr(sK[stage]) + swz(krow, ch), b0, b1, b2, b3);
                mma16816<kBF16>(s[2 * jp], qf[ks], b0, b1);
                mma16816<kBF16>(s[2 * jp + 1], qf[ks], b2, b3);
            }
        }
        // mask keys past the end
        const uint32_t kbase = jb * kBN;
        if (kbase + kBN > tokens) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t c = kbase + j * 8u + (lane & 3u) * 2u;
                if (c >= tokens) s[j][0] = s[j][2] = -INFINITY;
                if (c + 1 >= tokens) s[j][1] = s[j][3] = -INFINITY;
            }
        }
        // online softmax: rows g (elements 0,1) and g+8 (elements 2,3)
        float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
            mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        }
        float corr[2], ms[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            ms[h] = mx[h] * scale_log2;
            corr[h] = exp2f(m_r[h] * scale_log2 - ms[h]);
            m_r[h] = mx[h];
        }
        float ls[2] = {0.f, 0.f};
        uint32_t pf[4][4];  // P as A fragments for 4 k-steps of 16 keys
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float p0 = exp2f(s[j][0] * scale_log2 - ms[0]);
            const float p1 = exp2f(s[j][1] * scale_log2 - ms[0]);
            const float p2 = exp2f(s[j][2] * scale_log2 - ms[1]);
            const float p3 = exp2f(s[j][3] * scale_log2 - ms[1]);
            ls[0] += p0 + p1;
            ls[1] += p2 + p3;
            pf[j >> 1][(j & 1) * 2 + 0] = pack2<kBF16>(p0, p1);
            pf[j >> 1][(j & 1) * 2 + 1] = pack2<kBF16>(p2, p3);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) l_r[h] = l_r[h] * corr[h] + ls[h];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= corr[0];
            o[j][1] *= corr[0];
            o[j][2] *= corr[1];
            o[j][3] *= corr[1];
        }
        // O += P V
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const uint32_t a[4] = {pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3]};
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                uint32_t b0, b1, b2, b3;
                const uint32_t vrow = ks * 16u + r8 + (mi & 1u) * 8u;
                const uint32_t ch = jp * 2u + (mi >> 1);
                ldsm_x4_t(smem_addr(sV[stage]) + swz(vrow, ch), b0, b1, b2, b3);
                mma16816<kBF16>(o[2 * jp], a, b0, b1);
                mma16816<kBF16>(o[2 * jp + 1], a, b2, b3);
            }
        }
        __syncthreads();
    }
    // finalize: full row sums across the quad, divide, store
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 1);
        l_r[h] += __shfl_xor_sync(0xffffffffu, l_r[h], 2);
    }
    const float inv0 = 1.0f / fmaxf(l_r[0], 1.0e-20f);
    const float inv1 = 1.0f / fmaxf(l_r[1], 1.0e-20f);
    const uint32_t g = lane >> 2, t = lane & 3u;
    const uint32_t qa = q0 + warp * 16u + g, qb2 = qa + 8u;
    H* ob = out + img * tokens * out_ld + head * kD;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t d = j * 8u + t * 2u;
        if (qa < tokens)
            *reinterpret_cast<uint32_t*>(ob + (uint64_t)qa * out_ld + d) = pack2<kBF16>(o[j][0] * inv0, o[j][1] * inv0);
        if (qb2 < tokens)
            *reinterpret_cast<uint32_t*>(ob + (uint64_t)qb2 * out_ld + d) = pack2<kBF16>(o[j][2] * inv1, o[j][3] * inv1);
    }
}

}  // namespace

template <typename H>
int launch_attention(H* out, const H* qkv, uint32_t batch, uint32_t tokens, uint32_t heads, uint64_t qkv_ld,
                     uint64_t out_ld, cudaStream_t st) {
    if (tokens == 0 || heads == 0 || batch == 0) return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: empty");
    // the interleaved QKV layout runs on the tcgen05 kernel (attention_tc.cu)
    if (qkv_ld == 3ull * heads * 64 && out_ld % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0)
        return launch_attention_tc(out, false, qkv, std::is_same<H, __nv_bfloat16>::value, batch, tokens, heads,
                                   qkv_ld, out_ld, st);
    if ((qkv_ld * sizeof(H)) % 16 || (out_ld * sizeof(H)) % 4 || reinterpret_cast<uintptr_t>(qkv) % 16)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: misaligned rows");
    dim3 grid((tokens + kBM - 1) / kBM, heads, batch);
    attention_kernel<H><<<grid, 128, 0, st>>>(out, qkv, tokens, heads, qkv_ld, out_ld);
    return check_launch("attention");
}

template int launch_attention<__half>(__half*, const __half*, uint32_t, uint32_t, uint32_t, uint64_t, uint64_t,
                                      cudaStream_t);
template int launch_attention<__nv_bfloat16>(__nv_bfloat16*, const __nv_bfloat16*, uint32_t, uint32_t, uint32_t,
                                             uint64_t, uint64_t, cudaStream_t);

}  // namespace dav2cuda
