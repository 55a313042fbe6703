// Shared device helpers for the sm_100a kernels: status codes, the device
// error word, bounded mbarrier waits, TMA loads and tcgen05 (TMEM / UMMA)
// wrappers written as inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dav2cuda.h"

namespace dav2cuda {

// Kernels report failures through a device error word (never by
// trapping): a pointer to it is passed as a kernel argument; the host reads
// and clears it with dav2cuda_device_error(). Codes: 1 = pipeline wait
// timed out.

constexpr unsigned long long kWaitTimeoutNs = 4000000000ull;  // 4 s

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps until it completes or about hint_ns pass, instead of spinning and
// taking issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// limit_ns, or as soon as *abort is set by another role of the CTA; on a
// timeout it records error 1 and sets *abort. Returns false when the wait
// did not complete.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                              unsigned long long limit_ns) {
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity)) return true;
    const unsigned long long start = globaltimer();
    for (uint32_t spin = 1;; ++spin) {
        if (mbar_try_wait_hint(a, parity, 20000u)) return true;
        if ((spin & 15u) == 0) {
            if (*abort) return false;
            if (globaltimer() - start > limit_ns) {
                *abort = 1;
                atomicExch(err, 1);
                return false;
            }
        }
    }
}

// The pipelines' wait: limit kWaitTimeoutNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
    return mbar_wait_for(bar, parity, abort, err, kWaitTimeoutNs);
}

// ----------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// Tiled shared -> global store (bulk async-group completion). The writing
// threads must execute fence_async_smem() and synchronise before one thread
// issues the store. Coordinates are never negative here.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(c0), "r"(c1)
                 : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N committed store groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every committed store group has completed.
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Make this thread's generic-proxy shared-memory writes visible to the
// async proxy (TMA stores, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
                 "r"(columns)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
template <bool kInt8>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                     uint32_t accumulate) {
    if constexpr (kInt8) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Arrives on the mbarrier once all previously issued MMAs of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: each thread gets its lane's row.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Inverse of tmem_ld_32x32b_x32: each thread writes its lane's 32 columns.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored as rows
// of 128 bytes with the 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B): leading offset 16 B, 8-row group stride
// 1024 B, descriptor version 1, layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: dense, D format (1=f32, 2=s32), A/B format,
// both K-major, N>>3 at bit 17, M>>4 at bit 24.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_format, uint32_t ab_format, uint32_t m,
                                                  uint32_t n) {
    return (c_format << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ------------------------------------------------------------------- misc
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// code = rint(clamp(v, -127, 127)) as a byte (ties to even, as the
// reference's CPU packers: std::nearbyint).
__device__ __forceinline__ uint32_t q8(float v) {
    v = fminf(fmaxf(v, -127.0f), 127.0f);
    return static_cast<uint32_t>(__float2int_rn(v)) & 0xffu;
}

// ------------------------------------------------------- packed f32x2 math
// sm_100 executes two IEEE fp32 lanes per instruction (fma/mul/add .rn .f32x2).
// The assembler may contract a packed multiply and a following packed add
// into one fused operation, so these serve approximations (GELU, softmax)
// and not arithmetic that must reproduce separately rounded steps.
__device__ __forceinline__ void f2_fma(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                       float c1) {
    asm("{\n\t.reg .b64 a, b, c;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
        "fma.rn.f32x2 a, a, b, c;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void f2_mul(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "mul.rn.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ void f2_add(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
        "add.rn.f32x2 a, a, b;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Exact-erf GELU (torch.nn.GELU) with erf from Abramowitz & Stegun 7.1.26
// (|error| <= 1.5e-7): erf(z) = 1 - t(a1 + t(a2 + t(a3 + t(a4 + t a5)))) e^{-z^2},
// t = 1/(1 + p z) for z >= 0, odd extension for z < 0. Used where GELU is
// fused into another kernel (GEMM epilogue, row quantizer).
__device__ __forceinline__ float gelu_erf_as(float v) {
    const float z = fabsf(v) * 0.70710678118654752f;
    const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
    const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f),
                                     -0.284496736f), 0.254829592f);
    const float e = 1.0f - poly * __expf(-z * z);
    return 0.5f * v * (1.0f + copysignf(e, v));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// The same A&S 7.1.26 GELU on a pair, rearranged for fewer instructions:
// gelu(v) = max(v, 0) - |v|/2 * erfc(|v|/sqrt2), and with t = 1/(1 + p|v|/sqrt2),
// erfc = t(a1 + ... + t^4 a5) e^{-v^2/2}; the -1/2 goes into the coefficients
// (b_i = -a_i/2, exact) and e^{-v^2/2} = 2^{c v^2}, c = -log2(e)/2, so
//   gelu(v) = |v| * t(b1 + t(b2 + t(b3 + t(b4 + t b5)))) * 2^{c v^2} + max(v, 0).
// The negative branch has no cancellation (the result is the product term
// alone). Multiply-adds are issued as f32x2; reciprocal and exponential are
// the hardware approximations (relative error near 2^-22).
__device__ __forceinline__ void gelu_erf_as2(float& v0, float& v1) {
    constexpr float kP = 0.3275911f * 0.70710678118654752f;
    constexpr float kC = -0.72134752044448170f;
    constexpr float b1 = -0.5f * 0.254829592f, b2 = -0.5f * -0.284496736f, b3 = -0.5f * 1.421413741f,
                    b4 = -0.5f * -1.453152027f, b5 = -0.5f * 1.061405429f;
    const float a0 = fabsf(v0), a1 = fabsf(v1);
    float d0, d1, q0, q1, w0, w1;
    f2_fma(d0, d1, a0, a1, kP, kP, 1.0f, 1.0f);
    const float t0 = rcp_approx(d0), t1 = rcp_approx(d1);
    f2_mul(w0, w1, v0, v1, kC, kC);
    f2_fma(q0, q1, t0, t1, b5, b5, b4, b4);
    f2_mul(w0, w1, w0, w1, v0, v1);
    f2_fma(q0, q1, t0, t1, q0, q1, b3, b3);
    f2_fma(q0, q1, t0, t1, q0, q1, b2, b2);
    const float e0 = ex2_approx(w0), e1 = ex2_approx(w1);
    f2_fma(q0, q1, t0, t1, q0, q1, b1, b1);
    f2_mul(q0, q1, t0, t1, q0, q1);
    f2_mul(q0, q1, q0, q1, e0, e1);
    f2_fma(v0, v1, q0, q1, a0, a1, fmaxf(v0, 0.0f), fmaxf(v1, 0.0f));
}

// Four bytes q8(x[k] / scale) (IEEE quotient) packed little-endian, for a
// per-row scale = max(absmax/127, 1e-8) with |x| <= absmax — the quotient is
// then at most ~127.00003, so the clamp of q8 never acts. Without a division
// per element: q = x * rs (rs = correctly rounded 1/scale) is within 2e-5 of
// the quotient and can round to a different integer only within that
// distance of a half-integer. The rounding uses C = 1.5*2^23: q + C holds
// rint(q) in its low mantissa bits (round-half-even, |q| < 2^22), so its low
// byte is the two's-complement code. A group with an element within 1e-4 of
// a half-integer (or a NaN) takes the exact quotient (rare).
__device__ __forceinline__ uint32_t q8x4_quot(float x0, float x1, float x2, float x3, float scale, float rs) {
    constexpr float C = 12582912.0f;
    const float xs[4] = {x0, x1, x2, x3};
    float t[4];
    bool near_tie = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float q = __fmul_rn(xs[k], rs);
        t[k] = __fadd_rn(q, C);
        near_tie |= !(fabsf(__fsub_rn(q, __fsub_rn(t[k], C))) <= 0.4999f);
    }
    if (near_tie) {
#pragma unroll
        for (int k = 0; k < 4; ++k) t[k] = __fadd_rn(fminf(fmaxf(__fdiv_rn(xs[k], scale), -127.0f), 127.0f), C);
    }
    const uint32_t lo = __byte_perm(__float_as_uint(t[0]), __float_as_uint(t[1]), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(t[2]), __float_as_uint(t[3]), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
}

}  // namespace dav2cuda

#include "launch.h"
