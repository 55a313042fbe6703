// Persistent, warp-specialized tcgen05 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] . B[N, K]^T   (both operands K-major)
//
// A is either a plain row-major matrix (linear layers, 1x1 convolutions,
// explicit im2col) or a channels-last feature map read as an implicit 3x3
// (stride 1, pad 1) convolution: for tap (ky, kx) and channel block c0 the
// A tile of a 16x8-pixel output block is one 4-D TMA box loaded at pixel
// offset (kx-1, ky-1) — the tensor-memory-access unit zero-fills the halo.
// B is a K-major weight matrix ([Cout][ky][kx][Cin] for convolutions).
//
// Roles per CTA (320 threads, one CTA per SM):
//   warp 0        TMA producer: fills a STAGES-deep ring of 128-byte-swizzled
//                 A/B tiles (128 x 128 B and BN x 128 B);
//   warp 1        TMEM allocator + MMA issuer: 4 tcgen05.mma (K=32 bytes) per
//                 ring slot into one of two TMEM accumulators (128 lanes x
//                 BN columns each), tcgen05.commit frees slots / publishes
//                 accumulators;
//   warps 2..9    epilogue, two warps per TMEM lane quarter: tcgen05.ld
//                 32x32b rows out of TMEM, fused dequant / bias / GELU /
//                 LayerScale-residual / ReLU / residual adds / output-head
//                 dot; row-major results go through a shared-memory
//                 transpose so that global stores are whole 128-byte lines.
// The two accumulators let the epilogue of tile i overlap the MMAs of
// tile i+1. Every wait is bounded (common.cuh: mbar_wait); a timeout sets
// the device error word and the CTA drains and returns instead of hanging.
#pragma once

#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>


namespace dav2cuda {
// The kernel templates and their shared types live in a named namespace so
// that gemm_tc.cu (tensor maps, epilogue-program choice) and the
// gemm_tc_inst_*.cu files (one template instantiation set each, compiled in
// parallel) agree on them.
namespace gemm_impl {

constexpr int kMaxStages = 12;

struct GemmParamsDev {
    uint32_t m, n, num_kb, num_m_tiles, num_n_tiles;
    uint32_t a_mode;
    uint32_t conv_h, conv_w, tiles_x, tiles_y, kb_per_tap;
    uint32_t flags;
    int out_kind;
    int out_bf16;
    void* out;
    void* out2;
    uint64_t ldo;
    const float* bias;
    const float* s_in;
    const float* s_w;
    const float* gamma;
    const void* res1;
    const void* res2;
    const float* head_w;
    float* const* out_slot;  // kTmaHeadDot: destination pointer read from this device slot when set
    float head_b, head_max;
    uint32_t rows_per_img, out_rows_per_img, row_offset;
    uint64_t img_stride, col_stride;
    uint32_t ct_k, ct_cout, ct_w, ct_h;
    int* err;
    int program;      // RowProgram for row-major outputs (transposed-store path)
    int tma_program;  // TmaProgram: thread-row epilogue with TMA stores, or 0
    uint32_t stages;         // depth of the A/B shared-memory ring
    uint32_t staging_bytes;  // epilogue staging area (TMA boxes or transposed-store slab)
};


__device__ __forceinline__ uint32_t pack_half2(float a, float b, bool bf16) {
    if (bf16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float half_at(const void* p, uint64_t i, bool bf16) {
    if (bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void unpack4(uint2 t, bool bf16, float (&o)[4]) {
    if (bf16) {
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&t.x);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&t.y);
        o[0] = __low2float(a); o[1] = __high2float(a); o[2] = __low2float(b); o[3] = __high2float(b);
    } else {
        const __half2 a = *reinterpret_cast<const __half2*>(&t.x);
        const __half2 b = *reinterpret_cast<const __half2*>(&t.y);
        o[0] = __low2float(a); o[1] = __high2float(a); o[2] = __low2float(b); o[3] = __high2float(b);
    }
}

template <bool kInt8>
__device__ __forceinline__ void epilogue_chunk(const GemmParamsDev& p, const uint32_t (&acc)[32], bool valid,
                                               uint64_t r, uint32_t col0) {
    if (!valid) return;
    const uint32_t f = p.flags;
    const bool full = col0 + 32 <= p.n;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = kInt8 ? (float)(int32_t)acc[j] : __uint_as_float(acc[j]);
    // per-column parameters as 16-byte loads for whole, aligned chunks
    const bool vec_sw = full && (reinterpret_cast<uintptr_t>(p.s_w) & 15u) == 0;
    const bool vec_b = full && (reinterpret_cast<uintptr_t>(p.bias) & 15u) == 0;
    if (f & kEpiDequant) {
        const float si = __ldg(p.s_in + r);
        if (vec_sw) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 sw = __ldg(reinterpret_cast<const float4*>(p.s_w + col0 + j));
                v[j] = __fmul_rn(__fmul_rn(v[j], si), sw.x);
                v[j + 1] = __fmul_rn(__fmul_rn(v[j + 1], si), sw.y);
                v[j + 2] = __fmul_rn(__fmul_rn(v[j + 2], si), sw.z);
                v[j + 3] = __fmul_rn(__fmul_rn(v[j + 3], si), sw.w);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float sw = (full || col0 + j < p.n) ? __ldg(p.s_w + col0 + j) : 0.f;
                v[j] = __fmul_rn(__fmul_rn(v[j], si), sw);
            }
        }
    }
    if (f & kEpiBias) {
        if (vec_b) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + j));
                v[j] = __fadd_rn(v[j], b.x);
                v[j + 1] = __fadd_rn(v[j + 1], b.y);
                v[j + 2] = __fadd_rn(v[j + 2], b.z);
                v[j + 3] = __fadd_rn(v[j + 3], b.w);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (full || col0 + j < p.n) v[j] = __fadd_rn(v[j], __ldg(p.bias + col0 + j));
        }
    }
    if (f & kEpiGelu) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) gelu_erf_as2(v[j], v[j + 1]);
    }

    // --- output-head dot product (one value per row)
    if (f & kEpiHeadDot) {
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float a = fmaxf(v[j], 0.0f);
            if (full || col0 + j < p.n) d = fmaf(a, __ldg(p.head_w + col0 + j), d);
        }
        d += p.head_b;
        d = (f & kEpiMetricHead) ? p.head_max / (1.0f + expf(-d)) : fmaxf(d, 0.0f);
        uint64_t orow = r;
        if (p.rows_per_img) orow = (r / p.rows_per_img) * p.out_rows_per_img + p.row_offset + r % p.rows_per_img;
        reinterpret_cast<float*>(p.out)[orow] = d;
        return;
    }

    // --- element addresses
    if (p.out_kind == kOutF32Rows || p.out_kind == kOutHalfRows) {
        uint64_t orow = r;
        if (p.rows_per_img) orow = (r / p.rows_per_img) * p.out_rows_per_img + p.row_offset + r % p.rows_per_img;
        const uint64_t base = orow * p.ldo + col0;
        const bool hb = p.out_bf16 != 0;
        if (p.out_kind == kOutF32Rows) {
            if (f & (kEpiLayerScale | kEpiResidual1 | kEpiResidual2)) {
                const float* r1 = reinterpret_cast<const float*>(p.res1);
                const float* r2 = reinterpret_cast<const float*>(p.res2);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (!(full || col0 + j < p.n)) continue;
                    if (f & kEpiLayerScale) v[j] = __fadd_rn(r1[base + j], __fmul_rn(v[j], __ldg(p.gamma + col0 + j)));
                    else if (f & kEpiResidual1) v[j] = v[j] + r1[base + j];
                    if (f & kEpiResidual2) v[j] = r2[base + j] + v[j];
                }
            }
            if (f & kEpiRelu) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
            }
            float* o = reinterpret_cast<float*>(p.out) + base;
            if (full && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                for (int j = 0; j < 32; ++j)
                    if (col0 + j < p.n) o[j] = v[j];
            }
            if (f & kEpiReluCopy) {
                float* o2 = reinterpret_cast<float*>(p.out2) + base;
                for (int j = 0; j < 32; ++j)
                    if (col0 + j < p.n) o2[j] = fmaxf(v[j], 0.f);
            }
        } else {
            if (f & (kEpiResidual1 | kEpiResidual2)) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (!(full || col0 + j < p.n)) continue;
                    if (f & kEpiResidual1) v[j] = v[j] + half_at(p.res1, base + j, hb);
                    if (f & kEpiResidual2) v[j] = half_at(p.res2, base + j, hb) + v[j];
                }
            }
            if (f & kEpiRelu) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
            }
            uint16_t* o = reinterpret_cast<uint16_t*>(p.out) + base;
            uint16_t* o2 = (f & kEpiReluCopy) ? reinterpret_cast<uint16_t*>(p.out2) + base : nullptr;
            if (full && ((reinterpret_cast<uintptr_t>(o) & 15) == 0)) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                    uint4 w;
                    w.x = pack_half2(v[j], v[j + 1], hb);
                    w.y = pack_half2(v[j + 2], v[j + 3], hb);
                    w.z = pack_half2(v[j + 4], v[j + 5], hb);
                    w.w = pack_half2(v[j + 6], v[j + 7], hb);
                    *reinterpret_cast<uint4*>(o + j) = w;
                    if (o2) {
                        uint4 z;
                        z.x = pack_half2(fmaxf(v[j], 0.f), fmaxf(v[j + 1], 0.f), hb);
                        z.y = pack_half2(fmaxf(v[j + 2], 0.f), fmaxf(v[j + 3], 0.f), hb);
                        z.z = pack_half2(fmaxf(v[j + 4], 0.f), fmaxf(v[j + 5], 0.f), hb);
                        z.w = pack_half2(fmaxf(v[j + 6], 0.f), fmaxf(v[j + 7], 0.f), hb);
                        *reinterpret_cast<uint4*>(o2 + j) = z;
                    }
                }
            } else {
                for (int j = 0; j < 32; j += 2) {
                    if (col0 + j >= p.n) break;
                    const uint32_t w = pack_half2(v[j], v[j + 1], hb);
                    o[j] = (uint16_t)(w & 0xffff);
                    if (col0 + j + 1 < p.n) o[j + 1] = (uint16_t)(w >> 16);
                    if (o2) {
                        const uint32_t z = pack_half2(fmaxf(v[j], 0.f), fmaxf(v[j + 1], 0.f), hb);
                        o2[j] = (uint16_t)(z & 0xffff);
                        if (col0 + j + 1 < p.n) o2[j + 1] = (uint16_t)(z >> 16);
                    }
                }
            }
        }
        return;
    }
    if (f & kEpiRelu) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
    }
    if (p.out_kind == kOutF32Planar) {
        uint64_t img = 0, px = r;
        if (p.rows_per_img) {
            img = r / p.rows_per_img;
            px = r % p.rows_per_img;
        }
        float* o = reinterpret_cast<float*>(p.out) + img * p.img_stride + p.row_offset + px +
                   (uint64_t)col0 * p.col_stride;
        if (full) {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[(uint64_t)j * p.col_stride] = v[j];
        } else {
            for (int j = 0; j < 32; ++j)
                if (col0 + j < p.n) o[(uint64_t)j * p.col_stride] = v[j];
        }
        return;
    }
    // conv-transpose scatter (kernel == stride)
    const uint32_t hw = p.ct_w * p.ct_h;
    const uint64_t img = r / hw;
    const uint32_t pp = (uint32_t)(r % hw);
    const uint32_t y = pp / p.ct_w, x = pp % p.ct_w;
    const uint32_t ow = p.ct_w * p.ct_k, oh = p.ct_h * p.ct_k;
    for (int j = 0; j < 32; ++j) {
        const uint32_t col = col0 + j;
        if (col >= p.n) break;
        const uint32_t kk = col / p.ct_cout, co = col % p.ct_cout;
        const uint32_t oy = y * p.ct_k + kk / p.ct_k, ox = x * p.ct_k + kk % p.ct_k;
        if (p.out_kind == kOutConvTF32) {
            reinterpret_cast<float*>(p.out)[((img * p.ct_cout + co) * oh + oy) * ow + ox] = v[j];
        } else {
            const uint64_t idx = ((img * oh + oy) * ow + ox) * (p.ldo ? p.ldo : p.ct_cout) + co;
            if (p.out_bf16)
                reinterpret_cast<__nv_bfloat16*>(p.out)[idx] = __float2bfloat16_rn(v[j]);
            else
                reinterpret_cast<__half*>(p.out)[idx] = __float2half_rn(v[j]);
        }
    }
}

// Row-major outputs (linear layers, channels-last maps): the 32x32 chunk a
// warp reads from TMEM (thread = row) is staged through a padded shared
// slab (stride 33 floats: conflict-free both ways) and re-read with 8 lanes
// per row and 4 consecutive columns per lane, so residual loads and output
// stores are 16-byte vectors covering whole 128-byte lines (64 bytes for half
// outputs). Per-row scaling happens before the transpose, per-column work
// (weight scale, bias, GELU, LayerScale, residuals, ReLU) after it, where
// each lane needs the parameters of only its 4 columns.
template <bool kInt8, bool F32, bool BIAS, bool GELU, bool LS, bool R1, bool R2, bool RELU, bool RC, bool CT = false>
__device__ __forceinline__ void epilogue_rows(const GemmParamsDev& p, const uint32_t (&acc)[32], bool valid,
                                              uint64_t r, uint32_t col0, float* slab, uint32_t lane) {
    float si = 1.0f;
    if (kInt8 && valid) si = __ldg(p.s_in + r);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        float v = kInt8 ? (float)(int32_t)acc[j] : __uint_as_float(acc[j]);
        if (kInt8) v = __fmul_rn(v, si);
        slab[lane * 33 + j] = v;
    }
    __syncwarp();
    uint64_t orow_l = r;
    if (p.rows_per_img) orow_l = (r / p.rows_per_img) * p.out_rows_per_img + p.row_offset + r % p.rows_per_img;
    const uint32_t cq = (lane & 7u) * 4u;
    const uint32_t c = col0 + cq;
    const bool cols_full = c + 4 <= p.n;
    float sw[4], bs[4], gm[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool ok = c + k < p.n;
        sw[k] = (kInt8 && ok) ? __ldg(p.s_w + c + k) : 1.0f;
        bs[k] = (BIAS && ok) ? __ldg(p.bias + c + k) : 0.0f;
        gm[k] = (LS && ok) ? __ldg(p.gamma + c + k) : 0.0f;
    }
    const bool hb = p.out_bf16 != 0;
    const int my_valid = valid ? 1 : 0;
    // Output element offsets of the 8 row groups this lane stores, and (for
    // residual programs) the residual values there. All residual loads of
    // the chunk are issued before any store: the output usually aliases the
    // residual (in-place update), so loads interleaved with stores would
    // serialise into one memory round trip per row group.
    uint64_t base[8];
    bool live[8];
    float ra[8][4], rb[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t src = 4u * i + (lane >> 3);
        const int vrow = __shfl_sync(0xffffffffu, my_valid, src);
        const unsigned long long orow = __shfl_sync(0xffffffffu, (unsigned long long)orow_l, src);
        live[i] = vrow && c < p.n;
        base[i] = orow * p.ldo + c;
        if (CT) {
            // conv-transpose (kernel == stride): GEMM row = input pixel,
            // column = (ky*k + kx)*Cout + co -> channels-last output pixel
            const uint32_t hw = p.ct_w * p.ct_h;
            const uint64_t img = orow / hw;
            const uint32_t pp = (uint32_t)(orow % hw);
            const uint32_t kk = c / p.ct_cout, co = c % p.ct_cout;
            const uint32_t oy = (pp / p.ct_w) * p.ct_k + kk / p.ct_k, ox = (pp % p.ct_w) * p.ct_k + kk % p.ct_k;
            base[i] = ((img * p.ct_h * p.ct_k + oy) * (uint64_t)(p.ct_w * p.ct_k) + ox) * p.ldo + co;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) ra[i][k] = rb[i][k] = 0.f;
        if ((LS || R1 || R2) && live[i]) {
            const bool vec = cols_full && ((base[i] & 3u) == 0);
            if (F32) {
                if (LS || R1) {
                    const float* r1 = reinterpret_cast<const float*>(p.res1) + base[i];
                    if (vec) {
                        const float4 t = *reinterpret_cast<const float4*>(r1);
                        ra[i][0] = t.x; ra[i][1] = t.y; ra[i][2] = t.z; ra[i][3] = t.w;
                    } else {
                        for (int k = 0; k < 4; ++k) ra[i][k] = c + k < p.n ? r1[k] : 0.f;
                    }
                }
                if (R2) {
                    const float* r2 = reinterpret_cast<const float*>(p.res2) + base[i];
                    if (vec) {
                        const float4 t = *reinterpret_cast<const float4*>(r2);
                        rb[i][0] = t.x; rb[i][1] = t.y; rb[i][2] = t.z; rb[i][3] = t.w;
                    } else {
                        for (int k = 0; k < 4; ++k) rb[i][k] = c + k < p.n ? r2[k] : 0.f;
                    }
                }
            } else if (vec) {
                if (R1) unpack4(*reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p.res1) + base[i]), hb, ra[i]);
                if (R2) unpack4(*reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p.res2) + base[i]), hb, rb[i]);
            } else {
                for (int k = 0; k < 4; ++k) {
                    if (c + k >= p.n) break;
                    if (R1) ra[i][k] = half_at(p.res1, base[i] + k, hb);
                    if (R2) rb[i][k] = half_at(p.res2, base[i] + k, hb);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t src = 4u * i + (lane >> 3);
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = slab[src * 33 + cq + k];
        if (live[i]) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (kInt8) v[k] = __fmul_rn(v[k], sw[k]);
                if (BIAS) v[k] = __fadd_rn(v[k], bs[k]);
            }
            if (GELU) {
                gelu_erf_as2(v[0], v[1]);
                gelu_erf_as2(v[2], v[3]);
            }
            const bool vec = cols_full && ((base[i] & 3u) == 0) && (!CT || (p.ct_cout & 3u) == 0);
            if (F32) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (LS) v[k] = __fadd_rn(ra[i][k], __fmul_rn(v[k], gm[k]));
                    else if (R1) v[k] = v[k] + ra[i][k];
                    if (R2) v[k] = rb[i][k] + v[k];
                    if (RELU) v[k] = fmaxf(v[k], 0.f);
                }
                float* o = reinterpret_cast<float*>(p.out) + base[i];
                if (vec) {
                    *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
                    if (RC)
                        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out2) + base[i]) =
                            make_float4(fmaxf(v[0], 0.f), fmaxf(v[1], 0.f), fmaxf(v[2], 0.f), fmaxf(v[3], 0.f));
                } else {
                    for (int k = 0; k < 4; ++k)
                        if (c + k < p.n) {
                            o[k] = v[k];
                            if (RC) reinterpret_cast<float*>(p.out2)[base[i] + k] = fmaxf(v[k], 0.f);
                        }
                }
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if (R1) v[k] = v[k] + ra[i][k];
                    if (R2) v[k] = rb[i][k] + v[k];
                    if (RELU) v[k] = fmaxf(v[k], 0.f);
                }
                uint16_t* o = reinterpret_cast<uint16_t*>(p.out) + base[i];
                if (vec) {
                    *reinterpret_cast<uint2*>(o) = make_uint2(pack_half2(v[0], v[1], hb), pack_half2(v[2], v[3], hb));
                    if (RC)
                        *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p.out2) + base[i]) =
                            make_uint2(pack_half2(fmaxf(v[0], 0.f), fmaxf(v[1], 0.f), hb),
                                       pack_half2(fmaxf(v[2], 0.f), fmaxf(v[3], 0.f), hb));
                } else {
                    for (int k = 0; k < 4; ++k) {
                        if (c + k >= p.n) break;
                        o[k] = (uint16_t)(pack_half2(v[k], 0.f, hb) & 0xffffu);
                        if (RC)
                            reinterpret_cast<uint16_t*>(p.out2)[base[i] + k] =
                                (uint16_t)(pack_half2(fmaxf(v[k], 0.f), 0.f, hb) & 0xffffu);
                    }
                }
            }
        }
    }
    __syncwarp();
}

// Row-epilogue programs with a compiled instance (flags -> id); other flag
// combinations use the generic per-element path (epilogue_chunk).
enum RowProgram : int {
    kRowGeneric = 0,
    kRowF32,            // f32 (+bias)
    kRowF32Bias,
    kRowF32BiasGelu,
    kRowF32BiasLS,      // LayerScale residual (proj, fc2)
    kRowF32BiasR1,      // residual (patch embedding onto positions)
    kRowHalf,
    kRowHalfBias,
    kRowHalfBiasGelu,   // fc1
    kRowHalfBiasRelu,   // RCU conv1
    kRowHalfRC,         // layer_rn
    kRowHalfBiasR1,     // RCU2 conv2
    kRowHalfBiasR1R2RC, // RCU1 conv2 + fusion add
    kRowHalfBiasCT,     // conv-transpose scatter into channels-last half
};

template <bool kInt8>
__device__ __forceinline__ void epilogue_dispatch(const GemmParamsDev& p, int prog, const uint32_t (&acc)[32],
                                                  bool valid, uint64_t r, uint32_t col0, float* slab, uint32_t lane) {
    switch (prog) {
        case kRowF32: epilogue_rows<kInt8, true, false, false, false, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowF32Bias: epilogue_rows<kInt8, true, true, false, false, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowF32BiasGelu: epilogue_rows<kInt8, true, true, true, false, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowF32BiasLS: epilogue_rows<kInt8, true, true, false, true, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowF32BiasR1: epilogue_rows<kInt8, true, true, false, false, true, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalf: epilogue_rows<kInt8, false, false, false, false, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfBias: epilogue_rows<kInt8, false, true, false, false, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfBiasGelu: epilogue_rows<kInt8, false, true, true, false, false, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfBiasRelu: epilogue_rows<kInt8, false, true, false, false, false, false, true, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfRC: epilogue_rows<kInt8, false, false, false, false, false, false, false, true>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfBiasR1: epilogue_rows<kInt8, false, true, false, false, true, false, false, false>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfBiasR1R2RC: epilogue_rows<kInt8, false, true, false, false, true, true, false, true>(p, acc, valid, r, col0, slab, lane); break;
        case kRowHalfBiasCT: epilogue_rows<kInt8, false, true, false, false, false, false, false, false, true>(p, acc, valid, r, col0, slab, lane); break;
        default: epilogue_chunk<kInt8>(p, acc, valid, r, col0); break;
    }
}

// ------------------------------------------------- thread-row TMA epilogue
// For row-major outputs whose column count is a multiple of the tile width:
// each epilogue thread owns one accumulator row (its TMEM lane) and 32
// consecutive columns per chunk, exactly as tcgen05.ld 32x32b delivers them,
// so there is no transpose, shuffle or per-row address arithmetic. Per-column
// parameters (weight scales, bias, LayerScale) are warp-uniform vector loads.
// Results are written into a 32-row shared-memory box in the tensor map's
// swizzled layout (128-byte swizzle for f32 rows of 128 B, 64-byte swizzle
// for f16 rows of 64 B; both conflict-free for 16-byte row-wise writes) and
// leave with one TMA store per box; rows beyond M are clipped by the map.
// The LayerScale residual (x += gamma * y, in place) arrives by TMA into the
// other staging buffer one chunk ahead of its use.
enum TmaProgram : int {
    kTmaNone = 0,
    kTmaHalf,
    kTmaHalfBias,
    kTmaHalfBiasGelu,    // fc1
    kTmaHalfBiasRelu,    // RCU conv1
    kTmaHalfRC,          // layer_rn: output + ReLU copy
    kTmaHalfBiasR1,      // RCU2 conv2: + residual
    kTmaHalfBiasR1R2RC,  // RCU1 conv2: + residual + fusion input, ReLU copy
    kTmaF32,
    kTmaF32Bias,
    kTmaF32BiasGelu,
    kTmaF32BiasLS,  // attention projection, fc2
    kTmaHeadDot,    // output head: relu(acc + b) . w (+ head bias, ReLU or sigmoid*max)
    kTmaHalfBiasCT, // conv-transpose (kernel == stride) scatter into a channels-last half map
};

// Tensor maps of the thread-row epilogue: output, ReLU-copy output and the
// two residual inputs (2-D [rows][ld] for row-major A, 4-D [B][H][W][ld]
// channels-last for the implicit convolution).
struct EpiMaps {
    CUtensorMap out, out2, res1, res2;
};

constexpr uint32_t kStageBufBytes = 2048;  // one 32-row box of 64-byte rows (32 f16 or 16 f32 columns)

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Four accumulator columns to values, the column parameters already in
// registers (loaded ahead of the accumulator wait).
template <bool kInt8, bool BIAS, bool GELU>
__device__ __forceinline__ void dequant4_pre(const uint32_t* acc, float si, float4 w, float4 b, float* v) {
    const float ws[4] = {w.x, w.y, w.z, w.w}, bs[4] = {b.x, b.y, b.z, b.w};
    if (kInt8 && GELU) {
        // followed by GELU, whose result is an approximation anyway: one fused
        // multiply-add acc * (s_in * s_w) + b per value, issued as f32x2
        float s[4];
        f2_mul(s[0], s[1], si, si, ws[0], ws[1]);
        f2_mul(s[2], s[3], si, si, ws[2], ws[3]);
#pragma unroll
        for (int k = 0; k < 4; k += 2)
            f2_fma(v[k], v[k + 1], (float)(int32_t)acc[k], (float)(int32_t)acc[k + 1], s[k], s[k + 1],
                   BIAS ? bs[k] : 0.0f, BIAS ? bs[k + 1] : 0.0f);
        gelu_erf_as2(v[0], v[1]);
        gelu_erf_as2(v[2], v[3]);
        return;
    }
    // (acc * s_in) * s_w + b with the reference's separate roundings (scalar:
    // bit-exact with the oracle), then GELU on pairs of columns
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float t = kInt8 ? (float)(int32_t)acc[k] : __uint_as_float(acc[k]);
        if (kInt8) t = __fmul_rn(__fmul_rn(t, si), ws[k]);
        if (BIAS) t = __fadd_rn(t, bs[k]);
        v[k] = t;
    }
    if (GELU) {
        gelu_erf_as2(v[0], v[1]);
        gelu_erf_as2(v[2], v[3]);
    }
}

// dequant4_pre with the column parameters loaded here.
template <bool kInt8, bool BIAS, bool GELU>
__device__ __forceinline__ void dequant4(const uint32_t* acc, float si, const float* s_w, const float* bias,
                                         uint32_t c, float* v) {
    float4 w = make_float4(1.f, 1.f, 1.f, 1.f), b = make_float4(0.f, 0.f, 0.f, 0.f);
    if (kInt8) w = ldg4(s_w + c);
    if (BIAS) b = ldg4(bias + c);
    dequant4_pre<kInt8, BIAS, GELU>(acc, si, w, b, v);
}

// One chunk (64 bytes of output per row: 16 f32 or 32 f16 columns):
// registers -> 64-byte-swizzled staging boxes. Row `lane` is at lane*64; its
// 16-byte unit u sits at unit u ^ ((lane >> 1) & 3), conflict-free for
// row-wise 16-byte writes. Box A holds the first residual on entry (LS, R1)
// and the output on exit; box B holds the second residual (R2) on entry and
// the ReLU copy (RC) on exit.
template <bool kInt8, bool F32, bool BIAS, bool GELU, bool LS, bool RELU, bool R1, bool R2, bool RC>
__device__ __forceinline__ void tma_chunk_compute(const GemmParamsDev& p, const uint32_t* acc, float si,
                                                  uint32_t col0, uint8_t* box, uint8_t* box2, uint32_t lane,
                                                  const float4* pre_w = nullptr, const float4* pre_b = nullptr) {
    const bool hb = p.out_bf16 != 0;
    const uint32_t sw = (lane >> 1) & 3u;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const uint32_t off = lane * 64u + (((uint32_t)u ^ sw) << 4);
        uint8_t* q = box + off;
        if (F32) {
            const uint32_t c = col0 + 4u * u;
            float v[4];
            if (pre_w) dequant4_pre<kInt8, BIAS, GELU>(acc + 4 * u, si, pre_w[u], pre_b[u], v);
            else dequant4<kInt8, BIAS, GELU>(acc + 4 * u, si, p.s_w, p.bias, c, v);
            if (LS) {
                const float4 gm = ldg4(p.gamma + c);
                const float4 r = *reinterpret_cast<const float4*>(q);
                v[0] = __fadd_rn(r.x, __fmul_rn(v[0], gm.x));
                v[1] = __fadd_rn(r.y, __fmul_rn(v[1], gm.y));
                v[2] = __fadd_rn(r.z, __fmul_rn(v[2], gm.z));
                v[3] = __fadd_rn(r.w, __fmul_rn(v[3], gm.w));
            }
            if (RELU) {
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = fmaxf(v[k], 0.f);
            }
            *reinterpret_cast<float4*>(q) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
            const uint32_t c = col0 + 8u * u;
            float v[8];
            dequant4<kInt8, BIAS, GELU>(acc + 8 * u, si, p.s_w, p.bias, c, v);
            dequant4<kInt8, BIAS, GELU>(acc + 8 * u + 4, si, p.s_w, p.bias, c + 4u, v + 4);
            if (R1 || R2) {
                float a[8], b2[8];
                if (R1) {
                    const uint4 t = *reinterpret_cast<const uint4*>(q);
                    unpack4(make_uint2(t.x, t.y), hb, *reinterpret_cast<float(*)[4]>(a));
                    unpack4(make_uint2(t.z, t.w), hb, *reinterpret_cast<float(*)[4]>(a + 4));
                }
                if (R2) {
                    const uint4 t = *reinterpret_cast<const uint4*>(box2 + off);
                    unpack4(make_uint2(t.x, t.y), hb, *reinterpret_cast<float(*)[4]>(b2));
                    unpack4(make_uint2(t.z, t.w), hb, *reinterpret_cast<float(*)[4]>(b2 + 4));
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    if (R1) v[k] = v[k] + a[k];
                    if (R2) v[k] = b2[k] + v[k];
                }
            }
            if (RELU) {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = fmaxf(v[k], 0.f);
            }
            *reinterpret_cast<uint4*>(q) = make_uint4(pack_half2(v[0], v[1], hb), pack_half2(v[2], v[3], hb),
                                                      pack_half2(v[4], v[5], hb), pack_half2(v[6], v[7], hb));
            if (RC)
                *reinterpret_cast<uint4*>(box2 + off) =
                    make_uint4(pack_half2(fmaxf(v[0], 0.f), fmaxf(v[1], 0.f), hb),
                               pack_half2(fmaxf(v[2], 0.f), fmaxf(v[3], 0.f), hb),
                               pack_half2(fmaxf(v[4], 0.f), fmaxf(v[5], 0.f), hb),
                               pack_half2(fmaxf(v[6], 0.f), fmaxf(v[7], 0.f), hb));
        }
    }
}

// Box origin of (tile, column) for this warp's 32 rows: rows m_blk*128 +
// 32*quarter for row-major A; pixels (x0..x0+15, y0+2q..y0+2q+1) of one image
// for the implicit convolution (an 8 x 16 pixel tile).
template <int AMODE>
struct BoxAt {
    int c, x, y, z;
    __device__ __forceinline__ BoxAt(const GemmParamsDev& p, uint32_t m_blk, uint32_t quarter, uint32_t col) {
        c = (int)col;
        if constexpr (AMODE == kAModeRows) {
            x = (int)(m_blk * 128u + quarter * 32u);
            y = z = 0;
        } else {
            const uint32_t per_img = p.tiles_x * p.tiles_y;
            const uint32_t rem = m_blk % per_img;
            x = (int)((rem % p.tiles_x) * 16u);
            y = (int)((rem / p.tiles_x) * 8u + 2u * quarter);
            z = (int)(m_blk / per_img);
        }
    }
    __device__ __forceinline__ void store(const CUtensorMap* m, const void* src) const {
        if constexpr (AMODE == kAModeRows) tma_store_2d(m, src, c, x);
        else tma_store_4d(m, src, c, x, y, z);
    }
    __device__ __forceinline__ void load(const CUtensorMap* m, void* dst, uint64_t* bar) const {
        if constexpr (AMODE == kAModeRows) tma_load_2d(dst, m, bar, c, x);
        else tma_load_4d(dst, m, bar, c, x, y, z);
    }
};

// The epilogue warp's whole tile loop for one program. EPI epilogue warps:
// EPI/4 per TMEM lane quarter, sharing the quarter's chunks round-robin.
// `bufs` is this warp's pair of staging boxes, `rbar` its pair of residual
// mbarriers. Programs with one output and at most one residual double-buffer
// the boxes (a residual is prefetched one chunk ahead); programs with a
// second residual or a ReLU copy use the pair as boxes A and B of one chunk.
template <int BN, int EPI, int AMODE, bool kInt8, bool F32, bool BIAS, bool GELU, bool LS, bool RELU, bool R1, bool R2,
          bool RC>
__device__ __noinline__ void epilogue_tma_loop(const GemmParamsDev& p, const EpiMaps* em, uint32_t tmem_base,
                                               uint64_t* tfull, uint64_t* tempty, uint64_t* rbar, uint8_t* staging,
                                               volatile int* abort_flag, uint32_t warp, uint32_t lane) {
    constexpr uint32_t CW = F32 ? 16u : 32u;      // columns per chunk
    constexpr uint32_t kStride = (EPI / 4) * CW;  // column step between this warp's chunks
    constexpr bool kPair = R2 || RC;
    constexpr bool kRes = LS || R1;
    constexpr uint32_t kBoxes = 2;  // per warp: double-buffered output, residual prefetch, or boxes A and B
    uint8_t* bufs = staging + kBoxes * kStageBufBytes * (warp - 2u);
    if ((warp - 1u) * kBoxes * kStageBufBytes > p.staging_bytes) {
        // the launch's staging area is too small for this program: fail cleanly
        if (lane == 0) {
            atomicExch(p.err, 3);
            *abort_flag = 1;
        }
        return;
    }
    const uint32_t quarter = warp & 3u;
    const uint32_t sub = (warp - 2u) >> 2;
    const uint32_t num_tiles = p.num_m_tiles * p.num_n_tiles;
    const uint32_t first_c = sub * CW;
    const bool has_chunks = first_c < (uint32_t)BN;
    uint32_t seq = 0;  // chunks processed by this warp
    auto origin = [&](uint32_t tile, uint32_t c) {
        return BoxAt<AMODE>(p, tile / p.num_n_tiles, quarter, (tile % p.num_n_tiles) * (uint32_t)BN + c);
    };
    if (kRes && !kPair && has_chunks && lane == 0 && blockIdx.x < num_tiles) {
        mbar_arrive_expect_tx(&rbar[0], kStageBufBytes);
        origin(blockIdx.x, first_c).load(&em->res1, bufs, &rbar[0]);
    }

    uint32_t local = 0;
    for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1u;
        // the row scale is loaded before the accumulator wait (its latency
        // overlaps the wait)
        const uint32_t m_blk = tile / p.num_n_tiles;
        float si = 0.f;
        if (kInt8) {
            uint64_t r;
            bool valid;
            if constexpr (AMODE == kAModeRows) {
                r = (uint64_t)m_blk * 128u + quarter * 32u + lane;
                valid = r < p.m;
            } else {
                const uint32_t per_img = p.tiles_x * p.tiles_y, rem = m_blk % per_img;
                const uint32_t y = (rem / p.tiles_x) * 8u + 2u * quarter + lane / 16u;
                const uint32_t x = (rem % p.tiles_x) * 16u + lane % 16u;
                valid = y < p.conv_h && x < p.conv_w;
                r = ((uint64_t)(m_blk / per_img) * p.conv_h + y) * p.conv_w + x;
            }
            if (valid) si = __ldg(p.s_in + r);
        }
        if (!mbar_wait(&tfull[buf], (local >> 1) & 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * (uint32_t)BN;
        bool ok = true;
#pragma unroll 1
        for (uint32_t c = first_c; c < (uint32_t)BN; c += kStride) {
            // f32 outputs without LayerScale (fc1): this chunk's 16 column scales
            // and biases are loaded before the TMEM read, so their latency
            // overlaps it (measured 3% on fc1; the LayerScale programs, which
            // also hold residuals, keep their loads in place)
            constexpr bool kPre = F32 && !LS;
            float4 pre_w[4], pre_b[4];
            if constexpr (kPre) {
                const uint32_t col = origin(tile, c).c;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    pre_w[u] = kInt8 ? ldg4(p.s_w + col + 4u * u) : make_float4(1.f, 1.f, 1.f, 1.f);
                    pre_b[u] = BIAS ? ldg4(p.bias + col + 4u * u) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
            uint32_t acc[CW];
            if constexpr (CW == 32) {
                tmem_ld_32x32b_x32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(acc));
            } else {
                tmem_ld_32x32b_x16(taddr + c, *reinterpret_cast<uint32_t(*)[16]>(acc));
            }
            tmem_ld_wait();
            if (c + kStride >= (uint32_t)BN) {  // last TMEM read of this tile: release the accumulator
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            const BoxAt<AMODE> at = origin(tile, c);
            uint8_t* box = kPair ? bufs : bufs + (seq & 1u) * kStageBufBytes;
            uint8_t* box2 = bufs + kStageBufBytes;
            if (kPair) {
                // both boxes are reused every chunk: the previous stores must
                // have read them out before the residuals land
                if (lane == 0) {
                    bulk_wait_group_read<0>();
                    if (R1 || R2) {
                        mbar_arrive_expect_tx(&rbar[0], (R1 && R2 ? 2u : 1u) * kStageBufBytes);
                        if (R1) at.load(&em->res1, box, &rbar[0]);
                        if (R2) at.load(&em->res2, box2, &rbar[0]);
                    }
                }
                if (R1 || R2) {
                    if (!mbar_wait(&rbar[0], seq & 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                } else {
                    __syncwarp();
                }
            } else if (kRes) {
                const uint32_t b = seq & 1u;
                if (lane == 0) {
                    // prefetch the next chunk's residual into the other box, once
                    // the store that last used that box has read it out
                    uint32_t nt = tile, nc = c + kStride;
                    if (nc >= (uint32_t)BN) {
                        nt = tile + gridDim.x;
                        nc = first_c;
                    }
                    if (nt < num_tiles) {
                        bulk_wait_group_read<0>();
                        mbar_arrive_expect_tx(&rbar[b ^ 1u], kStageBufBytes);
                        origin(nt, nc).load(&em->res1, bufs + (b ^ 1u) * kStageBufBytes, &rbar[b ^ 1u]);
                    }
                }
                if (!mbar_wait(&rbar[b], (seq >> 1) & 1u, abort_flag, p.err)) {
                    ok = false;
                    break;
                }
            } else {
                if (lane == 0) bulk_wait_group_read<1>();
                __syncwarp();
            }
            tma_chunk_compute<kInt8, F32, BIAS, GELU, LS, RELU, R1, R2, RC>(
                p, acc, si, (uint32_t)at.c, box, box2, lane, kPre ? pre_w : nullptr, kPre ? pre_b : nullptr);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                at.store(&em->out, box);
                if (RC) at.store(&em->out2, box2);
                bulk_commit_group();
            }
            ++seq;
        }
        if (!has_chunks) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
        if (!ok) break;
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
}

// Output head on the implicit convolution (N = 32): each thread owns one
// pixel's accumulator row and reduces it to the depth value,
// d = sum_j relu(acc_j + b_j) * w_j in column order (the transposed-store
// path's order), then + head bias and ReLU, or max_depth * sigmoid for a
// metric head; one f32 store per pixel (a warp's 32 pixels are two 16-pixel
// runs). Parameters are warp-uniform vector loads. With p.out_slot set the
// output pointer is read from that device slot (a captured graph then writes
// into whichever buffer the launching call stored there).
template <int BN>
__device__ __noinline__ void epilogue_head_loop(const GemmParamsDev& p, uint32_t tmem_base, uint64_t* tfull,
                                                uint64_t* tempty, volatile int* abort_flag, uint32_t warp,
                                                uint32_t lane) {
    const uint32_t quarter = warp & 3u;
    const bool owner = ((warp - 2u) >> 2) == 0u;  // one warp per lane quarter holds the 32 columns
    const uint32_t num_tiles = p.num_m_tiles * p.num_n_tiles;
    const bool metric = (p.flags & kEpiMetricHead) != 0;
    // the destination: fixed, or read once from the slot that the launching
    // stream filled before this kernel (plain load: the slot changes between launches)
    float* dst = nullptr;
    uint32_t local = 0;
    for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1u;
        if (!mbar_wait(&tfull[buf], (local >> 1) & 1u, abort_flag, p.err)) break;
        tc_fence_after();
        uint32_t acc[32];
        if (owner) {
            tmem_ld_32x32b_x32(tmem_base + ((quarter * 32u) << 16) + buf * (uint32_t)BN, acc);
            tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        if (!owner) continue;
        const uint32_t m_blk = tile / p.num_n_tiles;
        if (dst == nullptr) dst = p.out_slot ? *p.out_slot : reinterpret_cast<float*>(p.out);
        const uint32_t per_img = p.tiles_x * p.tiles_y, rem = m_blk % per_img;
        const uint32_t y = (rem / p.tiles_x) * 8u + 2u * quarter + lane / 16u;
        const uint32_t x = (rem % p.tiles_x) * 16u + lane % 16u;
        float d = 0.f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
            const float4 b4 = ldg4(p.bias + 4 * g), w4 = ldg4(p.head_w + 4 * g);
            const float bs[4] = {b4.x, b4.y, b4.z, b4.w}, ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float v = __fadd_rn(__uint_as_float(acc[4 * g + k]), bs[k]);
                d = fmaf(fmaxf(v, 0.0f), ws[k], d);
            }
        }
        d += p.head_b;
        d = metric ? p.head_max / (1.0f + expf(-d)) : fmaxf(d, 0.0f);
        if (y < p.conv_h && x < p.conv_w)
            dst[((uint64_t)(m_blk / per_img) * p.conv_h + y) * p.conv_w + x] = d;
    }
}

// Conv-transpose with kernel == stride k (row-major A: GEMM row = input pixel
// (img, py, px), column = (ky*k + kx)*Cout + co): each thread owns one input
// pixel's row; a 32-column chunk has one (ky, kx) and 32 consecutive output
// channels, i.e. 64 contiguous bytes of output pixel (py*k + ky, px*k + kx),
// written with four 16-byte stores. The pixel decomposition is done once per
// tile. Requires Cout % 32 == 0 and 16-byte aligned output rows.
template <int BN, int EPI, bool kInt8>
__device__ __noinline__ void epilogue_ct_loop(const GemmParamsDev& p, uint32_t tmem_base, uint64_t* tfull,
                                              uint64_t* tempty, volatile int* abort_flag, uint32_t warp,
                                              uint32_t lane) {
    constexpr uint32_t kStride = (EPI / 4) * 32u;
    const uint32_t quarter = warp & 3u;
    const uint32_t first_c = ((warp - 2u) >> 2) * 32u;
    const uint32_t num_tiles = p.num_m_tiles * p.num_n_tiles;
    const bool hb = p.out_bf16 != 0;
    const uint32_t k = p.ct_k, ow = p.ct_w * k, oh = p.ct_h * k, hw = p.ct_w * p.ct_h;
    uint32_t local = 0;
    for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1u;
        if (!mbar_wait(&tfull[buf], (local >> 1) & 1u, abort_flag, p.err)) break;
        tc_fence_after();
        const uint32_t n_blk = tile % p.num_n_tiles, m_blk = tile / p.num_n_tiles;
        const uint32_t r = m_blk * 128u + quarter * 32u + lane;
        const bool valid = r < p.m;
        const float si = (kInt8 && valid) ? __ldg(p.s_in + r) : 0.f;
        const uint32_t img = r / hw, pp = r % hw, py = pp / p.ct_w, px = pp % p.ct_w;
        const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * (uint32_t)BN;
        if (first_c >= (uint32_t)BN) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            continue;
        }
#pragma unroll 1
        for (uint32_t c = first_c; c < (uint32_t)BN; c += kStride) {
            uint32_t acc[32];
            tmem_ld_32x32b_x32(taddr + c, acc);
            tmem_ld_wait();
            if (c + kStride >= (uint32_t)BN) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
            }
            const uint32_t col0 = n_blk * (uint32_t)BN + c;
            const uint32_t kk = col0 / p.ct_cout, co0 = col0 % p.ct_cout;
            const uint32_t oy = py * k + kk / k, ox = px * k + kk % k;
            uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p.out) +
                                                ((uint64_t)(img * oh + oy) * ow + ox) * p.ldo + co0);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float v[8];
                dequant4<kInt8, true, false>(acc + 8 * u, si, p.s_w, p.bias, col0 + 8u * u, v);
                dequant4<kInt8, true, false>(acc + 8 * u + 4, si, p.s_w, p.bias, col0 + 8u * u + 4u, v + 4);
                if (valid)
                    o[u] = make_uint4(pack_half2(v[0], v[1], hb), pack_half2(v[2], v[3], hb), pack_half2(v[4], v[5], hb),
                                      pack_half2(v[6], v[7], hb));
            }
        }
    }
}

template <int BN, int EPI, int AMODE, bool kInt8>
__device__ __forceinline__ void epilogue_tma_dispatch(const GemmParamsDev& p, const EpiMaps* em, uint32_t tmem_base,
                                                      uint64_t* tfull, uint64_t* tempty, uint64_t* rbar,
                                                      uint8_t* staging, volatile int* abort_flag, uint32_t warp,
                                                      uint32_t lane) {
#define DAV2_TMA_EPI(F32, BIAS, GELU, LS, RELU, R1, R2, RC)                                                     \
    epilogue_tma_loop<BN, EPI, AMODE, kInt8, F32, BIAS, GELU, LS, RELU, R1, R2, RC>(p, em, tmem_base, tfull, \
                                                                                   tempty, rbar, staging,     \
                                                                                   abort_flag, warp, lane)
    constexpr bool kRows = AMODE == kAModeRows;
    // row-major A with 8 epilogue warps: only the long-K LayerScale residual
    // (the host selects 8 warps for it alone)
    constexpr bool kLite = kRows && EPI == 8;
    switch (p.tma_program) {
        case kTmaHalf:
            if constexpr (!kLite) DAV2_TMA_EPI(false, false, false, false, false, false, false, false);
            break;
        case kTmaHalfBias:
            if constexpr (!kLite) DAV2_TMA_EPI(false, true, false, false, false, false, false, false);
            break;
        case kTmaHalfBiasRelu:
            if constexpr (!kLite) DAV2_TMA_EPI(false, true, false, false, true, false, false, false);
            break;
        case kTmaHalfRC:
            if constexpr (!kLite) DAV2_TMA_EPI(false, false, false, false, false, false, false, true);
            break;
        case kTmaHalfBiasR1:
            if constexpr (!kLite) DAV2_TMA_EPI(false, true, false, false, false, true, false, false);
            break;
        case kTmaHalfBiasR1R2RC:
            if constexpr (!kLite) DAV2_TMA_EPI(false, true, false, false, false, true, true, true);
            break;
        case kTmaHalfBiasGelu:
            if constexpr (kRows && !kLite) DAV2_TMA_EPI(false, true, true, false, false, false, false, false);
            break;
        case kTmaF32:
            if constexpr (kRows && !kLite) DAV2_TMA_EPI(true, false, false, false, false, false, false, false);
            break;
        case kTmaF32Bias:
            if constexpr (kRows && !kLite) DAV2_TMA_EPI(true, true, false, false, false, false, false, false);
            break;
        case kTmaF32BiasGelu:
            if constexpr (kRows && !kLite) DAV2_TMA_EPI(true, true, true, false, false, false, false, false);
            break;
        default:
            if constexpr (kRows) DAV2_TMA_EPI(true, true, false, true, false, false, false, false);
            break;
    }
#undef DAV2_TMA_EPI
}

template <int BN, int ELEM, int AMODE, int EPI>
__global__ void __launch_bounds__(64 + 32 * EPI, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ EpiMaps em,
                   const __grid_constant__ GemmParamsDev p) {
    constexpr bool kInt8 = ELEM == kElemS8;
    constexpr uint32_t kABytes = 128u * 128u;
    constexpr uint32_t kBBytes = (uint32_t)BN * 128u;
    constexpr uint32_t kTmemCols = 2u * BN < 32u ? 32u : 2u * BN;
    // f16: A/B format 0; bf16: 1; s8 (signed): 1. D: f32 = 1, s32 = 2.
    constexpr uint32_t kIdesc = make_idesc(kInt8 ? 2u : 1u, ELEM == kElemF16 ? 0u : 1u, 128u, (uint32_t)BN);
    const uint32_t STAGES = p.stages;

    // [A ring][B ring][1 KB: barriers, TMEM slot, abort flag][epilogue staging]
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * kABytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * kBBytes);
    uint64_t* empty = full + kMaxStages;
    uint64_t* tfull = empty + kMaxStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* rbars = drain + 1;  // epilogue warps x 2 residual barriers
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbars + 2 * EPI);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    uint8_t* staging = reinterpret_cast<uint8_t*>(full) + 1024;
    float* slabs = reinterpret_cast<float*>(staging);  // 8 x 32 x 33 floats (transposed-store path)

    const uint32_t warp = threadIdx.x >> 5;
    const uint32_t lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        if (p.tma_program != kTmaNone) {
            tma_prefetch_desc(&em.out);
            tma_prefetch_desc(&em.out2);
            tma_prefetch_desc(&em.res1);
            tma_prefetch_desc(&em.res2);
        }
        for (uint32_t s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&tfull[0], 1);
        mbar_init(&tfull[1], 1);
        mbar_init(&tempty[0], EPI);
        mbar_init(&tempty[1], EPI);
        mbar_init(drain, 1);
        for (int i = 0; i < 2 * EPI; ++i) mbar_init(&rbars[i], 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const uint32_t num_tiles = p.num_m_tiles * p.num_n_tiles;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            for (uint32_t tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
                const uint32_t n_blk = tile % p.num_n_tiles;
                const uint32_t m_blk = tile / p.num_n_tiles;
                int img = 0, y0 = 0, x0 = 0;
                if constexpr (AMODE == kAModeConv3x3) {
                    const uint32_t per_img = p.tiles_x * p.tiles_y;
                    img = (int)(m_blk / per_img);
                    const uint32_t rem = m_blk % per_img;
                    y0 = (int)(rem / p.tiles_x) * 8;
                    x0 = (int)(rem % p.tiles_x) * 16;
                }
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.err)) break;
                    mbar_arrive_expect_tx(&full[stage], kABytes + kBBytes);
                    const int kcol = (int)(kb * (kInt8 ? 128u : 64u));
                    if constexpr (AMODE == kAModeRows) {
                        tma_load_2d(sA + stage * kABytes, &tm_a, &full[stage], kcol, (int)(m_blk * 128u));
                    } else {
                        const uint32_t tap = kb / p.kb_per_tap;
                        const int c0 = (int)((kb % p.kb_per_tap) * (kInt8 ? 128u : 64u));
                        const int ky = (int)(tap / 3), kx = (int)(tap % 3);
                        tma_load_4d(sA + stage * kABytes, &tm_a, &full[stage], c0, x0 + kx - 1, y0 + ky - 1, img);
                    }
                    tma_load_2d(sB + stage * kBBytes, &tm_b, &full[stage], kcol, (int)(n_blk * (uint32_t)BN));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, local = 0;
            for (uint32_t tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
                const uint32_t buf = local & 1u;
                if (!mbar_wait(&tempty[buf], ((local >> 1) & 1u) ^ 1u, abort_flag, p.err)) break;
                tc_fence_after();
                const uint32_t d = tmem_base + buf * (uint32_t)BN;
                bool ok = true;
                for (uint32_t kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_addr(sA + stage * kABytes);
                    const uint32_t b_addr = smem_addr(sB + stage * kBBytes);
#pragma unroll
                    for (uint32_t j = 0; j < 4; ++j) {
                        umma<kInt8>(d, smem_desc_sw128(a_addr + 32u * j), smem_desc_sw128(b_addr + 32u * j), kIdesc,
                                    (kb | j) != 0u ? 1u : 0u);
                    }
                    mma_issued = true;
                    umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[buf]);
            }
        }
    } else if (p.tma_program == kTmaHalfBiasCT) {
        if constexpr (AMODE == kAModeRows && EPI == 16)
            epilogue_ct_loop<BN, EPI, kInt8>(p, tmem_base, tfull, tempty, abort_flag, warp, lane);
    } else if (p.tma_program == kTmaHeadDot) {
        if constexpr (BN == 32 && AMODE == kAModeConv3x3 && ELEM != kElemS8 && EPI == 8)
            epilogue_head_loop<BN>(p, tmem_base, tfull, tempty, abort_flag, warp, lane);
    } else if (p.tma_program != kTmaNone) {
        if constexpr (AMODE == kAModeRows || (AMODE == kAModeConv3x3 && ELEM != kElemS8 && EPI == 8))
            epilogue_tma_dispatch<BN, EPI, AMODE, kInt8>(p, &em, tmem_base, tfull, tempty, rbars + 2u * (warp - 2u),
                                                         staging, abort_flag, warp, lane);
    } else if constexpr (EPI == 8) {
        // warps 2..9: two warps per TMEM lane quarter, splitting the chunks
        const uint32_t quarter = warp & 3u;
        const uint32_t half = (warp - 2u) >> 2;  // 0 or 1
        const uint32_t row_in_tile = quarter * 32u + lane;
        float* slab = slabs + (warp - 2u) * (32u * 33u);
        uint32_t local = 0;
        for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const uint32_t buf = local & 1u;
            if (!mbar_wait(&tfull[buf], (local >> 1) & 1u, abort_flag, p.err)) break;
            tc_fence_after();
            const uint32_t n_blk = tile % p.num_n_tiles;
            const uint32_t m_blk = tile / p.num_n_tiles;
            uint64_t r;
            bool valid;
            if constexpr (AMODE == kAModeRows) {
                r = (uint64_t)m_blk * 128u + row_in_tile;
                valid = r < p.m;
            } else {
                const uint32_t per_img = p.tiles_x * p.tiles_y;
                const uint32_t img = m_blk / per_img;
                const uint32_t rem = m_blk % per_img;
                const uint32_t y = (rem / p.tiles_x) * 8u + row_in_tile / 16u;
                const uint32_t x = (rem % p.tiles_x) * 16u + row_in_tile % 16u;
                valid = y < p.conv_h && x < p.conv_w;
                r = ((uint64_t)img * p.conv_h + y) * p.conv_w + x;
            }
            const uint32_t taddr = tmem_base + ((quarter * 32u) << 16) + buf * (uint32_t)BN;
            // chunk c (32 columns) belongs to this warp when (c/32) % 2 == half;
            // two chunks are loaded from TMEM before waiting.
#pragma unroll 1
            for (uint32_t c = half * 32u; c < (uint32_t)BN; c += 128u) {
                uint32_t acc0[32], acc1[32];
                const bool two = c + 64u < (uint32_t)BN;
                tmem_ld_32x32b_x32(taddr + c, acc0);
                if (two) tmem_ld_32x32b_x32(taddr + c + 64u, acc1);
                tmem_ld_wait();
                const uint32_t col0 = n_blk * (uint32_t)BN + c;
                if (col0 < p.n) epilogue_dispatch<kInt8>(p, p.program, acc0, valid, r, col0, slab, lane);
                if (two && col0 + 64u < p.n) epilogue_dispatch<kInt8>(p, p.program, acc1, valid, r, col0 + 64u, slab, lane);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
        }
    }

    __syncthreads();
    if (*abort_flag) {
        // Drain: let issued MMAs and in-flight tensor copies finish (bounded)
        // before the accumulator memory is released.
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
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

constexpr uint32_t kSmemOptin = 232448;      // B200 per-block opt-in limit
constexpr uint32_t kSlabBytes = 8 * 32 * 33 * 4;  // transposed-store epilogue scratch

// Ring depth that fits beside the epilogue staging area, and the dynamic
// shared-memory size of that configuration.
inline uint32_t stages_for(int bn, uint32_t staging) {
    const uint32_t per_stage = 128u * 128u + (uint32_t)bn * 128u;
    uint32_t s = (kSmemOptin - 2048u - staging) / per_stage;
    return s > (uint32_t)kMaxStages ? (uint32_t)kMaxStages : s;
}

inline size_t smem_for(int bn, uint32_t stages, uint32_t staging) {
    return (size_t)stages * (128u * 128u + (uint32_t)bn * 128u) + 1024u + staging + 1024u;
}


template <int BN, int ELEM, int AMODE, int EPI>
int run(const CUtensorMap& ma, const CUtensorMap& mb, const EpiMaps& em, GemmParamsDev p,
        uint32_t staging, int max_ctas, cudaStream_t st) {
    auto kernel = gemm_tc_kernel<BN, ELEM, AMODE, EPI>;
    p.stages = stages_for(BN, staging);
    p.staging_bytes = staging;
    const size_t smem = smem_for(BN, p.stages, staging);
    if (p.stages < 2 || smem > kSmemOptin) return set_error(DAV2CUDA_INTERNAL_ERROR, "gemm: shared memory plan");
    static std::atomic<uint64_t> configured{0};  // one bit per device ordinal
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured_on(configured, dev)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemOptin) != cudaSuccess ||
            cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return set_error(DAV2CUDA_LAUNCH_FAILED, "gemm: cannot set shared memory size");
        mark_configured(configured, dev);
    }
    const int sms = sm_count(dev);
    if (sms <= 0) return set_error(DAV2CUDA_LAUNCH_FAILED, "gemm: cannot query the SM count");
    const uint32_t tiles = p.num_m_tiles * p.num_n_tiles;
    uint32_t grid = (uint32_t)(max_ctas > 0 ? max_ctas : sms);
    if (grid > tiles) grid = tiles;
    kernel<<<grid, 64 + 32 * EPI, smem, st>>>(ma, mb, em, p);
    return check_launch("gemm_tc");
}

// Thread-row TMA epilogue programs of row-major A run with 16 epilogue warps;
// the implicit convolution (its K loop is long enough for 8 epilogue warps to
// keep up) and the transposed-store programs with 8, which leaves room for a
// 4-deep ring at BN = 256.
template <int ELEM, int AMODE>
int dispatch_bn(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const EpiMaps& em, const GemmParamsDev& p,
                uint32_t staging, int max_ctas, cudaStream_t st, bool epi8 = false) {
    if constexpr (AMODE == kAModeRows) {
        if (p.tma_program != kTmaNone && !epi8) {
            switch (bn) {
                case 256: return run<256, ELEM, AMODE, 16>(ma, mb, em, p, staging, max_ctas, st);
                case 128: return run<128, ELEM, AMODE, 16>(ma, mb, em, p, staging, max_ctas, st);
                case 64: return run<64, ELEM, AMODE, 16>(ma, mb, em, p, staging, max_ctas, st);
                default: return run<32, ELEM, AMODE, 16>(ma, mb, em, p, staging, max_ctas, st);
            }
        }
    }
    switch (bn) {
        case 256: return run<256, ELEM, AMODE, 8>(ma, mb, em, p, staging, max_ctas, st);
        case 128: return run<128, ELEM, AMODE, 8>(ma, mb, em, p, staging, max_ctas, st);
        case 64: return run<64, ELEM, AMODE, 8>(ma, mb, em, p, staging, max_ctas, st);
        default: return run<32, ELEM, AMODE, 8>(ma, mb, em, p, staging, max_ctas, st);
    }
}


// One instantiation set per (operand type, A mode), defined in gemm_tc_inst_*.cu.
#define DAV2_GEMM_DISPATCH_DECL(NAME)                                                                         \
    int NAME(int bn, const CUtensorMap& ma, const CUtensorMap& mb, const EpiMaps& em, const GemmParamsDev& p, \
             uint32_t staging, int max_ctas, cudaStream_t st, bool epi8);
DAV2_GEMM_DISPATCH_DECL(dispatch_s8_rows)
DAV2_GEMM_DISPATCH_DECL(dispatch_s8_conv)
DAV2_GEMM_DISPATCH_DECL(dispatch_f16_rows)
DAV2_GEMM_DISPATCH_DECL(dispatch_f16_conv)
DAV2_GEMM_DISPATCH_DECL(dispatch_bf16_rows)
DAV2_GEMM_DISPATCH_DECL(dispatch_bf16_conv)
#undef DAV2_GEMM_DISPATCH_DECL

}  // namespace gemm_impl
}  // namespace dav2cuda
