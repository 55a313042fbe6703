// Host side of the tcgen05 GEMM (gemm_tc_kernel.cuh): tensor maps, the
// epilogue program and tile width of each call, and the launch through the
// instantiation set of its operand type and A mode (gemm_tc_inst_*.cu).
#include "gemm_tc_kernel.cuh"

#include <cstdio>
#include <mutex>

namespace dav2cuda {
using namespace gemm_impl;
namespace {

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

CUtensorMapDataType tm_type(int elem) {
    switch (elem) {
        case kElemS8: return CU_TENSOR_MAP_DATA_TYPE_UINT8;
        case kElemF16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
        default: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    }
}

int make_map_typed(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const cuuint64_t* dims,
                   const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
    if (!get_encoder()) return set_error(DAV2CUDA_INTERNAL_ERROR, "cuTensorMapEncodeTiled unavailable");
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult rc = g_encode(map, type, rank, const_cast<void*>(base), dims, strides_bytes, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) {
        char msg[160];
        snprintf(msg, sizeof msg, "cuTensorMapEncodeTiled failed (%d)", (int)rc);
        return set_error(DAV2CUDA_INVALID_ARGUMENT, msg);
    }
    return DAV2CUDA_OK;
}

int make_map(CUtensorMap* map, int elem, int rank, const void* base, const cuuint64_t* dims,
             const cuuint64_t* strides_bytes, const cuuint32_t* box) {
    return make_map_typed(map, tm_type(elem), rank, base, dims, strides_bytes, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

int launch_gemm(const GemmArgs& g, cudaStream_t st) {
    if (g.m == 0 || g.n == 0 || g.k == 0) return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: empty extent");
    const uint32_t es = g.elem == kElemS8 ? 1u : 2u;
    const uint32_t bk = 128u / es;
    const int bn = g.block_n ? g.block_n : (g.n >= 256 && g.n % 256 == 0 ? 256 : (g.n > 64 ? 128 : (g.n > 32 ? 64 : 32)));
    if ((g.flags & kEpiHeadDot) && (bn != 32 || g.n > 32))
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: head dot needs N <= 32");
    if (reinterpret_cast<uintptr_t>(g.a) % 16 || reinterpret_cast<uintptr_t>(g.b) % 16)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: operands must be 16-byte aligned");
    if ((g.ldb * es) % 16) return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: weight rows must be 16-byte multiples");

    GemmParamsDev p{};
    p.m = g.m;
    p.n = g.n;
    p.a_mode = (uint32_t)g.a_mode;
    p.flags = g.flags;
    p.out_kind = g.out_kind;
    p.out_bf16 = g.out_half_bf16 ? 1 : 0;
    p.out = g.out;
    p.out2 = g.out2;
    p.ldo = g.ldo;
    p.bias = g.bias;
    p.s_in = g.s_in;
    p.s_w = g.s_w;
    p.gamma = g.gamma;
    p.res1 = g.res1;
    p.res2 = g.res2;
    p.head_w = g.head_w;
    p.head_b = g.head_b;
    p.head_max = g.head_max_depth;
    p.out_slot = g.out_slot;
    p.rows_per_img = g.rows_per_img;
    p.out_rows_per_img = g.out_rows_per_img;
    p.row_offset = g.row_offset;
    p.img_stride = g.img_stride;
    p.col_stride = g.col_stride;
    p.ct_k = g.convt_k;
    p.ct_cout = g.convt_cout;
    p.ct_w = g.convt_w;
    p.ct_h = g.convt_h;
    p.num_n_tiles = (g.n + bn - 1) / bn;
    p.program = kRowGeneric;
    if (g.out_kind == kOutConvTHalf && (g.flags & ~uint32_t(kEpiDequant)) == kEpiBias &&
        ((g.flags & kEpiDequant) != 0) == (g.elem == kElemS8))
        p.program = kRowHalfBiasCT;
    if ((g.out_kind == kOutF32Rows || g.out_kind == kOutHalfRows) && !(g.flags & kEpiHeadDot)) {
        const uint32_t f = g.flags & ~uint32_t(kEpiDequant);
        const bool f32 = g.out_kind == kOutF32Rows;
        if (f32) {
            if (f == 0) p.program = kRowF32;
            else if (f == kEpiBias) p.program = kRowF32Bias;
            else if (f == (kEpiBias | kEpiGelu)) p.program = kRowF32BiasGelu;
            else if (f == (kEpiBias | kEpiLayerScale)) p.program = kRowF32BiasLS;
            else if (f == (kEpiBias | kEpiResidual1)) p.program = kRowF32BiasR1;
        } else {
            if (f == 0) p.program = kRowHalf;
            else if (f == kEpiBias) p.program = kRowHalfBias;
            else if (f == (kEpiBias | kEpiGelu)) p.program = kRowHalfBiasGelu;
            else if (f == (kEpiBias | kEpiRelu)) p.program = kRowHalfBiasRelu;
            else if (f == kEpiReluCopy) p.program = kRowHalfRC;
            else if (f == (kEpiBias | kEpiResidual1)) p.program = kRowHalfBiasR1;
            else if (f == (kEpiBias | kEpiResidual1 | kEpiResidual2 | kEpiReluCopy)) p.program = kRowHalfBiasR1R2RC;
        }
        if (((g.flags & kEpiDequant) != 0) != (g.elem == kElemS8)) p.program = kRowGeneric;
    }
    p.err = device_error_word();
    if (!p.err) return set_error(DAV2CUDA_INTERNAL_ERROR, "gemm: no device error word");

    CUtensorMap ma, mb;
    {
        const cuuint64_t dims[2] = {g.k, g.n};
        const cuuint64_t strides[1] = {g.ldb * es};
        const cuuint32_t box[2] = {bk, (cuuint32_t)bn};
        if (int rc = make_map(&mb, g.elem, 2, g.b, dims, strides, box)) return rc;
    }
    if (g.a_mode == kAModeRows) {
        if ((g.lda * es) % 16) return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: A rows must be 16-byte multiples");
        const cuuint64_t dims[2] = {g.k, g.m};
        const cuuint64_t strides[1] = {g.lda * es};
        const cuuint32_t box[2] = {bk, 128};
        if (int rc = make_map(&ma, g.elem, 2, g.a, dims, strides, box)) return rc;
        p.num_m_tiles = (g.m + 127) / 128;
        p.num_kb = (g.k + bk - 1) / bk;
    } else {
        if (g.conv_c % bk) return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: conv channels must be a multiple of 128 bytes");
        if (g.k != 9 * g.conv_c) return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: conv K must be 9*C");
        const cuuint64_t dims[4] = {g.conv_c, g.conv_w, g.conv_h, g.conv_batch};
        const cuuint64_t strides[3] = {(cuuint64_t)g.conv_c * es, (cuuint64_t)g.conv_c * g.conv_w * es,
                                       (cuuint64_t)g.conv_c * g.conv_w * g.conv_h * es};
        const cuuint32_t box[4] = {bk, 16, 8, 1};
        if (int rc = make_map(&ma, g.elem, 4, g.a, dims, strides, box)) return rc;
        p.conv_h = g.conv_h;
        p.conv_w = g.conv_w;
        p.tiles_x = (g.conv_w + 15) / 16;
        p.tiles_y = (g.conv_h + 7) / 8;
        p.kb_per_tap = g.conv_c / bk;
        p.num_m_tiles = p.tiles_x * p.tiles_y * g.conv_batch;
        p.num_kb = 9 * p.kb_per_tap;
        if (g.m != g.conv_batch * g.conv_h * g.conv_w)
            return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: conv M must be batch*H*W");
    }
    // Thread-row epilogue with TMA stores: row-major outputs without row
    // remap (linear layers, 1x1 convolutions) or channels-last outputs of the
    // implicit convolution with 16-bit operands; whole tiles along N, 16-byte
    // aligned rows; residuals in the output's layout.
    EpiMaps em;
    em.out = em.out2 = em.res1 = em.res2 = mb;  // placeholders when unused (never read)
    uint32_t staging = kSlabBytes;
    bool epi8 = false;
    p.tma_program = kTmaNone;
    const bool conv = g.a_mode != kAModeRows;
    if (conv && g.elem != kElemS8 && bn == 32 && g.n == 32 && g.out_kind == kOutHeadF32 &&
        (g.flags & ~uint32_t(kEpiMetricHead)) == (kEpiBias | kEpiHeadDot) &&
        reinterpret_cast<uintptr_t>(g.bias) % 16 == 0 && reinterpret_cast<uintptr_t>(g.head_w) % 16 == 0)
        p.tma_program = kTmaHeadDot;  // 8-warp kernel; needs no staging area, so the ring can be deeper
    if (!conv && g.out_kind == kOutConvTHalf && (g.flags & ~uint32_t(kEpiDequant)) == kEpiBias &&
        ((g.flags & kEpiDequant) != 0) == (g.elem == kElemS8) && g.convt_cout % 32 == 0 && g.n % bn == 0 &&
        reinterpret_cast<uintptr_t>(g.out) % 16 == 0 && g.ldo % 8 == 0 && reinterpret_cast<uintptr_t>(g.bias) % 16 == 0 &&
        (!(g.flags & kEpiDequant) || reinterpret_cast<uintptr_t>(g.s_w) % 16 == 0))
        p.tma_program = kTmaHalfBiasCT;  // 16-warp kernel, direct stores: no staging area
    if (g.out_slot && p.tma_program != kTmaHeadDot)
        return set_error(DAV2CUDA_INVALID_ARGUMENT, "gemm: an output slot needs the output-head epilogue");
    if (p.tma_program == kTmaHeadDot || p.tma_program == kTmaHalfBiasCT) staging = 0;
    if (p.tma_program == kTmaNone && (!conv || g.elem != kElemS8) && !p.rows_per_img &&
        (g.out_kind == kOutF32Rows || g.out_kind == kOutHalfRows) && !(g.flags & kEpiHeadDot) &&
        ((g.flags & kEpiDequant) != 0) == (g.elem == kElemS8) && g.n % bn == 0) {
        const bool f32 = g.out_kind == kOutF32Rows;
        const uint32_t oes = f32 ? 4u : 2u;
        const uint32_t f = g.flags & ~uint32_t(kEpiDequant);
        int prog = kTmaNone;
        if (f32) {
            if (conv) prog = kTmaNone;
            else if (f == 0) prog = kTmaF32;
            else if (f == kEpiBias) prog = kTmaF32Bias;
            else if (f == (kEpiBias | kEpiGelu)) prog = kTmaF32BiasGelu;
            else if (f == (kEpiBias | kEpiLayerScale)) prog = kTmaF32BiasLS;
        } else {
            if (f == 0) prog = kTmaHalf;
            else if (f == kEpiBias) prog = kTmaHalfBias;
            else if (f == (kEpiBias | kEpiGelu) && !conv) prog = kTmaHalfBiasGelu;
            else if (f == (kEpiBias | kEpiRelu)) prog = kTmaHalfBiasRelu;
            else if (f == kEpiReluCopy) prog = kTmaHalfRC;
            else if (f == (kEpiBias | kEpiResidual1)) prog = kTmaHalfBiasR1;
            else if (f == (kEpiBias | kEpiResidual1 | kEpiResidual2 | kEpiReluCopy)) prog = kTmaHalfBiasR1R2RC;
        }
        auto a16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
        const bool uses_r1 = prog == kTmaF32BiasLS || prog == kTmaHalfBiasR1 || prog == kTmaHalfBiasR1R2RC;
        const bool uses_r2 = prog == kTmaHalfBiasR1R2RC;
        const bool uses_o2 = prog == kTmaHalfRC || prog == kTmaHalfBiasR1R2RC;
        const bool aligned = a16(g.out) && (g.ldo * oes) % 16 == 0 && (!uses_r1 || a16(g.res1)) &&
                             (!uses_r2 || a16(g.res2)) && (!uses_o2 || a16(g.out2));
        const bool params_aligned = (!(g.flags & kEpiDequant) || a16(g.s_w)) && (!(g.flags & kEpiBias) || a16(g.bias)) &&
                                    (prog != kTmaF32BiasLS || a16(g.gamma));
        if (prog != kTmaNone && aligned && params_aligned) {
            const CUtensorMapDataType t =
                f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                    : (g.out_half_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
            const CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_64B;
            auto make = [&](CUtensorMap* m, const void* base) -> int {
                if (!conv) {
                    const cuuint64_t dims[2] = {g.n, g.m};
                    const cuuint64_t strides[1] = {g.ldo * oes};
                    const cuuint32_t box[2] = {f32 ? 16u : 32u, 32u};  // 64-byte rows, 32 rows
                    return make_map_typed(m, t, 2, base, dims, strides, box, sw);
                }
                // channels-last [B][H][W][ldo]; box = 2 image rows x 16 pixels
                const cuuint64_t dims[4] = {g.n, g.conv_w, g.conv_h, g.conv_batch};
                const cuuint64_t strides[3] = {g.ldo * oes, (cuuint64_t)g.conv_w * g.ldo * oes,
                                               (cuuint64_t)g.conv_h * g.conv_w * g.ldo * oes};
                const cuuint32_t box[4] = {32u, 16u, 2u, 1u};
                return make_map_typed(m, t, 4, base, dims, strides, box, sw);
            };
            if (int rc = make(&em.out, g.out)) return rc;
            if (uses_o2)
                if (int rc = make(&em.out2, g.out2)) return rc;
            if (uses_r1)
                if (int rc = make(&em.res1, g.res1)) return rc;
            if (uses_r2)
                if (int rc = make(&em.res2, g.res2)) return rc;
            p.tma_program = prog;
            // epilogue warps x 2 boxes (the 8-warp kernel's staging area is the
            // transposed-store slab, which is larger)
            // the LayerScale residual with a long K loop (fc2: 13 us of MMA per
            // tile covers its epilogue) runs with 8 epilogue warps: half the
            // staging boxes, one more ring stage at BN = 256 (measured: qkv's
            // epilogue needs 16 warps)
            epi8 = !conv && prog == kTmaF32BiasLS && g.k >= 2048;
            staging = conv ? kSlabBytes : (epi8 ? 8u : 16u) * 2u * kStageBufBytes;
        }
    }
    const int mc = g.max_ctas;
    if (g.a_mode == kAModeRows) {
        switch (g.elem) {
            case kElemS8: return dispatch_s8_rows(bn, ma, mb, em, p, staging, mc, st, epi8);
            case kElemF16: return dispatch_f16_rows(bn, ma, mb, em, p, staging, mc, st, epi8);
            default: return dispatch_bf16_rows(bn, ma, mb, em, p, staging, mc, st, epi8);
        }
    }
    switch (g.elem) {
        case kElemS8: return dispatch_s8_conv(bn, ma, mb, em, p, staging, mc, st, epi8);
        case kElemF16: return dispatch_f16_conv(bn, ma, mb, em, p, staging, mc, st, epi8);
        default: return dispatch_bf16_conv(bn, ma, mb, em, p, staging, mc, st, epi8);
    }
}

}  // namespace dav2cuda
