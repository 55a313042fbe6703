// Flash attention on tcgen05 tensor cores (head dim 64, f16 or bf16
// operands, f32 accumulation; output f16/bf16 or f32) — attention_head64 of the reference (src/operators.cpp:
// 1098-1209: QK^T*0.125 -> softmax_lastdim.glsl -> PV) without materialising
// the [heads, T, T] scores.
//
// Work unit = one (image, head, 256-query block) = two 128-query tiles that
// share every K/V block. The kernel is persistent: one CTA per SM (a kernel
// that allocates tensor memory is resident once per SM; all 512 TMEM columns)
// walks units blockIdx.x, blockIdx.x + gridDim.x, ..., so that the next
// unit's Q, first K/V blocks and first S overlap the current unit's last
// blocks and output merge. Units whose second tile lies past T (one live
// tile) are numbered after all two-tile units, which spreads them evenly over
// the CTAs. Tile t uses TMEM columns 256t + [0,128) for S and 256t + 128 + 64h
// for O_h, h = key half.
//   warp 0       TMA: per unit the Q tiles (loaded as soon as the previous
//                unit's last S is computed), then K_j / V_j (128 keys x 64
//                dims each) into a 4-stage ring that
//                runs on across units. The 3-D tensor map over qkv [B][T][3E]
//                zero-fills rows past T.
//   warps 1, 18  MMA issuers, one per tile (so neither tile's pipeline waits
//                on the other; a K/V stage is released once both have
//                committed — the issuer of a tile with no rows in a unit
//                releases each stage as soon as it is filled): S_{j+1} =
//                Q K_{j+1}^T (M=128, N=128, K=64) as soon as the tile's softmax
//                holds S_j in registers, so it is computed while that softmax
//                works on block j; then, once P_j is published, O_h +=
//                P_j[:, 64h:64h+64] V_j[64h:64h+64, :] for both key halves
//                (M=128, N=64, K=64; V read as an MN-major operand),
//                accumulating in TMEM across key blocks.
//   warps 2..9   softmax of tile 0, warps 10..17 of tile 1: two warps per query
//                row (TMEM lane), warp half h owning keys [64h, 64h+64) of every
//                block with its own running maximum m_h, sum l_h and O_h — an
//                independent online softmax per key half, merged once per unit.
//                Per block: S loaded once into registers, row maximum,
//                P = exp2(s*c - m*c) (f16) into a 128-byte-swizzled shared tile,
//                l_h += sum(P). The maximum used for P is only raised when the
//                block maximum exceeds it by more than 8 (log2 units): P stays
//                <= 2^8 and O_h in TMEM is rescaled only on those rare raises.
//                Full key blocks skip the key-range mask. The two tiles take
//                turns for the exponentials (the issue- and MUFU-heavy phase), so each
//                tile's other work overlaps the other tile's exp phase.
// Ordering between the roles uses mbarriers whose phases are counted across
// units; every wait is bounded and a timeout sets the device error word
// instead of hanging.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>

namespace dav2cuda {
namespace {

struct AttnParams {
    uint32_t tokens, heads, num_kb;
    uint32_t units;       // batch * heads * query blocks
    uint32_t full_units;  // units with two live tiles, numbered first
    uint32_t full_per_bh; // two-tile units per (image, head)
    uint64_t out_ld;
    void* out;        // [B*T][out_ld]: the operand type, or f32 when out_f32
    uint32_t out_f32;
    int* err;
};

constexpr uint32_t kQTiles = 2;       // 128-query tiles per unit
constexpr uint32_t kQ = 128 * kQTiles;  // queries per unit
constexpr uint32_t kQBufs = 1;        // Q buffers per tile
constexpr uint32_t kKV = 128;         // keys per block
// K/V ring depth and P buffers per tile (P_j in buffer j % kPBufs). Measured
// on B200 (ViT-L, 64 images, one launch): 1 Q buffer x 4 stages x 1 P buffer
// 0.839 ms, 2 x 3 x 1 0.846 ms, 1 x 2 x 2 (the only double-buffered-P layout
// that fits) 1.006 ms: its K/V ring runs dry.
constexpr uint32_t kStages = 4;
constexpr uint32_t kPBufs = 1;
constexpr uint32_t kTile = 128 * 128; // bytes of a 128 x 64 f16 tile
constexpr uint32_t kThreads = 64 + 256 * kQTiles + 32;  // TMA, MMA(tile 0), softmax, MMA(tile 1)
constexpr uint32_t kMma1Warp = 2 + 8 * kQTiles;
// Q[tile][buffer], K[stage], V[stage], P[tile][buffer][key half], 1 KB barriers
constexpr uint32_t kSmem = kTile * (kQBufs * kQTiles + 2 * kStages + 2 * kPBufs * kQTiles) + 1024;
constexpr uint32_t kBarrierBytes = 8 * (2 * kStages + 2 * kQBufs * kQTiles + (6 + kPBufs) * kQTiles) + 8;
static_assert(kQTiles == 2, "unit decoding assumes two tiles per unit");
static_assert(kBarrierBytes <= 1024, "barrier block overflows its 1 KB");
static_assert(kSmem <= 232448, "shared memory above the per-block limit");

// 8-column TMEM row access (the rare O rescale; keeps register use low)
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x of two f16 values at once (one exponential-unit operation).
__device__ __forceinline__ uint32_t ex2_h2(uint32_t x) {
    uint32_t y;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ __half2 as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }


// Packed f32x2 arithmetic of sm_100 (two IEEE fp32 lanes per instruction,
// each lane rounded exactly as the scalar operation) and the three-input
// maximum: they halve the issue slots of the softmax's per-score work.
__device__ __forceinline__ uint64_t pack_f32x2(float lo, float hi) {
    return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}

__device__ __forceinline__ void ffma2(float& x0, float& x1, uint64_t mul, uint64_t add) {
    asm("{\n\t.reg .b64 a;\n\tmov.b64 a, {%0, %1};\n\tfma.rn.f32x2 a, a, %2, %3;\n\tmov.b64 {%0, %1}, a;\n\t}"
        : "+f"(x0), "+f"(x1)
        : "l"(mul), "l"(add));
}

__device__ __forceinline__ void fadd2(float& a0, float& a1, float x0, float x1) {
    asm("{\n\t.reg .b64 a, b;\n\tmov.b64 a, {%0, %1};\n\tmov.b64 b, {%2, %3};\n\tadd.rn.f32x2 a, a, b;\n\t"
        "mov.b64 {%0, %1}, a;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(x0), "f"(x1));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr) {
    // MN-major operand, 128-byte swizzle: 8-row (K) groups 1024 B apart.
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

struct Unit {
    uint32_t img, head, q0, ntiles;
};

// Two-tile units first, (image, head)-major with the query block fastest
// (the units of one (image, head) run side by side and share K/V in L2), then
// the single-tile units (query block past T - 128), one per (image, head).
__device__ __forceinline__ Unit unit_at(const AttnParams& p, uint32_t u) {
    uint32_t bh, qb;
    if (u < p.full_units) {
        bh = u / p.full_per_bh;
        qb = u - bh * p.full_per_bh;
    } else {
        bh = u - p.full_units;
        qb = p.full_per_bh;
    }
    Unit w;
    w.head = bh % p.heads;
    w.img = bh / p.heads;
    w.q0 = qb * kQ;
    w.ntiles = p.tokens - w.q0 > 128u ? 2u : 1u;
    return w;
}

// Two f32 values as a packed f16x2 or bf16x2 word (round to nearest even).
template <bool kBF16>
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    if constexpr (kBF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm, const AttnParams p) {
    extern __shared__ uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if ((smem_addr(smem) & 1023u) != 0) {  // the 128-byte swizzle needs 1 KB aligned tiles
        if (threadIdx.x == 0) atomicExch(p.err, 2);
        return;
    }
    uint8_t* sQ = smem;                                // [tile][buffer]
    uint8_t* sK = smem + kQBufs * kQTiles * kTile;     // [stage]
    uint8_t* sV = sK + kStages * kTile;                // [stage]
    uint8_t* sP = sV + kStages * kTile;                // [tile][buffer][key half]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBufs * kQTiles * kTile);
    uint64_t* q_full = bars;                           // [tile][buffer]
    uint64_t* q_empty = q_full + kQBufs * kQTiles;     // [tile][buffer]
    uint64_t* kv_full = q_empty + kQBufs * kQTiles;    // [stage]
    uint64_t* kv_empty = kv_full + kStages;    // [stage]
    uint64_t* s_full = kv_empty + kStages;     // [tile]
    uint64_t* s_empty = s_full + kQTiles;      // [tile]
    uint64_t* p_full = s_empty + kQTiles;      // [tile]
    uint64_t* p_empty = p_full + kQTiles;      // [tile][buffer]
    uint64_t* o_full = p_empty + kPBufs * kQTiles;  // [tile]
    uint64_t* drain = o_full + kQTiles;        // [tile]
    uint64_t* turn = drain + kQTiles;          // [tile]: the tile may run its exp phase
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(turn + kQTiles);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const uint32_t E = p.heads * 64u;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm);
        for (uint32_t t = 0; t < kQTiles; ++t) {
            for (uint32_t b = 0; b < kQBufs; ++b) {
                mbar_init(&q_full[kQBufs * t + b], 1);
                mbar_init(&q_empty[kQBufs * t + b], 1);
            }
            mbar_init(&s_full[t], 1);
            mbar_init(&p_full[t], 8);
            for (uint32_t b = 0; b < kPBufs; ++b) mbar_init(&p_empty[kPBufs * t + b], 1);
            mbar_init(&o_full[t], 1);
            mbar_init(&s_empty[t], 8);
            mbar_init(&drain[t], 1);
            mbar_init(&turn[t], 8);
        }
        for (uint32_t st = 0; st < kStages; ++st) {
            mbar_init(&kv_full[st], 1);
            mbar_init(&kv_empty[st], kQTiles);  // one release per tile issuer and block
        }
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
            uint32_t g = 0;                        // K/V blocks loaded so far (all units)
            uint32_t qn[kQTiles] = {0u, 0u};       // Q tiles loaded so far, per tile
            bool ok = true;
            for (uint32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
#pragma unroll
                for (uint32_t t = 0; t < kQTiles; ++t) {
                    if (t >= w.ntiles || !ok) break;
                    const uint32_t b = qn[t] % kQBufs;
                    // the buffer's previous Q (two units back) must be done
                    if (qn[t] >= kQBufs &&
                        !mbar_wait(&q_empty[kQBufs * t + b], ((qn[t] / kQBufs) - 1u) & 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&q_full[kQBufs * t + b], kTile);
                    tma_load_3d(sQ + (kQBufs * t + b) * kTile, &tm, &q_full[kQBufs * t + b], (int)(w.head * 64u),
                                (int)(w.q0 + 128u * t), (int)w.img);
                    ++qn[t];
                }
                for (uint32_t j = 0; ok && j < nkb; ++j, ++g) {
                    const uint32_t st = g % kStages;
                    if (*abort_flag || !mbar_wait(&kv_empty[st], ((g / kStages) & 1u) ^ 1u, abort_flag, p.err)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&kv_full[st], 2 * kTile);
                    tma_load_3d(sK + st * kTile, &tm, &kv_full[st], (int)(E + w.head * 64u), (int)(j * kKV),
                                (int)w.img);
                    tma_load_3d(sV + st * kTile, &tm, &kv_full[st], (int)(2 * E + w.head * 64u), (int)(j * kKV),
                                (int)w.img);
                }
            }
        }
    } else if (warp == 1 || warp == kMma1Warp) {
        // one MMA issuer per tile, so that neither tile's pipeline waits on the other
        const uint32_t t = warp == 1 ? 0u : 1u;
        if (lane == 0) {
            constexpr uint32_t ab = kBF16 ? 1u : 0u;  // kind::f16 operand format: 0 f16, 1 bf16
            constexpr uint32_t idesc_s = make_idesc(1u, ab, 128u, 128u);
            constexpr uint32_t idesc_o = make_idesc(1u, ab, 128u, 64u) | (1u << 16);  // B (V) MN-major
            uint32_t g = 0;   // K/V blocks consumed (all units)
            uint32_t gt = 0;  // blocks this tile has computed (its S/P/O barrier phases)
            uint32_t qn = 0;  // units this tile has computed (its Q buffer phases)
            bool ok = true;
            for (uint32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
                const Unit w = unit_at(p, u);
                if (t >= w.ntiles) {
                    // no rows of this tile in the unit: release each K/V stage once
                    // it is filled (the fill proves the stage's previous phase is over)
                    for (uint32_t j = 0; j < nkb; ++j, ++g) {
                        const uint32_t st = g % kStages;
                        if (!mbar_wait(&kv_full[st], (g / kStages) & 1u, abort_flag, p.err)) {
                            ok = false;
                            break;
                        }
                        mbar_arrive(&kv_empty[st]);
                    }
                    continue;
                }
                const uint32_t qbuf = kQBufs * t + qn % kQBufs;
                const uint32_t q_addr = smem_addr(sQ + qbuf * kTile);
                auto issue_s = [&](uint32_t gg) {
                    const uint32_t k_addr = smem_addr(sK + (gg % kStages) * kTile);
#pragma unroll
                    for (uint32_t kk = 0; kk < 4; ++kk)
                        umma<false>(tmem + 256u * t, smem_desc_sw128(q_addr + 32u * kk),
                                    smem_desc_sw128(k_addr + 32u * kk), idesc_s, kk ? 1u : 0u);
                    umma_commit(&s_full[t]);
                };
                auto issue_o = [&](uint32_t gg, uint32_t j, uint32_t gtt) {
                    const uint32_t v_addr = smem_addr(sV + (gg % kStages) * kTile);
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h) {
                        const uint32_t p_addr = smem_addr(sP + ((kPBufs * t + gtt % kPBufs) * 2u + h) * kTile);
#pragma unroll
                        for (uint32_t kk = 0; kk < 4; ++kk)
                            umma<false>(tmem + 256u * t + 128u + 64u * h, smem_desc_sw128(p_addr + 32u * kk),
                                        desc_mn_sw128(v_addr + (4u * h + kk) * 2048u), idesc_o, (j | kk) ? 1u : 0u);
                    }
                    umma_commit(&o_full[t]);
                    umma_commit(&p_empty[kPBufs * t + gtt % kPBufs]);
                    umma_commit(&kv_empty[gg % kStages]);
                };
                // S_0 needs this unit's Q, K_0 and the S columns back from the
                // softmax (it loaded the previous unit's last S)
                ok = mbar_wait(&q_full[qbuf], (qn / kQBufs) & 1u, abort_flag, p.err) &&
                     mbar_wait(&kv_full[g % kStages], (g / kStages) & 1u, abort_flag, p.err) &&
                     (gt == 0 || mbar_wait(&s_empty[t], (gt - 1u) & 1u, abort_flag, p.err));
                if (!ok) break;
                tc_fence_after();
                issue_s(g);
                mma_issued = true;
                if (nkb == 1) umma_commit(&q_empty[qbuf]);
                for (uint32_t j = 0; j < nkb; ++j) {
                    const uint32_t gg = g + j, gtt = gt + j;
                    // S_{j+1} as soon as the softmax holds S_j in registers (it is
                    // computed while that softmax works on block j) ...
                    if (j + 1 < nkb) {
                        ok = mbar_wait(&kv_full[(gg + 1) % kStages], ((gg + 1) / kStages) & 1u, abort_flag, p.err) &&
                             mbar_wait(&s_empty[t], gtt & 1u, abort_flag, p.err);
                        if (!ok) break;
                        tc_fence_after();
                        issue_s(gg + 1);
                        if (j + 2 == nkb) umma_commit(&q_empty[qbuf]);  // the unit's last read of Q
                    }
                    // ... and the O updates of block j once its P is published (the
                    // softmax has also rescaled O, or read out the previous unit's
                    // O, by then)
                    ok = mbar_wait(&p_full[t], gtt & 1u, abort_flag, p.err);
                    if (!ok) break;
                    tc_fence_after();
                    issue_o(gg, j, gtt);
                }
                g += nkb;
                gt += nkb;
                ++qn;
            }
        }
    } else {
        const uint32_t t = (warp - 2u) / 8u;
        const uint32_t quarter = warp & 3u;
        const uint32_t half = ((warp - 2u) >> 2) & 1u;
        const uint32_t row = quarter * 32u + lane;
        const uint32_t tS = tmem + 256u * t + ((quarter * 32u) << 16);  // S of this lane quarter
        const uint32_t tO = tS + 128u + 64u * half;                      // this key half's O
        const uint32_t pair_id = t * 4u + quarter;  // named barrier 1 + pair_id, shared by the two warps
        const float c = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        constexpr float kRaise = 8.0f;                 // raise the maximum only beyond 2^8
        uint8_t* atoms = sP + (kPBufs * t * 2u + half) * kTile + row * 128u;  // + 2*kTile per buffer
        // warp-uniform wait: on a timeout every lane leaves together, so the
        // warp-collective TMEM accesses and votes below never diverge
        auto warp_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, p.err));
        };
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
        uint32_t gt = 0;  // blocks this tile has computed (its S/P/O barrier phases)
        uint32_t b2 = 0;  // blocks of two-tile units (the turn phases)
        bool ok = true;
        for (uint32_t u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
            const bool turns = unit_at(p, u).ntiles == 2;
            if (t == 1 && !turns) continue;
            float m = -INFINITY, l = 0.f;
            for (uint32_t j = 0; j < nkb; ++j) {
                const uint32_t gtt = gt + j, bt = b2 + j;
                if (!warp_wait(&s_full[t], gtt & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t sr[2][32];
                tmem_ld_32x32b_x32(tS + 64u * half, sr[0]);
                tmem_ld_32x32b_x32(tS + 64u * half + 32u, sr[1]);
                tmem_ld_wait();
                // S_j is in registers: its TMEM columns may take S_{j+1}
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_empty[t]);
                float s[64];
#pragma unroll
                for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(sr[i >> 5][i & 31]);
                const uint32_t kbase = j * kKV + 64u * half;
                if (kbase + 64u > p.tokens) {  // tail block: keys >= T do not exist
#pragma unroll
                    for (int i = 0; i < 64; ++i)
                        if (kbase + i >= p.tokens) s[i] = -INFINITY;
                }
                // row maximum by a tree of three-input maxima (32 operations, depth 4)
                float ma[22], mb[8];
#pragma unroll
                for (int i = 0; i < 21; ++i) ma[i] = fmax3(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
                ma[21] = s[63];
#pragma unroll
                for (int i = 0; i < 7; ++i) mb[i] = fmax3(ma[3 * i], ma[3 * i + 1], ma[3 * i + 2]);
                mb[7] = ma[21];
                const float mx = fmax3(fmax3(mb[0], mb[1], mb[2]), fmax3(mb[3], mb[4], mb[5]), fmax3(mb[6], mb[7], m));
                if (j == 0) {
                    m = mx;
                } else {
                    const bool raise = (mx - m) * c > kRaise;  // false while both are -inf
                    if (__any_sync(0xffffffffu, raise)) {
                        // O_h must hold blocks 0..j-1 before it is rescaled
                        if (!warp_wait(&o_full[t], (gtt - 1u) & 1u)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const float alpha = raise ? ex2_approx((m - mx) * c) : 1.0f;
#pragma unroll 1
                        for (uint32_t k = 0; k < 8; ++k) {
                            uint32_t ov[8];
                            tmem_ld_x8(tO + 8u * k, ov);
                            tmem_ld_wait();
#pragma unroll
                            for (int i = 0; i < 8; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
                            tmem_st_x8(tO + 8u * k, ov);
                        }
                        tmem_st_wait();
                        if (raise) {
                            l *= alpha;
                            m = mx;
                        }
                    }
                }
                const float mc = m == -INFINITY ? 0.f : m * c;  // a half with no key yet has P = 0
                // the MMA that last read this P buffer (kPBufs blocks back) must be done
                if (!warp_wait(&p_empty[kPBufs * t + gtt % kPBufs], ((gtt / kPBufs) & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                // ping-pong: in two-tile units the exp phases alternate (tile 0
                // block j, tile 1 block j, tile 0 block j+1, ...; counted across
                // units), so that each tile's max, loads and waits overlap the
                // other tile's exponentials
                if (turns && (t == 1 || bt > 0) && !warp_wait(&turn[t], (t == 0 ? bt - 1u : bt) & 1u)) {
                    ok = false;
                    break;
                }
                // all 64 exponentials first (independent, in place: the MUFU queue
                // stays full; arguments s*c - m*c two at a time), then eight
                // partial sums (pairwise) and the f16 P tile
                const uint64_t mul2 = pack_f32x2(c, c), add2 = pack_f32x2(-mc, -mc);
#pragma unroll
                for (int i = 0; i < 64; i += 2) ffma2(s[i], s[i + 1], mul2, add2);
                float ls[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                if constexpr (!kBF16) {
                    // f16 P: the exponent arguments (s - m)*c rounded to f16 pairs
                    // and exponentiated two per MUFU operation (ex2.approx.f16x2),
                    // which halves the exponential unit's work. The reference's fp16
                    // attention rounds the scores themselves to f16 before its
                    // softmax (bmm_score_fp16.glsl, softmax_lastdim_half.glsl), a
                    // coarser rounding than this one of the max-shifted argument.
                    // Row sum of the block: a pairwise f16x2 tree over the 64 P
                    // values (six levels), converted to f32 once and added to l in f32.
                    uint32_t h[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) h[i] = pack_h2<false>(s[2 * i], s[2 * i + 1]);
#pragma unroll
                    for (int i = 0; i < 32; ++i) h[i] = ex2_h2(h[i]);
                    __half2 part[8];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        part[q] = __hadd2(__hadd2(as_h2(h[4 * q]), as_h2(h[4 * q + 1])),
                                          __hadd2(as_h2(h[4 * q + 2]), as_h2(h[4 * q + 3])));
                        *reinterpret_cast<uint4*>(atoms + (gtt % kPBufs) * 2u * kTile +
                                                  (((uint32_t)q ^ (row & 7u)) << 4)) =
                            make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
                    }
                    const __half2 t4 = __hadd2(__hadd2(__hadd2(part[0], part[1]), __hadd2(part[2], part[3])),
                                               __hadd2(__hadd2(part[4], part[5]), __hadd2(part[6], part[7])));
                    const float2 f = __half22float2(t4);
                    ls[0] = f.x + f.y;
                } else {
#pragma unroll
                    for (int i = 0; i < 64; ++i) s[i] = ex2_approx(s[i]);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        uint32_t hv[4];
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            fadd2(ls[2 * v], ls[2 * v + 1], s[8 * q + 2 * v], s[8 * q + 2 * v + 1]);
                            hv[v] = pack_h2<true>(s[8 * q + 2 * v], s[8 * q + 2 * v + 1]);
                        }
                        *reinterpret_cast<uint4*>(atoms + (gtt % kPBufs) * 2u * kTile +
                                                  (((uint32_t)q ^ (row & 7u)) << 4)) =
                            make_uint4(hv[0], hv[1], hv[2], hv[3]);
                    }
                }
                l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
                tc_fence_before();
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&p_full[t]);
                    if (turns) mbar_arrive(&turn[t ^ 1u]);
                }
            }
            gt += nkb;
            if (turns) b2 += nkb;
            // merge the two key halves: m = max(m0, m1), weights exp2((m_h - m) c).
            // Both warps of a pair always reach both pair barriers (also after a
            // timeout) and leave the unit loop together.
            if (ok) ok = warp_wait(&o_full[t], (gt - 1u) & 1u);  // the unit's last O (and P read) is done
            tc_fence_after();
            // (m, l, ok) travel through this row's own P atoms, free until this
            // warp writes the next unit's first P
            *reinterpret_cast<float4*>(atoms) = make_float4(m, l, ok ? 1.f : 0.f, 0.f);
            pair_sync();
            const float4 other = *reinterpret_cast<const float4*>(half ? atoms - kTile : atoms + kTile);
            pair_sync();  // the partner has read this row's values before they are overwritten
            ok = ok && other.z != 0.f;
            const float m_o = other.x, l_o = other.y;
            const float mm = fmaxf(m, m_o);
            const float f_own = ex2_approx((m - mm) * c), f_oth = ex2_approx((m_o - mm) * c);
            const float inv = 1.0f / fmaxf(l * f_own + l_o * f_oth, 1.0e-30f);
            // this warp writes output dims [32*half, 32*half+32): its own O_h and the
            // partner's O_{1-h} for those dims
            uint32_t oa[32], ob[32];
            tmem_ld_32x32b_x32(tO + 32u * half, oa);
            tmem_ld_32x32b_x32(tS + 128u + 64u * (half ^ 1u) + 32u * half, ob);
            tmem_ld_wait();
            // O is in registers: the next unit's first O MMA (ordered after this
            // warp's next P publication) may overwrite it
            tc_fence_before();
            const Unit w = unit_at(p, u);
            const uint32_t qrow = w.q0 + 128u * t + row;
            if (ok && qrow < p.tokens) {
                const float wa = f_own * inv, wb = f_oth * inv;
                const uint64_t at = ((uint64_t)w.img * p.tokens + qrow) * p.out_ld + w.head * 64u + half * 32u;
#pragma unroll
                for (int i = 0; i < 32; i += 8) {
                    float x[8];
#pragma unroll
                    for (int v = 0; v < 8; ++v)
                        x[v] = __uint_as_float(oa[i + v]) * wa + __uint_as_float(ob[i + v]) * wb;
                    if (p.out_f32) {
                        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + at + i);
                        dst[0] = make_float4(x[0], x[1], x[2], x[3]);
                        dst[1] = make_float4(x[4], x[5], x[6], x[7]);
                    } else {
                        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + at + i) =
                            make_uint4(pack_h2<kBF16>(x[0], x[1]), pack_h2<kBF16>(x[2], x[3]),
                                       pack_h2<kBF16>(x[4], x[5]), pack_h2<kBF16>(x[6], x[7]));
                    }
                }
            }
        }
    }

    __syncthreads();
    if (*abort_flag) {
        if ((warp == 1 || warp == kMma1Warp) && lane == 0 && mma_issued) {
            uint64_t* d = &drain[warp == 1 ? 0 : 1];
            umma_commit(d);
            const unsigned long long t0 = globaltimer();
            while (!mbar_try_wait(smem_addr(d), 0) && globaltimer() - t0 < 100000000ull) {
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

int launch_attention_tc(void* out, bool out_f32, const void* qkv, bool bf16, uint32_t batch, uint32_t tokens,
                        uint32_t heads, uint64_t qkv_ld, uint64_t out_ld, cudaStream_t st) {
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
    const CUresult rc = g_enc(&tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                              const_cast<void*>(qkv), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: tensor map encoding failed");
    auto kernel = bf16 ? attention_tc_kernel<true> : attention_tc_kernel<false>;
    static std::atomic<uint64_t> configured[2];  // one bit per device ordinal, per operand type
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured_on(configured[bf16], dev)) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess ||
            cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return set_error(DAV2CUDA_LAUNCH_FAILED, "attention: cannot set shared memory size");
        mark_configured(configured[bf16], dev);
    }
    AttnParams p;
    p.tokens = tokens;
    p.heads = heads;
    p.num_kb = (tokens + kKV - 1) / kKV;
    const uint32_t nqb = (tokens + kQ - 1) / kQ;
    const bool single_tail = tokens - (nqb - 1) * kQ <= 128u;  // the last query block has one live tile
    const uint64_t bh = (uint64_t)batch * heads;
    if (bh * nqb > 0xFFFFFFFFull) return set_error(DAV2CUDA_INVALID_ARGUMENT, "attention: too many work units");
    p.units = (uint32_t)(bh * nqb);
    p.full_per_bh = single_tail ? nqb - 1 : nqb;
    p.full_units = (uint32_t)(bh * p.full_per_bh);
    p.out_ld = out_ld;
    p.out = out;
    p.out_f32 = out_f32 ? 1u : 0u;
    p.err = device_error_word();
    if (!p.err) return set_error(DAV2CUDA_INTERNAL_ERROR, "attention: no device error word");
    const int sms = sm_count(dev);
    if (sms <= 0) return set_error(DAV2CUDA_LAUNCH_FAILED, "attention: cannot query the SM count");
    // persistent: one CTA per SM (the TMEM allocation keeps it at one), each
    // walking units blockIdx.x + k * gridDim.x
    const uint32_t grid = p.units < (uint32_t)sms ? p.units : (uint32_t)sms;
    kernel<<<grid, kThreads, kSmem, st>>>(tm, p);
    return check_launch("attention_tc");
}

}  // namespace dav2cuda
