// jt_moe_dn16.cu - down projection of the routed experts on the sm_100a
// tensor cores with bf16 operands (tcgen05.mma kind::f16, fp32 TMEM
// accumulators, TMA operand feed), fused with the weighted combine of
// moe_layer.c:1443-1463 (y[token] += w * y_pair).
//
// Arithmetic, for kept row r (token t, combine weight w_r) of expert e and
// output channel o:
//   wd16[o][k] = bf16_rn(code(o, k) * bf16_rn(s[k/64][o]))   code = 2 li - 15
//   y_pair[o]  = sum_k h[r][k] * wd16[o][k]        (fp32 in the tensor core)
//   y[t][o]   += w_r * y_pair[o]                   (fp32 atomic add)
// with h the bf16 SwiGLU output of the routed gate/up (jt_moe_gu16.cu).
// bf16 keeps h's range equal to fp32's; the group scale is rounded to bf16
// before the product so that the unpack forms each weight with one bf16
// multiply (both roundings are part of the specification).
//
// Tile: up to 256 token rows of one expert, run as one or two sub-tiles of
// 128 rows (MMA M, TMEM lane = token row), x 256 output channels (MMA N).
// One pipeline stage is one 64-K scale group: the h rows (16 KB per
// sub-tile, 128-byte swizzle), the packed INT4 codes of the 256 weight rows
// (8 KB) and their fp16 group scales (512 B) arrive by TMA; eight unpack
// warps turn the codes into bf16 weights in the 128-byte-swizzled K-major
// layout the MMA reads, in a separate ring of two 32 KB buffers, which both
// sub-tiles' MMAs read.  Each sub-tile accumulates the whole K in a TMEM
// accumulator of 256 columns; the two accumulators are used in turn, and
// the epilogue threads each own one token row and add 128 consecutive
// channels of it into the layer output with 16-byte vector atomics.
//
// Unpack (jt::int4_bf16x8): four operations per pair of weights after two
// masks per packed word.
//
// Warp roles (18 warps): w0 TMA producer (operand stages, per tile the row
// metadata; the next tile's weight rows are prefetched into L2), w1 TMEM
// allocator + MMA issuer, w2-9 unpack (one weight row per thread), w10-17
// epilogue (two warps per TMEM lane quarter, 128 channels each).  Every
// wait is a bounded mbarrier wait.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_runtime.cuh"

namespace {

constexpr int kBM = 128;                  // token rows per sub-tile (MMA M)
constexpr int kTile = JT_TILE_ROWS;       // token rows per tile
constexpr int kSubs = kTile / kBM;        // sub-tiles per tile
constexpr int kBN = 256;                  // output channels per tile (MMA N)
constexpr int kThreads = 576;             // 18 warps
constexpr int kUnpack0 = 2;               // warps 2-9
constexpr int kUnpackWarps = 8;
constexpr int kEpi0 = 10;                 // warps 10-17
constexpr int kEpiWarps = 8;
constexpr int kMaxStages = 8;
static_assert(kSubs == 2, "two accumulators, one per sub-tile");
constexpr int kBBufs = 2;
constexpr int kMaxGroups = 64;            // f <= 4096
constexpr uint32_t kX16 = kBM * 128;      // bf16 h rows of one 64-K group, 16 KB per sub-tile
constexpr uint32_t kOffPk = kSubs * kX16; // packed codes, 8 KB
constexpr uint32_t kPk = kBN * 32;
constexpr uint32_t kSc = kBN * 2;         // group scales, 512 B
constexpr uint32_t kStage = 41984;        // X16 [kSubs] | packed | scales, 1024-aligned
constexpr uint32_t kB16 = kBN * 128;      // bf16 weights of one 64-K group, 32 KB
constexpr uint32_t kSlot = 5120;          // info | row meta [kTile] float4
constexpr uint32_t kOffMeta = 128;
constexpr uint32_t kBarBytes = 1024;
constexpr size_t kSmemLimit = 232448;
constexpr size_t kFixed = 1024 + kBBufs * (size_t)kB16 + 2 * (size_t)kSlot + kBarBytes;
static_assert(kStage >= kOffPk + kPk + kSc && kStage % 1024 == 0, "stage layout");
static_assert(kOffMeta + kTile * 16 <= kSlot, "slot layout");

struct Dn16Params {
    CUtensorMap tmA;   // packed INT4 rows [E*d][f/2], 32 B x 256 boxes
    CUtensorMap tmH;   // bf16 h rows [rows][2f bytes], 128 B x 128 boxes, swizzled
    CUtensorMap tmS;   // fp16 group scales [E*G][d] as bytes, 256 B x 1 boxes (two per stage)
    CUtensorMap tmM;   // row metadata [rows][16 B]
    const uint8_t *wd; // the packed rows again, for the L2 prefetch of the next tile
    const int4 *tiles; // {e, row0, row_end, 0}
    const int32_t *ntiles;
    int d, f, G, stages;
    float *y;          // [T][d] fp32
    int y_accumulate;  // 1: y[token] += w * row (atomic); 0: y[token] = w * row
    int *err;
};

__device__ __forceinline__ void st_shared_v4u(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

__device__ __forceinline__ void red_add_v4(float *addr, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__global__ void __launch_bounds__(kThreads, 1) k_moe_dn16(const __grid_constant__ Dn16Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int S = p.stages, G = p.G;
    uint8_t *bbuf = smem + (size_t)S * kStage;
    uint8_t *slot_base = bbuf + kBBufs * kB16;
    uint64_t *full = reinterpret_cast<uint64_t *>(slot_base + 2 * kSlot);
    uint64_t *empty = full + kMaxStages;
    uint64_t *bfull = empty + kMaxStages;
    uint64_t *bempty = bfull + kBBufs;
    uint64_t *tfull = bempty + kBBufs;
    uint64_t *tempty = tfull + 2;
    uint64_t *pfull = tempty + 2;
    uint64_t *pempty = pfull + 2;
    uint64_t *drain = pempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = jt::warp_id(), lane = jt::lane_id();
    const int nch = (p.d + kBN - 1) / kBN;  // the last channel tile may hold 128
    const int total = __ldg(p.ntiles) * nch;
    int *err = p.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            jt::mbar_init(&full[s], 1);
            jt::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < kBBufs; ++b) {
            jt::mbar_init(&bfull[b], kUnpackWarps);
            jt::mbar_init(&bempty[b], 1);
        }
        for (int b = 0; b < 2; ++b) {
            jt::mbar_init(&tfull[b], 1);
            jt::mbar_init(&tempty[b], kEpiWarps);
            jt::mbar_init(&pfull[b], 1);
            jt::mbar_init(&pempty[b], kEpiWarps);
        }
        jt::mbar_init(drain, 1);
        *abort_flag = 0;
        jt::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        jt::prefetch_tmap(&p.tmA);
        jt::prefetch_tmap(&p.tmH);
        jt::prefetch_tmap(&p.tmS);
        jt::prefetch_tmap(&p.tmM);
    }
    if (warp == 1) {
        jt::tmem_alloc(tmem_slot, 2 * kBN);
        jt::tmem_relinquish();
    }
    jt::tc_fence_before();
    __syncthreads();
    jt::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued_mask = 0, issued_phase = 0;
            uint32_t ts = 0, tphase = 0, t_issued = 0, t_phase = 0;
            bool ok = true;
            // a tile's packed rows are contiguous: prefetch them into L2 (this
            // tile's first, then each next tile's while this one runs)
            const uint32_t prow = (uint32_t)(p.f / 2);
            auto prefetch_rows = [&](int uu) {
                const int ce = (uu % nch) * kBN;
                const int rows = min(kBN, p.d - ce);
                jt::prefetch_l2(p.wd + ((size_t)__ldg(&p.tiles[uu / nch]).x * p.d + ce) * prow, rows * prow);
            };
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const int4 te = __ldg(&p.tiles[u / nch]);
                const int c0 = (u % nch) * kBN;
                const int wrow = te.x * p.d + c0;
                if (u == (int)blockIdx.x) prefetch_rows(u);
                if (u + (int)gridDim.x < total) prefetch_rows(u + (int)gridDim.x);
                if (!jt::mbar_wait(&pempty[ts], tphase ^ 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                const int nsub = min(te.z - te.y, kTile) > kBM ? 2 : 1;
                uint8_t *sl = slot_base + ts * kSlot;
                asm volatile("st.shared.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(jt::smem_u32(sl)), "r"(te.x),
                             "r"(te.y), "r"(te.z), "r"(c0)
                             : "memory");
                jt::mbar_arrive_expect_tx(&pfull[ts], nsub * kBM * 16);
                for (int sb = 0; sb < nsub; ++sb)
                    jt::tma_load_2d(sl + kOffMeta + sb * kBM * 16, &p.tmM, &pfull[ts], 0, te.y + sb * kBM);
                t_issued |= 1u << ts;
                t_phase = (t_phase & ~(1u << ts)) | (tphase << ts);
                if (++ts == 2) {
                    ts = 0;
                    tphase ^= 1u;
                }
                for (int kb = 0; kb < G; ++kb) {
                    if (!jt::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = smem + (size_t)stage * kStage;
                    jt::mbar_arrive_expect_tx(&full[stage], nsub * kX16 + kPk + kSc);
                    for (int sb = 0; sb < nsub; ++sb)
                        jt::tma_load_2d(st + sb * kX16, &p.tmH, &full[stage], kb * 128, te.y + sb * kBM);
                    jt::tma_load_2d(st + kOffPk, &p.tmA, &full[stage], kb * 32, wrow);
                    jt::tma_load_2d(st + kOffPk + kPk, &p.tmS, &full[stage], c0 * 2, te.x * G + kb);
                    jt::tma_load_2d(st + kOffPk + kPk + 256, &p.tmS, &full[stage], c0 * 2 + 256, te.x * G + kb);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == (uint32_t)S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {  // every issued TMA box lands before the CTA exits
                for (int s = 0; s < S; ++s) {
                    if (!(issued_mask & (1u << s))) continue;
                    const long long t0 = clock64();
                    while (!jt::mbar_try_wait(&full[s], (issued_phase >> s) & 1u) &&
                           clock64() - t0 < JT_SPIN_CYCLES / 16) {
                    }
                }
                for (int s = 0; s < 2; ++s) {
                    if (!(t_issued & (1u << s))) continue;
                    const long long t0 = clock64();
                    while (!jt::mbar_try_wait(&pfull[s], (t_phase >> s) & 1u) &&
                           clock64() - t0 < JT_SPIN_CYCLES / 16) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            // accumulator use n goes to buffer n % 2; a tile takes one use per sub-tile
            uint32_t stage = 0, phase = 0, bb = 0, bphase = 0, n = 0;
            bool ok = true;
            constexpr uint32_t idesc = jt::idesc_bf16(kBM, kBN);
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const int4 te = __ldg(&p.tiles[u / nch]);
                const uint32_t nsub = min(te.z - te.y, kTile) > kBM ? 2u : 1u;
                for (uint32_t sb = 0; sb < nsub && ok; ++sb)
                    ok = jt::mbar_wait(&tempty[(n + sb) & 1u], ((n + sb) >> 1) & 1u, abort_flag, err);
                if (!ok) break;
                jt::tc_fence_after();
                for (int kb = 0; kb < G; ++kb) {
                    if (!jt::mbar_wait(&bfull[bb], bphase, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    jt::tc_fence_after();
                    const uint64_t dW = jt::umma_desc_sw128(jt::smem_u32(bbuf + bb * kB16));
                    for (uint32_t sb = 0; sb < nsub; ++sb) {
                        const uint32_t acc = tmem_base + ((n + sb) & 1u) * kBN;
                        const uint64_t dH =
                            jt::umma_desc_sw128(jt::smem_u32(smem + (size_t)stage * kStage + sb * kX16));
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks)
                            mma_bf16(acc, dH + 2u * ks, dW + 2u * ks, idesc, (kb | ks) != 0 ? 1u : 0u);
                    }
                    jt::mma_commit(&empty[stage]);
                    jt::mma_commit(&bempty[bb]);
                    if (++stage == (uint32_t)S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (++bb == (uint32_t)kBBufs) {
                        bb = 0;
                        bphase ^= 1u;
                    }
                }
                if (!ok) break;
                for (uint32_t sb = 0; sb < nsub; ++sb) jt::mma_commit(&tfull[(n + sb) & 1u]);
                n += nsub;
            }
            if (!ok) {  // already-issued MMAs retire before TMEM is released
                jt::mma_commit(drain);
                const long long t0 = clock64();
                while (!jt::mbar_try_wait(drain, 0) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
                }
            }
        }
    } else if (warp < kEpi0) {
        // ------------------------------------------------ unpack warps
        const int r = threadIdx.x - 32 * kUnpack0;  // weight row (output channel of the tile)
        const uint32_t r7 = static_cast<uint32_t>(r & 7);
        uint32_t stage = 0, phase = 0, bb = 0, bphase = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
            for (int kb = 0; kb < G; ++kb) {
                if (!jt::mbar_wait(&full[stage], phase, abort_flag, err) ||
                    !jt::mbar_wait(&bempty[bb], bphase ^ 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                const uint8_t *st = smem + (size_t)stage * kStage;
                const __half sh = reinterpret_cast<const __half *>(st + kOffPk + kPk)[r];
                const __nv_bfloat162 s2 = __bfloat162bfloat162(__float2bfloat16_rn(__half2float(sh)));
                const uint4 *pk = reinterpret_cast<const uint4 *>(st + kOffPk + r * 32);
                const uint32_t row_addr = jt::smem_u32(bbuf + bb * kB16) + static_cast<uint32_t>(r) * 128u;
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // 32 codes -> 32 weights = chunks 4h .. 4h+3
                    const uint4 a = pk[h];
                    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        uint32_t o[4];
                        jt::int4_bf16x8(w[i], s2, o);
                        st_shared_v4u(row_addr + ((((uint32_t)(4 * h + i)) ^ r7) << 4), o[0], o[1], o[2], o[3]);
                    }
                }
                jt::fence_proxy_async();
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&bfull[bb]);
                if (++stage == (uint32_t)S) {
                    stage = 0;
                    phase ^= 1u;
                }
                if (++bb == (uint32_t)kBBufs) {
                    bb = 0;
                    bphase ^= 1u;
                }
            }
        }
    } else {
        // ------------------------------------------------ epilogue warps
        // warp w: token rows 32 (w % 4) .. +31 of the tile (its TMEM lane
        // quarter), output channels 128 ((w - 10) / 4) .. +127 of the tile
        const int q = warp & 3;
        const int ch0 = ((warp - kEpi0) >> 2) * 128;
        const int j = q * 32 + lane;
        const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        __syncwarp();
        if (lane == 0) {
            jt::mbar_arrive(&tempty[0]);
            jt::mbar_arrive(&tempty[1]);
        }
        uint32_t n = 0, ts = 0, tphase = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
            if (!jt::mbar_wait(&pfull[ts], tphase, abort_flag, err)) {
                ok = false;
                break;
            }
            const uint8_t *sl = slot_base + ts * kSlot;
            const int4 info = *reinterpret_cast<const int4 *>(sl);  // {e, row0, row_end, c0}
            const int rows = min(info.z - info.y, kTile);
            const uint32_t nsub = rows > kBM ? 2u : 1u;
            float4 mt[kSubs];
#pragma unroll
            for (int sb = 0; sb < kSubs; ++sb) mt[sb] = reinterpret_cast<const float4 *>(sl + kOffMeta)[sb * kBM + j];
            const bool cols = ch0 < p.d - info.w;  // this warp's channels exist (last tile of d % 256 == 128)
            __syncwarp();
            if (lane == 0) jt::mbar_arrive(&pempty[ts]);
            if (++ts == 2) {
                ts = 0;
                tphase ^= 1u;
            }
            for (uint32_t sb = 0; sb < nsub && ok; ++sb, ++n) {
                const bool live = (int)sb * kBM + j < rows;
                const uint32_t buf = n & 1u;
                if (!jt::mbar_wait(&tfull[buf], (n >> 1) & 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                jt::tc_fence_after();
                const uint32_t acc = tq + buf * kBN + ch0;
                float *dst = p.y + (size_t)__float_as_int(mt[sb].z) * p.d + info.w + ch0;
                const float wr = mt[sb].y;
#pragma unroll 2
                for (int c = 0; c < 128; c += 16) {
                    uint32_t a0[8], a1[8];
                    jt::tmem_ld8(acc + c, a0);
                    jt::tmem_ld8(acc + c + 8, a1);
                    jt::tmem_wait_ld8(a0);
                    jt::tmem_wait_ld8(a1);
                    if (live && cols) {
                        float v[16];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            v[i] = __fmul_rn(wr, __uint_as_float(a0[i]));
                            v[8 + i] = __fmul_rn(wr, __uint_as_float(a1[i]));
                        }
                        if (p.y_accumulate) {
#pragma unroll
                            for (int i = 0; i < 16; i += 4)
                                red_add_v4(dst + c + i, v[i], v[i + 1], v[i + 2], v[i + 3]);
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; i += 4)
                                *reinterpret_cast<float4 *>(dst + c + i) =
                                    make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
                        }
                    }
                }
                jt::tc_fence_before();
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&tempty[buf]);
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        jt::tc_fence_after();
        jt::tmem_dealloc(tmem_base, 2 * kBN);
    }
}

}  // namespace

// Routed down: wd packed INT4 [E][d][f/2], ds fp16 [E][f/64][d]; h bf16
// [rows][f]; y[token][d] += w_row * y_pair (y_accumulate 1, atomic) or
// y[token] = w_row * y_pair (0: one output row per routed row).
extern "C" int jtk_moe_down_routed(const uint8_t *wd, const void *ds, int E, int d, int f, const uint16_t *h,
                                   int rows_cap, const float4 *row_meta, const int4 *tiles,
                                   const int32_t *ntiles, float *y, int y_accumulate, int max_tiles_hint,
                                   cudaStream_t stream) {
    if (d % 128 || f % 64 || f / 64 > kMaxGroups || E <= 0 || rows_cap <= 0) return -1;
    const int G = f / 64;
    Dn16Params p{};
    const uint32_t prow = f / 2;
    if (!jt::make_tmap_2d_u8(&p.tmA, wd, prow, (uint64_t)E * d, prow, 32, kBN, false) ||
        !jt::make_tmap_2d_u8(&p.tmH, h, (uint64_t)f * 2, rows_cap, (uint64_t)f * 2, 128, kBM, true) ||
        !jt::make_tmap_2d_u8(&p.tmS, ds, (uint64_t)d * 2, (uint64_t)E * G, (uint64_t)d * 2, 256, 1, false) ||
        !jt::make_tmap_2d_u8(&p.tmM, row_meta, 16, rows_cap, 16, 16, kBM, false))
        return -2;
    int stages = (int)((kSmemLimit - kFixed) / kStage);
    if (stages > kMaxStages) stages = kMaxStages;
    const size_t smem = kFixed + (size_t)stages * kStage;
    p.wd = wd;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.d = d;
    p.f = f;
    p.G = G;
    p.stages = stages;
    p.y = y;
    p.y_accumulate = y_accumulate;
    p.err = jtk_error_word();
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_moe_dn16, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit) !=
            cudaSuccess)
            return -3;
        attr = true;
    }
    int grid = jtk_num_sms();
    if (max_tiles_hint > 0 && grid > max_tiles_hint) grid = max_tiles_hint;
    k_moe_dn16<<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
