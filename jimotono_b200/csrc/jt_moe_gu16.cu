// jt_moe_gu16.cu - gate/up projection of the routed experts on the sm_100a
// tensor cores with fp16 operands (tcgen05.mma kind::f16, fp32 TMEM
// accumulators, TMA operand feed), fused with SwiGLU; h leaves as bf16.
//
// Arithmetic, for kept row r (token t) of expert e and gate channel c:
//   w16[c][k] = fp16_rn(code(c, k) * s[k/64][c])   code in {-3, -1, 1, 3}
//   g[r][c]   = fl32(fl32(sum_k x[t][k] * w16[c][k]) * xs[t])
// and u likewise with the up weights: the group-64 fp16 scale is folded into
// the weight before the MMA (the product of a code and an fp16 scale is
// rounded once to fp16; +-1 times the scale is exact), x are the token's
// int8 codes (exact in fp16), and the K sum runs in fp32 inside the tensor
// core in an order the hardware chooses.  Then h = bf16_rn(SwiGLU(g, u))
// (moe_layer.c:146-148, jt_swiglu.cuh), the routed down projection's input
// (jt_moe_dn16.cu).
//
// Tile: 128 token rows of one expert (MMA M, TMEM lane = token row; an
// entry of the 128-row tile table jtk_split_tiles derives) x 128
// channels (MMA N = 256: the 128 gate rows, then the same 128 up rows), so
// a thread of the epilogue holds the gate and up sums of its token for
// the same channels and forms SwiGLU in registers.  One pipeline stage is one 64-K scale group: the token rows as
// fp16 (16 KB, 128-byte swizzle), the packed INT2 codes of the 256 weight
// rows (4 KB) and their fp16 group scales (512 B) arrive by TMA (seven
// stages in flight); eight unpack warps turn the codes into fp16 weights in
// the 128-byte-swizzled K-major layout the MMA reads, in a separate ring of
// two 32 KB buffers.  The whole K accumulates in one TMEM accumulator of
// 256 columns; two of them let the MMA run a tile ahead of the epilogue,
// which drains each tile once.
//
// Unpack: a row's four possible weight values of a group, {-t, -s, s, t}
// with t = fp16_rn(3 s), sit in two registers as a byte table; every code
// selects its two bytes with one byte permute (selector 0x22 * code + 0x10
// per code, formed for four codes at once by one multiply-add on the
// masked codes).  The values of a 16-code word come out in the order
// jt::kX16Order, which the token rows (jtk_quant_dispatch, jtk_ep_gather)
// are stored in, so the K sums pair the right elements.
//
// Warp roles (18 warps): w0 TMA producer (operand stages; per tile the row
// metadata into a double-buffered slot; the next tile's weight rows are
// prefetched into L2), w1 TMEM allocator + MMA issuer, w2-9 unpack (one
// weight row per thread), w10-17 epilogue (two warps per TMEM lane quarter,
// 64 channels each).  Every wait is a bounded mbarrier wait.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_runtime.cuh"
#include "jt_swiglu.cuh"

namespace {

constexpr int kBM = JT_SUB_ROWS;          // token rows per tile (MMA M)
constexpr int kCh = 128;                  // channels per tile
constexpr int kBN = 2 * kCh;              // MMA N: gate rows, then up rows
constexpr int kThreads = 576;             // 18 warps
constexpr int kUnpack0 = 2;               // warps 2-9
constexpr int kUnpackWarps = 8;
constexpr int kEpi0 = 10;                 // warps 10-17
constexpr int kEpiWarps = 8;
constexpr int kMaxStages = 8;
constexpr int kBBufs = 2;                 // unpacked weight buffers
constexpr int kMaxGroups = 64;            // d <= 4096
constexpr uint32_t kX16 = kBM * 128;      // fp16 token rows of one 64-K group, 16 KB
constexpr uint32_t kPk = kBN * 16;        // packed codes, 4 KB
constexpr uint32_t kSc = kBN * 2;         // group scales, 512 B
constexpr uint32_t kStage = 21504;        // X16 | packed | scales, 1024-aligned
constexpr uint32_t kB16 = kBN * 128;      // fp16 weights of one 64-K group, 32 KB
constexpr uint32_t kSlot = 3072;          // info | row meta [kBM] float4
constexpr uint32_t kOffMeta = 128;
constexpr uint32_t kBarBytes = 1024;
constexpr size_t kSmemLimit = 232448;
constexpr size_t kFixed = 1024 + kBBufs * (size_t)kB16 + 2 * (size_t)kSlot + kBarBytes;
static_assert(kStage >= kX16 + kPk + kSc && kStage % 1024 == 0, "stage layout");
static_assert(kOffMeta + kBM * 16 <= kSlot, "slot layout");

struct Gu16Params {
    CUtensorMap tmA0, tmA1;  // packed INT2 gate / up rows [E*f][d/4], 16 B x 128 boxes
    CUtensorMap tmX;         // fp16 token rows [rows][2d bytes], 128 B x 128 boxes, swizzled
    CUtensorMap tmS0, tmS1;  // fp16 group scales [E*G][f] as bytes, 256 B x 1 boxes
    CUtensorMap tmM;         // row metadata [rows][16 B]
    const uint8_t *wg, *wu;  // the packed rows again, for the L2 prefetch of the next tile
    const int4 *tiles;       // {e, row0, row_end, 0}
    const int32_t *ntiles;
    int f, d, G, stages;
    uint16_t *h;             // [rows][f] bf16
    int *err;
};

__device__ __forceinline__ void st_shared_v4u(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Instruction descriptor, kind::f16 with fp16 A and B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One 16-code word of a row -> 16 fp16 weights (kX16Order) stored as two
// 16-byte chunks of the row's swizzled 128-byte line.  lo / hi: the byte
// table {v0, v1} / {v2, v3} of the group's values for codes 0..3.
__device__ __forceinline__ void unpack_word(uint32_t w, uint32_t lo, uint32_t hi, uint32_t row_addr, uint32_t r7,
                                            uint32_t chunk) {
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t sel = ((w >> (2 * k)) & 0x03030303u) * 0x22u + 0x10101010u;
        o[2 * k] = __byte_perm(lo, hi, sel);
        o[2 * k + 1] = __byte_perm(lo, hi, sel >> 16);
    }
    st_shared_v4u(row_addr + (((chunk ^ r7) & 7u) << 4), o[0], o[1], o[2], o[3]);
    st_shared_v4u(row_addr + ((((chunk + 1u) ^ r7) & 7u) << 4), o[4], o[5], o[6], o[7]);
}

// One weight row of a stage: 64 codes (16 packed bytes) with the group's
// fp16 scale sb -> 64 fp16 weights in row r of the swizzled buffer.
__device__ __forceinline__ void unpack_row(const uint8_t *pk_row, uint32_t sb, uint32_t buf_addr, int r) {
    const uint32_t tb = __half_as_ushort(
        __float2half_rn(3.0f * __half2float(__ushort_as_half(static_cast<unsigned short>(sb)))));
    const uint32_t lo = (tb ^ 0x8000u) | ((sb ^ 0x8000u) << 16);  // -t, -s
    const uint32_t hi = sb | (tb << 16);                          // s, t
    const uint4 pk = *reinterpret_cast<const uint4 *>(pk_row);
    const uint32_t row_addr = buf_addr + static_cast<uint32_t>(r) * 128u, r7 = static_cast<uint32_t>(r & 7);
    unpack_word(pk.x, lo, hi, row_addr, r7, 0);
    unpack_word(pk.y, lo, hi, row_addr, r7, 2);
    unpack_word(pk.z, lo, hi, row_addr, r7, 4);
    unpack_word(pk.w, lo, hi, row_addr, r7, 6);
}

__global__ void __launch_bounds__(kThreads, 1) k_moe_gu16(const __grid_constant__ Gu16Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int S = p.stages, G = p.G;
    uint8_t *bbuf = smem + (size_t)S * kStage;          // unpacked weight buffers
    uint8_t *slot_base = bbuf + kBBufs * kB16;
    uint64_t *full = reinterpret_cast<uint64_t *>(slot_base + 2 * kSlot);
    uint64_t *empty = full + kMaxStages;   // MMAs done with the stage (and so the unpack)
    uint64_t *bfull = empty + kMaxStages;  // weight buffer unpacked [kBBufs]
    uint64_t *bempty = bfull + kBBufs;     // MMAs done with the weight buffer [kBBufs]
    uint64_t *tfull = bempty + kBBufs;     // accumulator complete [2]
    uint64_t *tempty = tfull + 2;          // accumulator drained [2]
    uint64_t *pfull = tempty + 2;          // tile slot filled [2]
    uint64_t *pempty = pfull + 2;          // tile slot released [2]
    uint64_t *drain = pempty + 2;          // abort path of the MMA issuer
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = jt::warp_id(), lane = jt::lane_id();
    const int nch = p.f / kCh;
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
        jt::prefetch_tmap(&p.tmA0);
        jt::prefetch_tmap(&p.tmA1);
        jt::prefetch_tmap(&p.tmX);
        jt::prefetch_tmap(&p.tmS0);
        jt::prefetch_tmap(&p.tmS1);
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
            const uint32_t wbytes = kCh * (uint32_t)(p.d / 4);  // 128 packed rows, contiguous
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const int4 te = __ldg(&p.tiles[u / nch]);
                const int c0 = (u % nch) * kCh;
                const int wrow = te.x * p.f + c0;
                if (u == (int)blockIdx.x) {
                    jt::prefetch_l2(p.wg + (size_t)wrow * (p.d / 4), wbytes);
                    jt::prefetch_l2(p.wu + (size_t)wrow * (p.d / 4), wbytes);
                }
                // the packed weights stream from HBM: pull the next tile's rows
                // into L2 while this tile's stages run
                if (u + (int)gridDim.x < total) {
                    const int un = u + (int)gridDim.x;
                    const int wn = __ldg(&p.tiles[un / nch]).x * p.f + (un % nch) * kCh;
                    jt::prefetch_l2(p.wg + (size_t)wn * (p.d / 4), wbytes);
                    jt::prefetch_l2(p.wu + (size_t)wn * (p.d / 4), wbytes);
                }
                if (!jt::mbar_wait(&pempty[ts], tphase ^ 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                uint8_t *sl = slot_base + ts * kSlot;
                asm volatile("st.shared.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(jt::smem_u32(sl)), "r"(te.x),
                             "r"(te.y), "r"(te.z), "r"(c0)
                             : "memory");
                jt::mbar_arrive_expect_tx(&pfull[ts], kBM * 16);
                jt::tma_load_2d(sl + kOffMeta, &p.tmM, &pfull[ts], 0, te.y);
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
                    jt::mbar_arrive_expect_tx(&full[stage], kX16 + kPk + kSc);
                    jt::tma_load_2d(st, &p.tmX, &full[stage], kb * 128, te.y);
                    jt::tma_load_2d(st + kX16, &p.tmA0, &full[stage], kb * 16, wrow);
                    jt::tma_load_2d(st + kX16 + kCh * 16, &p.tmA1, &full[stage], kb * 16, wrow);
                    jt::tma_load_2d(st + kX16 + kPk, &p.tmS0, &full[stage], c0 * 2, te.x * G + kb);
                    jt::tma_load_2d(st + kX16 + kPk + kCh * 2, &p.tmS1, &full[stage], c0 * 2, te.x * G + kb);
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
            uint32_t stage = 0, phase = 0, bb = 0, bphase = 0, tc = 0;
            bool ok = true;
            constexpr uint32_t idesc = idesc_f16(kBM, kBN);
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++tc) {
                const uint32_t buf = tc & 1u;
                if (!jt::mbar_wait(&tempty[buf], (tc >> 1) & 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                jt::tc_fence_after();
                const uint32_t acc = tmem_base + buf * kBN;
                for (int kb = 0; kb < G; ++kb) {
                    if (!jt::mbar_wait(&bfull[bb], bphase, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    jt::tc_fence_after();
                    const uint64_t dX = jt::umma_desc_sw128(jt::smem_u32(smem + (size_t)stage * kStage));
                    const uint64_t dW = jt::umma_desc_sw128(jt::smem_u32(bbuf + bb * kB16));
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16(acc, dX + 2u * ks, dW + 2u * ks, idesc, (kb | ks) != 0 ? 1u : 0u);
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
                if (ok) jt::mma_commit(&tfull[buf]);
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
        const int r0 = threadIdx.x - 32 * kUnpack0;  // weight row (0-127 gate, 128-255 up)
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
                const uint16_t *sc = reinterpret_cast<const uint16_t *>(st + kX16 + kPk);
                const uint32_t ba = jt::smem_u32(bbuf + bb * kB16);
                unpack_row(st + kX16 + r0 * 16, sc[r0], ba, r0);
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
        // quarter), channels 64 ((w - 10) / 4) .. +63 of the tile
        const int q = warp & 3;
        const int ch0 = ((warp - kEpi0) >> 2) * 64;
        const int j = q * 32 + lane;  // token row within the tile
        const uint32_t tq = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        __syncwarp();
        if (lane == 0) {  // both accumulators start free
            jt::mbar_arrive(&tempty[0]);
            jt::mbar_arrive(&tempty[1]);
        }
        uint32_t tc = 0, ts = 0, tphase = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total && ok; u += gridDim.x, ++tc) {
            if (!jt::mbar_wait(&pfull[ts], tphase, abort_flag, err)) {
                ok = false;
                break;
            }
            const uint8_t *sl = slot_base + ts * kSlot;
            const int4 info = *reinterpret_cast<const int4 *>(sl);  // {e, row0, row_end, c0}
            const float xs = reinterpret_cast<const float4 *>(sl + kOffMeta)[j].x;
            const bool live = j < min(info.z - info.y, kBM);
            __syncwarp();
            if (lane == 0) jt::mbar_arrive(&pempty[ts]);
            if (++ts == 2) {
                ts = 0;
                tphase ^= 1u;
            }
            const uint32_t buf = tc & 1u;
            if (!jt::mbar_wait(&tfull[buf], (tc >> 1) & 1u, abort_flag, err)) {
                ok = false;
                break;
            }
            jt::tc_fence_after();
            const uint32_t acc = tq + buf * kBN + ch0;
            // h = SwiGLU(g xs, u xs) eight channels at a time, stored as bf16
            uint4 *dst = reinterpret_cast<uint4 *>(p.h + (size_t)(info.y + j) * p.f + info.w + ch0);
            bool bad = false;
#pragma unroll 2
            for (int c = 0; c < 64; c += 8) {
                uint32_t ga[8], ua[8];
                jt::tmem_ld8(acc + c, ga);
                jt::tmem_ld8(acc + kCh + c, ua);
                jt::tmem_wait_ld8(ga);
                jt::tmem_wait_ld8(ua);
                uint32_t hw[4];
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    const float2 g2 = make_float2(__fmul_rn(__uint_as_float(ga[i]), xs),
                                                  __fmul_rn(__uint_as_float(ga[i + 1]), xs));
                    const float2 u2 = make_float2(__fmul_rn(__uint_as_float(ua[i]), xs),
                                                  __fmul_rn(__uint_as_float(ua[i + 1]), xs));
                    const float2 hv = jt::swiglu2(g2, u2);
                    bad |= live & (!isfinite(hv.x) | !isfinite(hv.y));
                    const __nv_bfloat162 hb = __floats2bfloat162_rn(hv.x, hv.y);
                    hw[i / 2] = *reinterpret_cast<const uint32_t *>(&hb);
                }
                if (live) dst[c / 8] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            }
            jt::tc_fence_before();
            __syncwarp();
            if (lane == 0) jt::mbar_arrive(&tempty[buf]);
            if (__any_sync(0xffffffffu, bad) && lane == 0) atomicExch(err, JT_KERR_NONFINITE);
        }
    }
    __syncthreads();
    if (warp == 1) {
        jt::tc_fence_after();
        jt::tmem_dealloc(tmem_base, 2 * kBN);
    }
}

}  // namespace

// Routed gate/up: wg, wu packed INT2 [E][f][d/4]; gs, us fp16 [E][d/64][f];
// xd fp16 [rows][d] in expert order (jt::kX16Order inside every 16-element
// block); writes h [rows][f] bf16.
extern "C" int jtk_moe_gateup_routed(const uint8_t *wg, const uint8_t *wu, const void *gs,
                                     const void *us, int E, int f, int d, const uint16_t *xd,
                                     int rows_cap, const float4 *row_meta, const int4 *tiles,
                                     const int32_t *ntiles, uint16_t *h, int max_tiles_hint,
                                     cudaStream_t stream) {
    if (f % kCh || d % 64 || d / 64 > kMaxGroups || E <= 0 || rows_cap <= 0) return -1;
    const int G = d / 64;
    Gu16Params p{};
    const uint32_t prow = d / 4;
    if (!jt::make_tmap_2d_u8(&p.tmA0, wg, prow, (uint64_t)E * f, prow, 16, kCh, false) ||
        !jt::make_tmap_2d_u8(&p.tmA1, wu, prow, (uint64_t)E * f, prow, 16, kCh, false) ||
        !jt::make_tmap_2d_u8(&p.tmX, xd, (uint64_t)d * 2, rows_cap, (uint64_t)d * 2, 128, kBM, true) ||
        !jt::make_tmap_2d_u8(&p.tmS0, gs, (uint64_t)f * 2, (uint64_t)E * G, (uint64_t)f * 2, kCh * 2, 1, false) ||
        !jt::make_tmap_2d_u8(&p.tmS1, us, (uint64_t)f * 2, (uint64_t)E * G, (uint64_t)f * 2, kCh * 2, 1, false) ||
        !jt::make_tmap_2d_u8(&p.tmM, row_meta, 16, rows_cap, 16, 16, kBM, false))
        return -2;
    int stages = (int)((kSmemLimit - kFixed) / kStage);
    if (stages > kMaxStages) stages = kMaxStages;
    const size_t smem = kFixed + (size_t)stages * kStage;
    p.wg = wg;
    p.wu = wu;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.f = f;
    p.d = d;
    p.G = G;
    p.stages = stages;
    p.h = h;
    p.err = jtk_error_word();
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_moe_gu16, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit) !=
            cudaSuccess)
            return -3;
        attr = true;
    }
    int grid = jtk_num_sms();
    if (max_tiles_hint > 0 && grid > max_tiles_hint) grid = max_tiles_hint;
    k_moe_gu16<<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
