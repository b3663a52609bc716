// jt_moe_gemm.cu - expert GEMMs of the quantized MoE layer on the sm_100a
// tensor cores (tcgen05.mma kind::i8, TMEM accumulators, TMA operand feed).
//
// One kernel template, three modes (the routed gate/up runs on fp16
// operands in jt_moe_gu16.cu):
//   GU_SHARED  gate/up of a shared expert: int8 weights with per-channel
//              fp32 scales (w8a8.c:1021-1072 with per-token A scales).
//   DN_ROUTED  down projection of the routed experts: INT4 weights with
//              group-64 fp16 scales, activations = requantized h with one
//              scale per 64 K.  Epilogue: weighted scatter-add of every
//              (token, slot) row into the fp32 layer output (the combine of
//              moe_layer.c:1443-1463, fused).
//   DN_SHARED  down projection of a shared expert (int8, per-channel), added
//              into the layer output (moe_layer.c:1549-1559).
//
// Orientation: the MMA M side is 128 weight rows (TMEM lane = weight row, so
// per-channel and per-group weight scales are per-thread scalars); the MMA N
// side is a tile of BN token rows.  Gate/up tiles stack 64 gate rows over the
// same 64 up rows, so one MMA produces both halves of the SwiGLU input.
// Ragged experts use a device-side tile list (expert e owns token tiles
// tile_off[e]..tile_off[e+1] over rows row_off[e]..row_off[e+1]), so one
// persistent launch covers every expert whatever the routing produced.
//
// Warp roles (23 warps): w0 TMA producer (operands every 128 K, the tile's
// fp16 group scales once per tile), w1 TMEM allocator + MMA issuer and w22
// second MMA issuer, w2-5 unpack (packed INT4 bytes -> int8 codes in the
// 128-byte-swizzled K-major layout), w6-21 epilogue (four warps per TMEM
// lane quarter, one per quarter of the token columns).
//
// Group scales of the down projections (the INT4 weights' and the
// activations' per-64-K scales) force a drain of the int32 accumulator
// every 64 K.  The drain
// is kept cheap and off the tensor core's critical path:
//   * a ring of 512/BN TMEM accumulators lets the MMAs run several groups
//     ahead of the epilogue;
//   * every accumulator is pre-set to the float bit pattern 0x4B400000
//     (= 12582912.0f) and the MMAs only accumulate, so each drained word is
//     the exact float 12582912 + P (|P| <= 64*127*127 < 2^22): one packed
//     subtract recovers P as a float, and the fold runs as packed f32x2 FMAs
//     with the same IEEE results as the scalar restatement;
//   * everything the epilogue needs per tile (the tile's expert and rows, the
//     per-row metadata, the fp16 group scales, the activation group scales
//     of the down projection) is fetched by the producer warp, which runs
//     stages ahead, into a double-buffered SMEM tile slot - the epilogue
//     never waits on global memory;
//   * the drain takes two 64-K units per pass (one TMEM load wait, one store
//     wait and one slot release round per pair).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_runtime.cuh"
#include "jt_swiglu.cuh"

namespace {

constexpr int kBM = 128;           // MMA M: weight rows per tile
constexpr int kBN = JT_TILE_ROWS;  // MMA N (max): token rows per tile
constexpr int kBH = 32;            // token columns per epilogue warp
constexpr int kBK = 128;           // K per pipeline stage
constexpr int kThreads = 736;      // 23 warps
constexpr int kEpiWarp0 = 6;       // warps 6..21: epilogue
constexpr int kEpiWarps = 16;
constexpr int kMmaWarp2 = 22;      // second MMA issuer
constexpr float kMagicF = 12582912.0f;
constexpr int kMaxGroups = 64;  // K <= 4096
constexpr size_t kSmemLimit = 232448;
static_assert(kBN == (kEpiWarps / 4) * kBH, "four epilogue warps per TMEM lane quarter");

enum Mode { GU_SHARED = 1, DN_ROUTED = 2, DN_SHARED = 3 };

__host__ __device__ constexpr uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <int MODE>
struct Cfg {
    static constexpr bool kGateUp = (MODE == GU_SHARED);
    static constexpr bool kPacked = (MODE == DN_ROUTED);
    static constexpr bool kDown = !kGateUp;
    static constexpr bool kMagic = (MODE != GU_SHARED);  // 64-K drain units
    static constexpr int kChTile = kGateUp ? 64 : 128;   // output channels per tile
    static constexpr int kBits = MODE == DN_ROUTED ? 4 : 8;
    static constexpr uint32_t kPackedRow = kPacked ? (kBK * kBits / 8) : 0;  // bytes/row/stage
    static constexpr uint32_t kAU = kBM * kBK;  // unpacked operand, 16 KB
    static constexpr uint32_t kX = kBN * kBK;   // token rows, 16 KB
    static constexpr uint32_t kAP = kBM * kPackedRow;
    static constexpr uint32_t kStage = kAU + kX + kAP;
    // per-tile slot: info | row meta [kBN] float4 | group scales fp16 [G][128] |
    //                activation group scales [kBN][hs_ld] (down)
    static constexpr uint32_t kOffMeta = 128;
    static constexpr uint32_t kOffScale = kOffMeta + kBN * 16;
    static constexpr uint32_t kOffBlk = kOffScale + (kPacked ? kMaxGroups * kBM * 2 : 0);
    static constexpr uint32_t kSlot = align_up(kOffBlk + (kDown ? kBN * kMaxGroups * 4 : 0), 1024);
    static constexpr uint32_t kHTile = kGateUp ? 2 * kBN * 64 * 4 : 0;  // g then u [row][64]
    // preset operands of the magic modes: A = bf16 ones [128][16], B = bf16
    // 786432 [kBN][16]; one kind::f16 MMA of them writes 16 * 786432 =
    // 12582912.0f (bits 0x4B400000) into every accumulator element
    static constexpr uint32_t kConst = kMagic ? (kBM + kBN) * 32 : 0;
    static constexpr size_t kFixed = 1024 + 2 * (size_t)kSlot + kHTile + kConst + 1024;
    static constexpr int kStagesRaw = (int)((kSmemLimit - kFixed) / kStage);
    static constexpr int kStages = kStagesRaw > 6 ? 6 : kStagesRaw;
    static constexpr int kSlots = 512 / kBN;        // TMEM accumulators
    // drain groups: the two slots of one 128-K stage (64-K units), or one
    // slot per tile (whole-K accumulation); one full/empty barrier pair each
    static constexpr int kGroups = kMagic ? kSlots / 2 : kSlots;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr size_t kSmem = kFixed + (size_t)kStages * kStage;
    static_assert(kStages >= 2, "pipeline depth");
    static_assert(kSmem <= kSmemLimit, "shared memory");
    static_assert(kSlots == 4, "two drain groups of two slots");
};

struct MoeGemmParams {
    CUtensorMap tmA0;  // gate (or down) weights: packed bytes or int8 rows
    CUtensorMap tmA1;  // up weights (gate/up modes)
    CUtensorMap tmX;   // token rows [rows][K] int8
    CUtensorMap tmS0;  // group scales of A0, fp16 [E][K/64][n_ch] as bytes (routed)
    CUtensorMap tmS1;  // group scales of A1
    CUtensorMap tmM;   // row metadata [rows][16 B]
    CUtensorMap tmH;   // activation group scales [rows][hs_ld] fp32 (down)
    const int4 *tiles;       // token-tile table {e, row0, row_end, 0}
    const int32_t *ntiles;   // its length
    int n_ch;   // output channels per expert (f for gate/up, d for down)
    int K;      // reduction length (d for gate/up, f for down)
    int hs_ld;  // row stride of the activation group scales (down) / of hs (gate/up out)
    int hs_rows;  // shared experts: hs is [K/64 groups][hs_rows] (group-major), hs_rows % 4 == 0
    const float *cs0;  // per-channel scales [n_ch] (shared)
    const float *cs1;
    int8_t *hq;        // gate/up out: codes [rows][n_ch]
    float *hs;         // gate/up out: scales [rows][hs_ld]
    float *y;          // down out: [T][n_ch] fp32
    int y_accumulate;  // down: 0 store, 1 atomic add
    int *err;
};

// Barrier of the epilogue warps on an mbarrier (one arrival per
// warp), so that a warp which left on an abort cannot strand the others: the
// wait is bounded like every other wait in the kernel.
__device__ __forceinline__ bool epi_sync(uint64_t *bar, uint32_t &phase, volatile int *abort_flag,
                                         int *err) {
    __syncwarp();
    if (jt::lane_id() == 0) jt::mbar_arrive(bar);
    const bool ok = jt::mbar_wait(bar, phase, abort_flag, err);
    phase ^= 1u;
    return ok;
}

// ---------------------------------------------------------------- unpack
// 8 INT4 codes (one 32-bit word; even k in the low nibble) -> 8 int8 values
// c = 2*li - 15 via ((li << 1) + 113) ^ 0x80 per byte (<= 143, no carry).
__device__ __forceinline__ uint2 unpack_int4_x8(uint32_t w) {
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
    const uint32_t vl = ((lo << 1) + 0x71717171u) ^ 0x80808080u;
    const uint32_t vh = ((hi << 1) + 0x71717171u) ^ 0x80808080u;
    uint2 o;
    o.x = __byte_perm(vl, vh, 0x5140);
    o.y = __byte_perm(vl, vh, 0x7362);
    return o;
}

// One operand row: packed bytes of a 128-K stage -> 128 int8 codes written
// into the 128-byte-swizzled K-major tile (16-byte chunk i of row r lands in
// chunk i ^ (r % 8), the layout TMA's 128B swizzle produces).
__device__ __forceinline__ void unpack_row_int4(const uint8_t *src, uint8_t *dst_tile, int r) {
    uint8_t *row = dst_tile + r * 128;
#pragma unroll 1
    for (int h = 0; h < 4; ++h) {  // 16 packed bytes -> 32 codes per pass
        const uint4 a = *reinterpret_cast<const uint4 *>(src + 16 * h);
        const uint2 l0 = unpack_int4_x8(a.x), h0 = unpack_int4_x8(a.y);
        const uint2 l1 = unpack_int4_x8(a.z), h1 = unpack_int4_x8(a.w);
        *reinterpret_cast<uint4 *>(row + (((2 * h) ^ (r & 7)) << 4)) = make_uint4(l0.x, l0.y, h0.x, h0.y);
        *reinterpret_cast<uint4 *>(row + (((2 * h + 1) ^ (r & 7)) << 4)) = make_uint4(l1.x, l1.y, h1.x, h1.y);
    }
}

__device__ __forceinline__ float2 as_f2(uint32_t a, uint32_t b) {
    return make_float2(__uint_as_float(a), __uint_as_float(b));
}

__device__ __forceinline__ void st_shared_v4(void *p, int4 v) {
    asm volatile("st.shared.v4.s32 [%0], {%1, %2, %3, %4};" ::"r"(jt::smem_u32(p)), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Fold one drained 32-column chunk of one 64-K unit into the running sums
// r2[0..15] (columns 2i, 2i+1).  blk points at the activation group scales
// of the chunk's first token row (down modes).
template <int MODE>
__device__ __forceinline__ void fold_chunk(float2 *r2, const uint32_t (&a)[32], float s,
                                           const float *blk, int hs_ld, int g) {
    const float2 s2 = make_float2(s, s);
    // activation group scales of the chunk's columns (SMEM broadcast), walked
    // with one running shared-memory address
    uint32_t hv_addr = jt::smem_u32(blk + g);
    const uint32_t hv_step = static_cast<uint32_t>(hs_ld) * 4u;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        float2 &rr = r2[j / 2];
        if (MODE == GU_SHARED) {
            rr = make_float2(__int2float_rn((int32_t)a[j]), __int2float_rn((int32_t)a[j + 1]));
        } else {
            const float2 pf = __fadd2_rn(as_f2(a[j], a[j + 1]), make_float2(-kMagicF, -kMagicF));
            float2 hv;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(hv.x) : "r"(hv_addr));
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(hv.y) : "r"(hv_addr + hv_step));
            hv_addr += 2u * hv_step;
            const float2 t = (MODE == DN_ROUTED) ? __fmul2_rn(pf, s2) : pf;
            rr = __ffma2_rn(t, hv, rr);
        }
    }
}

// Fold 16 drained columns (columns c0 .. c0+15 of the warp's 32) of one
// 64-K unit into r2[c0/2 .. c0/2+7]; same arithmetic as fold_chunk.
// TP != 0 (down modes): hvT points at the tile's activation group scales in
// group-major order (group stride hs_ld floats), offset to the warp's first
// column, and is read four columns per shared-memory load.
//
// Down projection of the routed experts: the scaled partial (float)P * s is
// formed in one fused operation from the drained word A = 12582912 + P as
// fmaf(A, s, -12582912 * s).  The product 12582912 * s is exact (3 * 2^22
// times an fp16 value: at most 13 significant bits), and A*s - 12582912*s is
// exactly P*s, so the single rounding gives the same bits as the subtraction
// followed by the rounded product.
template <int MODE, int TP>
__device__ __forceinline__ void fold16(float2 *r2, const uint32_t (&a)[16], float s, const float *blk, int hs_ld,
                                       int g, int c0, const float *hvT) {
    const float2 s2 = make_float2(s, s);
    const float nms = __fmul_rn(-kMagicF, s);
    const float2 nms2 = make_float2(nms, nms);
    if constexpr (TP != 0) {
        const float4 *h4p = reinterpret_cast<const float4 *>(hvT + (size_t)g * hs_ld + c0);
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            const float4 h4 = h4p[j / 4];
            float2 ta, tb;
            if (MODE == DN_ROUTED) {
                ta = __ffma2_rn(as_f2(a[j], a[j + 1]), s2, nms2);
                tb = __ffma2_rn(as_f2(a[j + 2], a[j + 3]), s2, nms2);
            } else {
                ta = __fadd2_rn(as_f2(a[j], a[j + 1]), make_float2(-kMagicF, -kMagicF));
                tb = __fadd2_rn(as_f2(a[j + 2], a[j + 3]), make_float2(-kMagicF, -kMagicF));
            }
            r2[(c0 + j) / 2] = __ffma2_rn(ta, make_float2(h4.x, h4.y), r2[(c0 + j) / 2]);
            r2[(c0 + j) / 2 + 1] = __ffma2_rn(tb, make_float2(h4.z, h4.w), r2[(c0 + j) / 2 + 1]);
        }
        return;
    }
    const uint32_t hv_step = static_cast<uint32_t>(hs_ld) * 4u;
    uint32_t hv_addr = jt::smem_u32(blk + g) + static_cast<uint32_t>(c0) * hv_step;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
        float2 &rr = r2[(c0 + j) / 2];
        float2 hv;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(hv.x) : "r"(hv_addr));
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(hv.y) : "r"(hv_addr + hv_step));
        hv_addr += 2u * hv_step;
        const float2 t = (MODE == DN_ROUTED) ? __ffma2_rn(as_f2(a[j], a[j + 1]), s2, nms2)
                                             : __fadd2_rn(as_f2(a[j], a[j + 1]), make_float2(-kMagicF, -kMagicF));
        rr = __ffma2_rn(t, hv, rr);
    }
}

// MMA N for a tile of `rows` token rows: rows rounded up to 16 (the kind::i8
// N granularity at M = 128), at most kBN.
__device__ __forceinline__ int mma_n(int rows) {
    int n = (rows + 15) & ~15;
    n = n < 16 ? 16 : n;
    return n > kBN ? kBN : n;
}

// TP (down modes): fold with the activation group scales transposed in the
// tile slot (needs hs_ld + K/64 <= kMaxGroups).
template <int MODE, int TP = 0>
__global__ void __launch_bounds__(kThreads, 1) k_moe_gemm(const __grid_constant__ MoeGemmParams p) {
    using C = Cfg<MODE>;
    constexpr int S = C::kStages;
    constexpr int NG = C::kGroups;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *slot_base = smem + S * C::kStage;  // 2 tile slots
    float *h_tile = reinterpret_cast<float *>(slot_base + 2 * C::kSlot);
    uint8_t *cst = reinterpret_cast<uint8_t *>(h_tile) + C::kHTile;  // preset operands
    uint8_t *tail = cst + C::kConst;
    uint64_t *full = reinterpret_cast<uint64_t *>(tail);  // TMA landed
    uint64_t *ready = full + S;      // operands unpacked (packed modes)
    uint64_t *empty = ready + S;     // MMAs finished reading the stage
    uint64_t *tfull = empty + S;     // drain group filled
    uint64_t *tempty = tfull + NG;   // drain group drained
    uint64_t *pfull = tempty + NG;   // tile slot filled (producer)
    uint64_t *pempty = pfull + 2;    // tile slot released (epilogue)
    uint64_t *drain = pempty + 2;    // [2]: one per MMA issuer
    uint64_t *epib = drain + 2;      // epilogue-warp barrier
    uint64_t *cqb = epib + 1;        // [4]: the four warps sharing a column quarter
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(cqb + 4);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    static_assert((3 * S + 2 * NG + 11) * 8 + 8 <= 1024, "barrier area");

    const int warp = jt::warp_id(), lane = jt::lane_id();
    const int nch_tiles = p.n_ch / C::kChTile;
    const int nk = p.K / kBK;
    const int ngroups = p.K / 64;
    const int total = __ldg(p.ntiles) * nch_tiles;
    int *err = p.err;
    // stage layout: [A unpacked 128 x 128 | X kBN x 128 | A packed 128 x kPackedRow]
    auto stage_ptr = [&](int s) { return smem + s * C::kStage; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            jt::mbar_init(&full[s], 1);
            jt::mbar_init(&ready[s], 4);
            jt::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < NG; ++b) {
            jt::mbar_init(&tfull[b], 1);
            jt::mbar_init(&tempty[b], kEpiWarps);  // one arrival per epilogue warp
        }
        for (int b = 0; b < 2; ++b) {
            jt::mbar_init(&pfull[b], 1);
            jt::mbar_init(&pempty[b], kEpiWarps);
            jt::mbar_init(&drain[b], 1);
        }
        jt::mbar_init(epib, kEpiWarps);
        for (int b = 0; b < 4; ++b) jt::mbar_init(&cqb[b], 4);
        *abort_flag = 0;
        jt::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        jt::prefetch_tmap(&p.tmA0);
        if (C::kGateUp) jt::prefetch_tmap(&p.tmA1);
        jt::prefetch_tmap(&p.tmX);
        jt::prefetch_tmap(&p.tmM);
        if (C::kPacked) jt::prefetch_tmap(&p.tmS0);
        if (C::kDown) jt::prefetch_tmap(&p.tmH);
    }
    if (warp == 1) {
        jt::tmem_alloc(tmem_slot, C::kTmemCols);
        jt::tmem_relinquish();
    }
    if (C::kMagic) {
        // Every element of each preset matrix is equal, so their layout inside
        // the region does not matter.
        uint32_t *cw = reinterpret_cast<uint32_t *>(cst);
        for (int i = threadIdx.x; i < (int)(C::kConst / 4); i += kThreads)
            cw[i] = i < kBM * 8 ? 0x3F803F80u : 0x49404940u;  // bf16 1.0 | bf16 786432
        jt::fence_proxy_async();
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
            constexpr uint32_t kTx = C::kX + (C::kPacked ? C::kAP : C::kAU);
            const uint32_t scale_box = ngroups * 128 * 2;
            const uint32_t slot_tx = kBN * 16 + (C::kPacked ? scale_box : 0) +
                                     (MODE == DN_ROUTED ? kBN * p.hs_ld * 4 : 0) +
                                     (MODE == DN_SHARED ? 2 * 256 * ngroups : 0);
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const int4 te = __ldg(&p.tiles[u / nch_tiles]);  // {e, row0, row_end, 0}
                const int c0 = (u % nch_tiles) * C::kChTile;
                const int wrow = te.x * p.n_ch + c0;  // first weight row of the tile
                // ---- per-tile slot: info, row meta, group scales, activation scales
                if (!jt::mbar_wait(&pempty[ts], tphase ^ 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                uint8_t *sl = slot_base + ts * C::kSlot;
                st_shared_v4(sl, make_int4(te.x, te.y, te.z, c0));
                jt::mbar_arrive_expect_tx(&pfull[ts], slot_tx);
                jt::tma_load_2d(sl + C::kOffMeta, &p.tmM, &pfull[ts], 0, te.y);
                if (C::kPacked) jt::tma_load_2d(sl + C::kOffScale, &p.tmS0, &pfull[ts], c0 * 2, te.x * ngroups);
                if (MODE == DN_ROUTED) jt::tma_load_2d(sl + C::kOffBlk, &p.tmH, &pfull[ts], 0, te.y);
                if (MODE == DN_SHARED) {  // group-major scales: two [groups][64 rows] boxes
                    jt::tma_load_2d(sl + C::kOffBlk, &p.tmH, &pfull[ts], te.y * 4, 0);
                    jt::tma_load_2d(sl + C::kOffBlk + 256 * ngroups, &p.tmH, &pfull[ts], te.y * 4 + 256, 0);
                }
                t_issued |= 1u << ts;
                t_phase = (t_phase & ~(1u << ts)) | (tphase << ts);
                if (++ts == 2) {
                    ts = 0;
                    tphase ^= 1u;
                }
                // ---- operand stages
                for (int kb = 0; kb < nk; ++kb) {
                    if (!jt::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = stage_ptr(stage);
                    uint8_t *xs = st + C::kAU, *ap = xs + C::kX;
                    jt::mbar_arrive_expect_tx(&full[stage], kTx);
                    if (C::kPacked) {
                        jt::tma_load_2d(ap, &p.tmA0, &full[stage], kb * C::kPackedRow, wrow);
                    } else {
                        if (C::kGateUp) {
                            jt::tma_load_2d(st, &p.tmA0, &full[stage], kb * kBK, wrow);
                            jt::tma_load_2d(st + 64 * kBK, &p.tmA1, &full[stage], kb * kBK, wrow);
                        } else {
                            jt::tma_load_2d(st, &p.tmA0, &full[stage], kb * kBK, wrow);
                        }
                    }
                    jt::tma_load_2d(xs, &p.tmX, &full[stage], kb * kBK, te.y);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {  // every issued TMA box must land before the CTA exits
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
    } else if (warp == 1 || warp == kMmaWarp2) {
        // ------------------------------------------------ MMA issuers
        // Magic modes: 128-K stages go to the two issuers alternately (issuer
        // m = stage count % 2); a stage's two 64-K units land in the slots
        // of drain group m, so each issuer waits once for its stage operands
        // and once for its drain group per two units, and the two issuers'
        // barrier latencies overlap.  Whole-K mode: issuer 0 alone, one slot
        // (drain group) per tile.
        const int m = warp == 1 ? 0 : 1;
        if (lane == 0 && (C::kMagic || m == 0)) {
            uint32_t stage = 0, phase = 0;
            uint32_t sc = 0;  // stages seen (magic) / tiles seen (whole K)
            bool ok = true;
            const uint64_t d_ones = jt::umma_desc_noswz(jt::smem_u32(cst), 128, 256);
            const uint64_t d_magic = jt::umma_desc_noswz(jt::smem_u32(cst + kBM * 32), 128, 256);
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const int4 te = __ldg(&p.tiles[u / nch_tiles]);
                const int nrun = mma_n(te.z - te.y);
                const uint32_t idesc = jt::idesc_i8(kBM, nrun);
                const uint32_t idesc_pre = jt::idesc_bf16(kBM, nrun);
                for (int kb = 0; kb < nk && ok; ++kb) {
                    const bool mine = !C::kMagic || (sc & 1u) == (uint32_t)m;
                    if (mine) {
                        uint64_t *gate = C::kPacked ? &ready[stage] : &full[stage];
                        if (!jt::mbar_wait(gate, phase, abort_flag, err)) {
                            ok = false;
                            break;
                        }
                        jt::tc_fence_after();
                        const uint32_t base = jt::smem_u32(stage_ptr(stage));
                        const uint64_t dA = jt::umma_desc_sw128(base);
                        const uint64_t dX = jt::umma_desc_sw128(base + C::kAU);
                        if (C::kMagic) {
                            const uint32_t g = sc & 1u;
                            if (!jt::mbar_wait(&tempty[g], (sc >> 1) & 1u, abort_flag, err)) {
                                ok = false;
                                break;
                            }
                            jt::tc_fence_after();
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint32_t acc = tmem_base + (2u * g + h) * kBN;
                                // preset to 0x4B400000, then accumulate the int8 products
                                jt::mma_bf16(acc, d_ones, d_magic, idesc_pre, 0u);
                                jt::mma_i8(acc, dA + 4u * h, dX + 4u * h, idesc, 1u);
                                jt::mma_i8(acc, dA + 4u * h + 2u, dX + 4u * h + 2u, idesc, 1u);
                            }
                            jt::mma_commit(&tfull[g]);
                        } else {
                            const uint32_t g = sc % NG;
                            if (kb == 0) {
                                if (!jt::mbar_wait(&tempty[g], (sc / NG) & 1u, abort_flag, err)) {
                                    ok = false;
                                    break;
                                }
                                jt::tc_fence_after();
                            }
#pragma unroll
                            for (int ks = 0; ks < kBK / 32; ++ks)
                                jt::mma_i8(tmem_base + g * kBN, dA + 2u * ks, dX + 2u * ks, idesc,
                                           (kb | ks) != 0 ? 1u : 0u);
                            if (kb == nk - 1) jt::mma_commit(&tfull[g]);
                        }
                        jt::mma_commit(&empty[stage]);
                    }
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (C::kMagic) ++sc;
                }
                if (!C::kMagic) ++sc;
            }
            if (!ok) {  // already-issued MMAs retire before TMEM is released
                jt::mma_commit(&drain[m]);
                const long long t0 = clock64();
                while (!jt::mbar_try_wait(&drain[m], 0) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
                }
            }
        }
    } else if (warp < kEpiWarp0) {
        // ------------------------------------------------ unpack warps
        if constexpr (C::kPacked) {
            const int r = threadIdx.x - 64;  // operand row 0..127
            uint32_t stage = 0, phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                for (int kb = 0; kb < nk; ++kb) {
                    if (!jt::mbar_wait(&full[stage], phase, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = stage_ptr(stage);
                    unpack_row_int4(st + C::kAU + C::kX + r * C::kPackedRow, st, r);
                    jt::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) jt::mbar_arrive(&ready[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------ epilogue warps
        // Four warps per TMEM lane quarter: warp w reads lanes 32*(w%4)..+31
        // and owns token columns 32*((w-6)/4)..+31 of every accumulator.
        const int q = warp & 3;                         // TMEM lane quarter
        const int cq = (warp - kEpiWarp0) >> 2;         // column quarter
        const int lr = q * 32 + lane;                   // operand row = TMEM lane
        const int ew = warp - kEpiWarp0;                // 0..15
        // gate/up: rows 0..63 gate of channel lr, rows 64..127 up of channel lr-64
        const bool is_up = C::kGateUp && lr >= 64;
        const int lch = C::kGateUp ? (lr & 63) : lr;
        const int j0 = cq * kBH;  // first token column owned
        const uint32_t tlane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + j0;
        // every accumulator slot starts free (the MMA issuers preset it)
        __syncwarp();
        if (lane == 0)
            for (int b = 0; b < NG; ++b) jt::mbar_arrive(&tempty[b]);
        uint32_t sc = 0, ts = 0, tphase = 0, ephase = 0, cqphase = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
            if (!jt::mbar_wait(&pfull[ts], tphase, abort_flag, err)) {
                ok = false;
                break;
            }
            const uint8_t *sl = slot_base + ts * C::kSlot;
            const int4 info = *reinterpret_cast<const int4 *>(sl);  // {e, row0, row_end, c0}
            const float4 *meta = reinterpret_cast<const float4 *>(sl + C::kOffMeta);
            const __half *sc_ptr = reinterpret_cast<const __half *>(sl + C::kOffScale) + lr;
            const float *blk = reinterpret_cast<const float *>(sl + C::kOffBlk) + j0 * p.hs_ld;
            // down modes: the four warps of this column quarter transpose the
            // tile's activation group scales of their 32 columns to
            // [group][kBN] (behind the row-major copy in the same slot), so
            // the fold reads four columns per load
            const float *hvT = nullptr;
            if constexpr (MODE == DN_SHARED && TP != 0)  // the two boxes of 64 rows
                hvT = reinterpret_cast<const float *>(sl + C::kOffBlk) + (j0 / 64) * ngroups * 64 + (j0 % 64);
            if constexpr (MODE == DN_ROUTED && TP != 0) {
                float *blkT = reinterpret_cast<float *>(const_cast<uint8_t *>(sl) + C::kOffBlk) + kBN * p.hs_ld;
                const float *blkR = reinterpret_cast<const float *>(sl + C::kOffBlk);
                for (int g = q; g < ngroups; g += 4) blkT[g * kBN + j0 + lane] = blkR[(j0 + lane) * p.hs_ld + g];
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&cqb[cq]);
                if (!jt::mbar_wait(&cqb[cq], cqphase, abort_flag, err)) {
                    ok = false;
                    break;
                }
                cqphase ^= 1u;
                hvT = blkT + j0;
            }
            const int sc_stride = C::kGateUp ? 64 : 128;
            // group stride of the activation scales the fold reads
            const int hv_ld = TP == 0 ? p.hs_ld : (MODE == DN_SHARED ? 64 : kBN);
            const int ch = info.w + lch;  // output channel within the expert
            const int nrow = min(info.z - info.y, kBN);
            // columns of this warp that hold token rows of the tile
            const bool active = j0 < nrow;
            float2 r2[kBH / 2];
#pragma unroll
            for (int j = 0; j < kBH / 2; ++j) r2[j] = make_float2(0.0f, 0.0f);
            // one drain group per 128-K stage (two 64-K units) or per tile
            const int npass = C::kMagic ? nk : 1;
            for (int ps = 0; ps < npass; ++ps, ++sc) {
                const uint32_t g = C::kMagic ? (sc & 1u) : (sc % NG);
                const uint32_t gph = C::kMagic ? ((sc >> 1) & 1u) : ((sc / NG) & 1u);
                if (!jt::mbar_wait(&tfull[g], gph, abort_flag, err)) {
                    ok = false;
                    break;
                }
                jt::tc_fence_after();
                if (active) {
                    if constexpr (C::kMagic) {
                        // four 16-column chunks (two units x two halves); the
                        // load of chunk i+1 is in flight while chunk i folds
                        const uint32_t t0 = tlane + 2u * g * kBN;
                        const float s0 = C::kPacked ? __half2float(sc_ptr[(2 * ps) * sc_stride]) : 1.0f;
                        const float s1 = C::kPacked ? __half2float(sc_ptr[(2 * ps + 1) * sc_stride]) : 1.0f;
                        uint32_t a0[16], a1[16];
                        jt::tmem_ld16(t0, a0);
                        jt::tmem_wait_ld16(a0);
                        jt::tmem_ld16(t0 + 16, a1);
                        fold16<MODE, TP>(r2, a0, s0, blk, hv_ld, 2 * ps, 0, hvT);
                        jt::tmem_wait_ld16(a1);
                        jt::tmem_ld16(t0 + kBN, a0);
                        fold16<MODE, TP>(r2, a1, s0, blk, hv_ld, 2 * ps, 16, hvT);
                        jt::tmem_wait_ld16(a0);
                        jt::tmem_ld16(t0 + kBN + 16, a1);
                        fold16<MODE, TP>(r2, a0, s1, blk, hv_ld, 2 * ps + 1, 0, hvT);
                        jt::tmem_wait_ld16(a1);
                        fold16<MODE, TP>(r2, a1, s1, blk, hv_ld, 2 * ps + 1, 16, hvT);
                    } else {
                        uint32_t a[32];
                        jt::tmem_ld32(tlane + g * kBN, a);
                        jt::tmem_wait_ld();
                        fold_chunk<MODE>(r2, a, 1.0f, blk, p.hs_ld, 0);
                    }
                }
                jt::tc_fence_before();
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&tempty[g]);
            }
            if (!ok) break;
            if constexpr (C::kGateUp) {
                const float cscale = __ldg(is_up ? &p.cs1[ch] : &p.cs0[ch]);
                // pass 1: stage g and u (activation- and channel-scaled) in SMEM
                float *dst_tile = h_tile + (is_up ? kBN * 64 : 0);
                if (active) {
#pragma unroll
                    for (int j = 0; j < kBH; ++j) {
                        const float xs = meta[j0 + j].x;
                        const float rv = (j & 1) ? r2[j / 2].y : r2[j / 2].x;
                        dst_tile[(j0 + j) * 64 + lch] = __fmul_rn(__fmul_rn(rv, xs), cscale);
                    }
                }
                if (!epi_sync(epib, ephase, abort_flag, err)) {
                    ok = false;
                    break;
                }
                // pass 2: four token rows per warp step, eight lanes per
                // row: lane l forms h = SwiGLU(g, u) (moe_layer.c:146-148) of
                // channels 8(l%8) .. 8(l%8)+7 of its row, the row's 64
                // channels are requantized together (w8a8.c:688-747) and
                // stored as 64 contiguous codes.
                {
                    const int sl = lane & 7, gq = lane >> 3;
                    for (int jb = 4 * ew; jb < nrow; jb += 4 * kEpiWarps) {
                        const int j = jb + gq;
                        const bool live = j < nrow;
                        float h[8];
                        if (live) {
                            const float4 *gp = reinterpret_cast<const float4 *>(h_tile + j * 64 + 8 * sl);
                            const float4 *up =
                                reinterpret_cast<const float4 *>(h_tile + kBN * 64 + j * 64 + 8 * sl);
                            const float4 g0 = gp[0], g1 = gp[1], u0 = up[0], u1 = up[1];
                            const float2 ha = jt::swiglu2(make_float2(g0.x, g0.y), make_float2(u0.x, u0.y));
                            const float2 hb = jt::swiglu2(make_float2(g0.z, g0.w), make_float2(u0.z, u0.w));
                            const float2 hc = jt::swiglu2(make_float2(g1.x, g1.y), make_float2(u1.x, u1.y));
                            const float2 hd = jt::swiglu2(make_float2(g1.z, g1.w), make_float2(u1.z, u1.w));
                            h[0] = ha.x, h[1] = ha.y, h[2] = hb.x, h[3] = hb.y;
                            h[4] = hc.x, h[5] = hc.y, h[6] = hd.x, h[7] = hd.y;
                        } else {
#pragma unroll
                            for (int i = 0; i < 8; ++i) h[i] = 0.0f;
                        }
                        bool bad = false;
                        float m = 0.0f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            bad |= !isfinite(h[i]);
                            m = fmaxf(m, fabsf(h[i]));
                        }
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                        if (__any_sync(0xffffffffu, bad) && lane == 0) atomicExch(err, JT_KERR_NONFINITE);
                        if (live) {
                            const jt::QuantBlockF qb = jt::quant_block_f(m);
                            uint32_t wd[2] = {0u, 0u};
#pragma unroll
                            for (int i = 0; i < 8; ++i)
                                wd[i >> 2] |= (uint32_t)(uint8_t)(int8_t)jt::quant_code_f(h[i], qb) << (8 * (i & 3));
                            const int row = info.y + j;
                            *reinterpret_cast<uint2 *>(p.hq + (size_t)row * p.n_ch + info.w + 8 * sl) =
                                make_uint2(wd[0], wd[1]);
                            if (sl == 0) p.hs[(size_t)(info.w / 64) * p.hs_rows + row] = qb.scale_f;
                        }
                    }
                }
                // all slot reads (meta) and h_tile reads done before release
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&pempty[ts]);
                if (!epi_sync(epib, ephase, abort_flag, err)) {  // h_tile free for the next tile
                    ok = false;
                    break;
                }
            } else {
                float cs = 1.0f;
                if (MODE == DN_SHARED) cs = __ldg(&p.cs0[ch]);
                if (active) {
#pragma unroll
                    for (int j = 0; j < kBH; ++j) {
                        const int row = info.y + j0 + j;
                        if (row >= info.z) continue;
                        const float4 mt = meta[j0 + j];
                        const float rv = (j & 1) ? r2[j / 2].y : r2[j / 2].x;
                        const float v = (MODE == DN_ROUTED) ? __fmul_rn(mt.y, rv) : __fmul_rn(rv, cs);
                        float *dst = p.y + (size_t)__float_as_int(mt.z) * p.n_ch + ch;
                        if (p.y_accumulate) atomicAdd(dst, v);
                        else *dst = v;
                    }
                }
                // generic-proxy writes (the transposed scales) precede the
                // producer's next TMA write of this slot
                jt::fence_proxy_async();
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&pempty[ts]);
            }
            if (++ts == 2) {
                ts = 0;
                tphase ^= 1u;
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        jt::tc_fence_after();
        jt::tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int MODE, int TP>
int launch_tp(MoeGemmParams &p, int max_tiles_hint, cudaStream_t stream) {
    using C = Cfg<MODE>;
    auto kern = k_moe_gemm<MODE, TP>;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)C::kSmem) != cudaSuccess)
            return -3;
        attr = true;
    }
    int grid = jtk_num_sms();
    if (max_tiles_hint > 0 && grid > max_tiles_hint) grid = max_tiles_hint;
    p.err = jtk_error_word();
    kern<<<grid, kThreads, C::kSmem, stream>>>(p);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int MODE>
int launch(MoeGemmParams &p, int max_tiles_hint, cudaStream_t stream) {
    if constexpr (MODE == DN_ROUTED)
        if (p.hs_ld + p.K / 64 <= kMaxGroups) return launch_tp<MODE, 1>(p, max_tiles_hint, stream);
    if constexpr (MODE == DN_SHARED) return launch_tp<MODE, 1>(p, max_tiles_hint, stream);
    return launch_tp<MODE, 0>(p, max_tiles_hint, stream);
}

int hs_stride(int n_ch) { return ((n_ch / 64) + 3) & ~3; }

bool meta_map(CUtensorMap *m, const float4 *row_meta, int rows) {
    return jt::make_tmap_2d_u8(m, row_meta, 16, rows, 16, 16, kBN, false);
}

}  // namespace

// Shared gate/up (one shared expert): wsg, wsu int8 [fs][d] with per-channel
// ssg, ssu; x int8 [T][d], sh_meta [T]; writes hq [T][fs] and hs group-major
// [fs/64][round_up(T, 4)].
extern "C" int jtk_moe_gateup_shared(const int8_t *wsg, const int8_t *wsu, const float *ssg,
                                     const float *ssu, int fs, int d, const int8_t *xq, int T,
                                     const float4 *sh_meta, const int4 *tiles,
                                     const int32_t *ntiles, int8_t *hq, float *hs,
                                     cudaStream_t stream) {
    if (fs % 64 || d % kBK || T <= 0) return -1;
    // 256-token CTA-pair tiles when the shape allows (jt_shared_pair.cu)
    const int rp = jtk_shared_gu_pair(wsg, wsu, ssg, ssu, fs, d, xq, sh_meta, T, hq, hs, stream);
    if (rp != -1) return rp;
    MoeGemmParams p{};
    if (!jt::make_tmap_2d_u8(&p.tmA0, wsg, d, fs, d, kBK, 64, true) ||
        !jt::make_tmap_2d_u8(&p.tmA1, wsu, d, fs, d, kBK, 64, true) ||
        !jt::make_tmap_2d_u8(&p.tmX, xq, d, T, d, kBK, kBN, true) || !meta_map(&p.tmM, sh_meta, T))
        return -2;
    p.tmS0 = p.tmA0;
    p.tmS1 = p.tmA0;
    p.tmH = p.tmM;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.n_ch = fs;
    p.K = d;
    p.hs_ld = hs_stride(fs);
    p.hs_rows = (T + 3) & ~3;
    p.cs0 = ssg;
    p.cs1 = ssu;
    p.hq = hq;
    p.hs = hs;
    return launch<GU_SHARED>(p, ((T + kBN - 1) / kBN) * (fs / 64), stream);
}

// Shared down: wsd int8 [d][fs] with per-channel ssd; hq [T][fs], hs group-major [fs/64][round_up(T, 4)];
// y[t][d] = (accumulate ? y + v : v).
extern "C" int jtk_moe_down_shared(const int8_t *wsd, const float *ssd, int d, int fs,
                                   const int8_t *hq, int T, const float *hs,
                                   const float4 *sh_meta, const int4 *tiles,
                                   const int32_t *ntiles, float *y, int accumulate,
                                   cudaStream_t stream) {
    if (d % kBM || fs % kBK || fs / 64 > kMaxGroups || T <= 0) return -1;
    MoeGemmParams p{};
    const int hs_ld = hs_stride(fs);
    if (!jt::make_tmap_2d_u8(&p.tmA0, wsd, fs, d, fs, kBK, kBM, true) ||
        !jt::make_tmap_2d_u8(&p.tmX, hq, fs, T, fs, kBK, kBN, true) || !meta_map(&p.tmM, sh_meta, T) ||
        !jt::make_tmap_2d_u8(&p.tmH, hs, (uint64_t)((T + 3) & ~3) * 4, (uint64_t)(fs / 64),
                             (uint64_t)((T + 3) & ~3) * 4, 256, fs / 64, false))
        return -2;
    p.tmA1 = p.tmA0;
    p.tmS0 = p.tmA0;
    p.tmS1 = p.tmA0;
    p.tiles = tiles;
    p.ntiles = ntiles;
    p.n_ch = d;
    p.K = fs;
    p.hs_ld = hs_ld;
    p.hs_rows = (T + 3) & ~3;
    p.cs0 = ssd;
    p.y = y;
    p.y_accumulate = accumulate;
    return launch<DN_SHARED>(p, ((T + kBN - 1) / kBN) * (d / kBM), stream);
}
