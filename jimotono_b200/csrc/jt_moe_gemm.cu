// jt_moe_gemm.cu - expert GEMMs of the quantized MoE layer on the sm_100a
// tensor cores (tcgen05.mma kind::i8, TMEM accumulators, TMA operand feed).
//
// One kernel template, four modes:
//   GU_ROUTED  gate/up of the routed experts: INT2 weights with one fp16
//              scale per 64 K (group-64 format), int8 token rows in expert
//              order.  Epilogue: fold of the group partials, SwiGLU, and
//              requantization of h per (row, 64-channel group).
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
// Orientation: the MMA M side is 128 weight channels (TMEM lane = output
// channel, so per-channel and per-group scales are per-thread scalars); the
// MMA N side is a tile of kBN token rows.  Ragged experts are handled by a
// device-side tile list (expert e owns token tiles tile_off[e]..tile_off[e+1]
// over its rows row_off[e]..row_off[e+1]), so one persistent launch covers
// every expert whatever the routing produced.
//
// Warp roles (10 warps): w0 TMA producer, w1 TMEM allocator + MMA issuer,
// w2-5 unpack (packed INT2/INT4 bytes in SMEM -> int8 codes in the
// 128-byte-swizzled K-major operand layout), w6-9 epilogue.  Group scales
// force the int32 accumulator to be drained every 64 K: two TMEM slots let
// the epilogue drain slot s while the MMAs fill slot s^1.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_runtime.cuh"
#include "jt_swiglu.cuh"

namespace {

constexpr int kBM = 128;  // MMA M: weight rows per tile
constexpr int kBN = 64;   // MMA N: token rows per tile
constexpr int kBK = 128;  // K per pipeline stage
constexpr int kThreads = 320;
constexpr int kEpiWarp0 = 6;

enum Mode { GU_ROUTED = 0, GU_SHARED = 1, DN_ROUTED = 2, DN_SHARED = 3 };

template <int MODE>
struct Cfg {
    static constexpr bool kGateUp = (MODE == GU_ROUTED || MODE == GU_SHARED);
    static constexpr bool kPacked = (MODE == GU_ROUTED || MODE == DN_ROUTED);
    // gate/up tiles stack 64 gate rows over the same 64 up rows
    static constexpr int kChTile = kGateUp ? 64 : 128;  // output channels per tile
    static constexpr int kBits = MODE == GU_ROUTED ? 2 : (MODE == DN_ROUTED ? 4 : 8);
    static constexpr uint32_t kPackedRow = kPacked ? (kBK * kBits / 8) : 0;  // bytes/row/stage
    static constexpr uint32_t kAU = kBM * kBK;  // unpacked operand, 16 KB
    static constexpr uint32_t kX = kBN * kBK;   // token rows, 8 KB
    static constexpr uint32_t kAP = kBM * kPackedRow;
    static constexpr uint32_t kStage = kAU + kX + kAP;
    static constexpr uint32_t kHTile = kBN * 64 * 4;  // gate/up: g then h [row][64 ch];
                                                      // down: hs [group][row]
    static constexpr int kStagesRaw = (int)((200 * 1024 - kHTile) / kStage);
    static constexpr int kStages = kStagesRaw > 6 ? 6 : kStagesRaw;
    // K per drain: group-64 weights and the 64-channel activation blocks
    // both drain every 64 K; the shared gate/up accumulates a whole tile.
    static constexpr int kUnitK = (MODE == GU_SHARED) ? 0 : 64;
    static constexpr uint32_t kTmemCols = 2 * kBN;
    static constexpr size_t kSmem = 1024 + (size_t)kStages * kStage + kHTile + 1024;
};

struct MoeGemmParams {
    CUtensorMap tmA0;  // gate (or down) weights: packed bytes or int8 rows
    CUtensorMap tmA1;  // up weights (gate/up modes)
    CUtensorMap tmX;   // token rows [rows][K] int8
    const int32_t *row_off;   // [E+1] token-row range per expert
    const int32_t *tile_off;  // [E+1] token-tile range per expert (tile_off[E] = total)
    int E;
    int n_ch;  // output channels per expert (f for gate/up, d for down)
    int K;     // reduction length (d for gate/up, f for down)
    const __half *gs0;  // group scales [E][n_ch][K/64] (routed)
    const __half *gs1;
    const float *cs0;  // per-channel scales [n_ch] (shared)
    const float *cs1;
    const float *row_scale;  // gate/up: per-row activation scale [rows]
    const float *blk_scale;  // down: per-(row, 64-K group) activation scale [rows][K/64]
    int8_t *hq;              // gate/up out: codes [rows][n_ch]
    float *hs;               // gate/up out: scales [rows][n_ch/64]
    float *y;                // down out: [T][n_ch] fp32
    const int32_t *row_tok;  // down: token of each row (routed)
    const float *row_w;      // down: weight of each row (routed)
    int y_accumulate;        // down: 0 store, 1 atomic add
    int *err;
};

__device__ __forceinline__ void named_bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Expert owning token tile v (tile_off ascending, tile_off[E] = total).
__device__ __forceinline__ int find_expert(const int32_t *tile_off, int E, int v) {
    int lo = 0, hi = E;  // invariant tile_off[lo] <= v < tile_off[hi]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(&tile_off[mid]) <= v) lo = mid;
        else hi = mid;
    }
    return lo;
}

struct TileInfo {
    int e, c0, r0, r_end;
};

template <int CH_TILE>
__device__ __forceinline__ TileInfo tile_info(const MoeGemmParams &p, int u, int nch_tiles) {
    TileInfo ti;
    const int c = u % nch_tiles;
    const int v = u / nch_tiles;
    ti.e = find_expert(p.tile_off, p.E, v);
    const int j = v - __ldg(&p.tile_off[ti.e]);
    ti.c0 = c * CH_TILE;
    ti.r0 = __ldg(&p.row_off[ti.e]) + j * kBN;
    ti.r_end = __ldg(&p.row_off[ti.e + 1]);
    return ti;
}

// ---------------------------------------------------------------- unpack
// 16 INT2 codes (one 32-bit packed word, little-endian along K) -> 16 int8
// values c = 2*li - 3.  Per byte: ((li << 1) + 125) ^ 0x80 = 2*li - 3 with
// no carry between bytes (2*li + 125 <= 131).
__device__ __forceinline__ uint4 unpack_int2_x16(uint32_t w) {
    uint32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t c = (w >> (2 * j)) & 0x03030303u;
        v[j] = ((c << 1) + 0x7D7D7D7Du) ^ 0x80808080u;
    }
    const uint32_t t01l = __byte_perm(v[0], v[1], 0x5140);
    const uint32_t t23l = __byte_perm(v[2], v[3], 0x5140);
    const uint32_t t01h = __byte_perm(v[0], v[1], 0x7362);
    const uint32_t t23h = __byte_perm(v[2], v[3], 0x7362);
    uint4 o;
    o.x = __byte_perm(t01l, t23l, 0x5410);
    o.y = __byte_perm(t01l, t23l, 0x7632);
    o.z = __byte_perm(t01h, t23h, 0x5410);
    o.w = __byte_perm(t01h, t23h, 0x7632);
    return o;
}

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
template <int BITS>
__device__ __forceinline__ void unpack_row(const uint8_t *src, uint8_t *dst_tile, int r) {
    uint8_t *row = dst_tile + r * 128;
    if (BITS == 2) {
        const uint4 a = *reinterpret_cast<const uint4 *>(src);
        const uint4 b = *reinterpret_cast<const uint4 *>(src + 16);
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
            *reinterpret_cast<uint4 *>(row + ((i ^ (r & 7)) << 4)) = unpack_int2_x16(w[i]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint2 a = *reinterpret_cast<const uint2 *>(src + 8 * i);
            const uint2 lo = unpack_int4_x8(a.x), hi = unpack_int4_x8(a.y);
            *reinterpret_cast<uint4 *>(row + ((i ^ (r & 7)) << 4)) =
                make_uint4(lo.x, lo.y, hi.x, hi.y);
        }
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) k_moe_gemm(const __grid_constant__ MoeGemmParams p) {
    using C = Cfg<MODE>;
    constexpr int S = C::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    float *h_tile = reinterpret_cast<float *>(smem + S * C::kStage);
    uint8_t *tail = smem + S * C::kStage + C::kHTile;
    uint64_t *full = reinterpret_cast<uint64_t *>(tail);  // TMA landed
    uint64_t *ready = full + S;    // operands unpacked (packed modes)
    uint64_t *empty = ready + S;   // MMAs finished reading the stage
    uint64_t *tfull = empty + S;   // drain slot filled
    uint64_t *tempty = tfull + 2;  // drain slot drained
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *s_rowa = reinterpret_cast<float *>(tail + 512);        // [kBN]
    int *s_rowt = reinterpret_cast<int *>(tail + 512 + 4 * kBN);  // [kBN]

    const int warp = jt::warp_id(), lane = jt::lane_id();
    const int nch_tiles = p.n_ch / C::kChTile;
    const int nk = p.K / kBK;
    const int total = __ldg(&p.tile_off[p.E]) * nch_tiles;
    int *err = p.err;
    // stage layout: [A unpacked 128 x 128 | X 64 x 128 | A packed 128 x kPackedRow]
    auto stage_ptr = [&](int s) { return smem + s * C::kStage; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            jt::mbar_init(&full[s], 1);
            jt::mbar_init(&ready[s], 4);
            jt::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            jt::mbar_init(&tfull[b], 1);
            jt::mbar_init(&tempty[b], 4);
        }
        jt::mbar_init(drain, 1);
        *abort_flag = 0;
        jt::fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        jt::prefetch_tmap(&p.tmA0);
        if (C::kGateUp) jt::prefetch_tmap(&p.tmA1);
        jt::prefetch_tmap(&p.tmX);
    }
    if (warp == 1) {
        jt::tmem_alloc(tmem_slot, C::kTmemCols);
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
            bool ok = true;
            constexpr uint32_t kTx = C::kX + (C::kPacked ? C::kAP : C::kAU);
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                const TileInfo ti = tile_info<C::kChTile>(p, u, nch_tiles);
                const int wrow = ti.e * p.n_ch + ti.c0;  // first weight row of the tile
                for (int kb = 0; kb < nk; ++kb) {
                    if (!jt::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *st = stage_ptr(stage);
                    uint8_t *xs = st + C::kAU, *ap = xs + C::kX;
                    jt::mbar_arrive_expect_tx(&full[stage], kTx);
                    if (C::kPacked) {
                        if (C::kGateUp) {
                            jt::tma_load_2d(ap, &p.tmA0, &full[stage], kb * C::kPackedRow, wrow);
                            jt::tma_load_2d(ap + 64 * C::kPackedRow, &p.tmA1, &full[stage],
                                            kb * C::kPackedRow, wrow);
                        } else {
                            jt::tma_load_2d(ap, &p.tmA0, &full[stage], kb * C::kPackedRow, wrow);
                        }
                    } else {
                        if (C::kGateUp) {
                            jt::tma_load_2d(st, &p.tmA0, &full[stage], kb * kBK, wrow);
                            jt::tma_load_2d(st + 64 * kBK, &p.tmA1, &full[stage], kb * kBK, wrow);
                        } else {
                            jt::tma_load_2d(st, &p.tmA0, &full[stage], kb * kBK, wrow);
                        }
                    }
                    jt::tma_load_2d(xs, &p.tmX, &full[stage], kb * kBK, ti.r0);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                for (int s = 0; s < S; ++s) {
                    if (!(issued_mask & (1u << s))) continue;
                    const uint32_t par = (issued_phase >> s) & 1u;
                    const long long t0 = clock64();
                    while (!jt::mbar_try_wait(&full[s], par) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t kIdesc = jt::idesc_i8(kBM, kBN);
            constexpr int kStepsPerUnit = C::kUnitK == 0 ? 1 : C::kUnitK / 32;
            uint32_t stage = 0, phase = 0;
            uint32_t slot = 0, slot_phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < total && ok; u += gridDim.x) {
                for (int kb = 0; kb < nk && ok; ++kb) {
                    uint64_t *gate = C::kPacked ? &ready[stage] : &full[stage];
                    if (!jt::mbar_wait(gate, phase, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    jt::tc_fence_after();
                    const uint32_t base = jt::smem_u32(stage_ptr(stage));
                    const uint64_t dA = jt::umma_desc_sw128(base);
                    const uint64_t dX = jt::umma_desc_sw128(base + C::kAU);
#pragma unroll
                    for (int ks = 0; ks < kBK / 32; ++ks) {
                        const bool unit_start = (C::kUnitK == 0) ? (kb == 0 && ks == 0)
                                                                 : (ks % kStepsPerUnit == 0);
                        const bool unit_end = (C::kUnitK == 0)
                                                  ? (kb == nk - 1 && ks == kBK / 32 - 1)
                                                  : (ks % kStepsPerUnit == kStepsPerUnit - 1);
                        if (unit_start) {
                            if (!jt::mbar_wait(&tempty[slot], slot_phase ^ 1u, abort_flag, err)) {
                                ok = false;
                                break;
                            }
                            jt::tc_fence_after();
                        }
                        jt::mma_i8(tmem_base + slot * kBN, dA + 2u * ks, dX + 2u * ks, kIdesc,
                                   unit_start ? 0u : 1u);
                        if (unit_end) {
                            jt::mma_commit(&tfull[slot]);
                            slot ^= 1u;
                            if (slot == 0) slot_phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    jt::mma_commit(&empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (!ok) {
                jt::mma_commit(drain);
                const long long t0 = clock64();
                while (!jt::mbar_try_wait(drain, 0) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
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
                    unpack_row<C::kBits>(st + C::kAU + C::kX + r * C::kPackedRow, st, r);
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
        const int q = warp & 3;                         // TMEM lane quarter
        const int lr = q * 32 + lane;                   // operand row = TMEM lane
        const int etid = threadIdx.x - kEpiWarp0 * 32;  // 0..127
        // gate/up: rows 0..63 gate of channel lr, rows 64..127 up of channel lr-64
        const bool is_up = C::kGateUp && lr >= 64;
        const int lch = C::kGateUp ? (lr & 63) : lr;
        uint32_t slot = 0, slot_phase = 0;
        const int ngroups = p.K / 64;
        for (int u = blockIdx.x; u < total; u += gridDim.x) {
            const TileInfo ti = tile_info<C::kChTile>(p, u, nch_tiles);
            const int ch = ti.c0 + lch;  // output channel within the expert
            named_bar_epi();  // previous tile done with the SMEM scratch
            if (etid < kBN) {
                const int row = ti.r0 + etid;
                const bool valid = row < ti.r_end;
                if (C::kGateUp) {
                    s_rowa[etid] = valid ? __ldg(&p.row_scale[row]) : 0.0f;
                } else {
                    s_rowa[etid] = (MODE == DN_ROUTED && valid) ? __ldg(&p.row_w[row]) : 0.0f;
                    s_rowt[etid] = valid ? (MODE == DN_ROUTED ? __ldg(&p.row_tok[row]) : row) : -1;
                }
            }
            if (!C::kGateUp) {
                // activation group scales of the tile as [group][row] (zero for rows
                // outside the expert; their results are never written)
                for (int i = etid; i < ngroups * kBN; i += 128) {
                    const int g = i / kBN, j = i % kBN, row = ti.r0 + j;
                    h_tile[i] = row < ti.r_end ? __ldg(&p.blk_scale[(size_t)row * ngroups + g]) : 0.0f;
                }
            }
            named_bar_epi();
            float r[kBN];
#pragma unroll
            for (int j = 0; j < kBN; ++j) r[j] = 0.0f;
            const __half *gsrow = nullptr;
            if (C::kPacked)
                gsrow = (is_up ? p.gs1 : p.gs0) + ((size_t)ti.e * p.n_ch + ch) * ngroups;
            const int nunits = C::kUnitK == 0 ? 1 : p.K / C::kUnitK;
            bool ok = true;
            float s_next = C::kPacked ? __half2float(gsrow[0]) : 1.0f;
            for (int un = 0; un < nunits; ++un) {
                const float s = s_next;
                if (C::kPacked && un + 1 < nunits) s_next = __half2float(gsrow[un + 1]);
                if (!jt::mbar_wait(&tfull[slot], slot_phase, abort_flag, err)) {
                    ok = false;
                    break;
                }
                jt::tc_fence_after();
                const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + slot * kBN;
                uint32_t a[kBN];
                {
                    uint32_t (&a0)[32] = *reinterpret_cast<uint32_t (*)[32]>(&a[0]);
                    uint32_t (&a1)[32] = *reinterpret_cast<uint32_t (*)[32]>(&a[32]);
                    jt::tmem_ld32(trow, a0);
                    jt::tmem_ld32(trow + 32, a1);
                    jt::tmem_wait_ld();
                }
                jt::tc_fence_before();
                __syncwarp();
                if (lane == 0) jt::mbar_arrive(&tempty[slot]);
                slot ^= 1u;
                if (slot == 0) slot_phase ^= 1u;
                if (MODE == GU_ROUTED) {
#pragma unroll
                    for (int j = 0; j < kBN; ++j)
                        r[j] = __fmaf_rn(__int2float_rn((int32_t)a[j]), s, r[j]);
                } else if (MODE == GU_SHARED) {
#pragma unroll
                    for (int j = 0; j < kBN; ++j) r[j] = __int2float_rn((int32_t)a[j]);
                } else {
                    const float *hsg = h_tile + un * kBN;
#pragma unroll
                    for (int j = 0; j < kBN; j += 4) {
                        const float4 h4 = *reinterpret_cast<const float4 *>(hsg + j);
                        const float hv[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float pf = __int2float_rn((int32_t)a[j + i]);
                            const float t = (MODE == DN_ROUTED) ? __fmul_rn(pf, s) : pf;
                            r[j + i] = __fmaf_rn(t, hv[i], r[j + i]);
                        }
                    }
                }
            }
            if (!ok) break;
            if constexpr (C::kGateUp) {
                float cscale = 1.0f;
                if (MODE == GU_SHARED) cscale = __ldg(is_up ? &p.cs1[ch] : &p.cs0[ch]);
                // pass 1: gate rows publish g[row][ch]
                if (!is_up) {
#pragma unroll
                    for (int j = 0; j < kBN; ++j) {
                        const float xs = s_rowa[j];
                        h_tile[j * 64 + lch] = (MODE == GU_ROUTED)
                                                   ? __fmul_rn(r[j], xs)
                                                   : __fmul_rn(__fmul_rn(r[j], xs), cscale);
                    }
                }
                named_bar_epi();
                // pass 2: up rows combine into h = SwiGLU(g, u) in place
                if (is_up) {
#pragma unroll
                    for (int j = 0; j < kBN; ++j) {
                        const float xs = s_rowa[j];
                        const float uv = (MODE == GU_ROUTED)
                                             ? __fmul_rn(r[j], xs)
                                             : __fmul_rn(__fmul_rn(r[j], xs), cscale);
                        h_tile[j * 64 + lch] = jt::swiglu(h_tile[j * 64 + lch], uv);
                    }
                }
                named_bar_epi();
                // pass 3: two threads per row, 32 channels each -> codes + scale
                const int j = etid >> 1, half = etid & 1;
                const float *hr = h_tile + j * 64 + half * 32;
                float m = 0.0f;
                int nf = 0;
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 v4 = *reinterpret_cast<const float4 *>(hr + i);
                    nf |= !isfinite(v4.x) | !isfinite(v4.y) | !isfinite(v4.z) | !isfinite(v4.w);
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(v4.x), fabsf(v4.y)), fmaxf(fabsf(v4.z), fabsf(v4.w))));
                }
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                nf |= __shfl_xor_sync(0xffffffffu, nf, 1);
                const int row = ti.r0 + j;
                if (row < ti.r_end) {
                    if (nf) atomicExch(err, JT_KERR_NONFINITE);
                    const jt::QuantBlock qb = jt::quant_block(m);
                    uint32_t words[8];
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        uint32_t word = 0;
#pragma unroll
                        for (int b2 = 0; b2 < 4; ++b2) {
                            const int c = jt::quant_code(hr[4 * w + b2], qb);
                            word |= (uint32_t)(uint8_t)(int8_t)c << (8 * b2);
                        }
                        words[w] = word;
                    }
                    int8_t *dst = p.hq + (size_t)row * p.n_ch + ti.c0 + half * 32;
                    *reinterpret_cast<uint4 *>(dst) = make_uint4(words[0], words[1], words[2], words[3]);
                    *reinterpret_cast<uint4 *>(dst + 16) = make_uint4(words[4], words[5], words[6], words[7]);
                    if (half == 0) p.hs[(size_t)row * (p.n_ch / 64) + ti.c0 / 64] = qb.scale_f;
                }
            } else {
                float cs = 1.0f;
                if (MODE == DN_SHARED) cs = __ldg(&p.cs0[ch]);
#pragma unroll
                for (int j = 0; j < kBN; ++j) {
                    const int tok = s_rowt[j];
                    if (tok < 0) continue;
                    const float v = (MODE == DN_ROUTED) ? __fmul_rn(s_rowa[j], r[j]) : __fmul_rn(r[j], cs);
                    float *dst = p.y + (size_t)tok * p.n_ch + ch;
                    if (p.y_accumulate) atomicAdd(dst, v);
                    else *dst = v;
                }
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        jt::tc_fence_after();
        jt::tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int MODE>
int launch(MoeGemmParams &p, int max_tiles_hint, cudaStream_t stream) {
    using C = Cfg<MODE>;
    auto kern = k_moe_gemm<MODE>;
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

}  // namespace

// Routed gate/up: wg, wu packed INT2 [E][f][d/4]; gs, us fp16 [E][f][d/64];
// xd int8 [rows][d] in expert order with xs_d [rows]; writes hq [rows][f],
// hs [rows][f/64].  max_tiles_hint bounds the grid (0 = all SMs).
extern "C" int jtk_moe_gateup_routed(const uint8_t *wg, const uint8_t *wu, const void *gs,
                                     const void *us, int E, int f, int d, const int8_t *xd,
                                     int rows_cap, const float *xs_d, const int32_t *row_off,
                                     const int32_t *tile_off, int8_t *hq, float *hs,
                                     int max_tiles_hint, cudaStream_t stream) {
    if (f % 64 || d % kBK || E <= 0 || rows_cap <= 0) return -1;
    MoeGemmParams p{};
    const uint32_t prow = d / 4;
    if (!jt::make_tmap_2d_u8(&p.tmA0, wg, prow, (uint64_t)E * f, prow, Cfg<GU_ROUTED>::kPackedRow, 64, false) ||
        !jt::make_tmap_2d_u8(&p.tmA1, wu, prow, (uint64_t)E * f, prow, Cfg<GU_ROUTED>::kPackedRow, 64, false) ||
        !jt::make_tmap_2d_u8(&p.tmX, xd, d, rows_cap, d, kBK, kBN, true))
        return -2;
    p.row_off = row_off;
    p.tile_off = tile_off;
    p.E = E;
    p.n_ch = f;
    p.K = d;
    p.gs0 = static_cast<const __half *>(gs);
    p.gs1 = static_cast<const __half *>(us);
    p.row_scale = xs_d;
    p.hq = hq;
    p.hs = hs;
    return launch<GU_ROUTED>(p, max_tiles_hint, stream);
}

// Routed down: wd packed INT4 [E][d][f/2], ds fp16 [E][d][f/64]; hq [rows][f]
// with hs [rows][f/64]; y[tok][d] += w_row * y_pair (atomic).
extern "C" int jtk_moe_down_routed(const uint8_t *wd, const void *ds, int E, int d, int f,
                                   const int8_t *hq, int rows_cap, const float *hs,
                                   const int32_t *row_off, const int32_t *tile_off,
                                   const int32_t *row_tok, const float *row_w, float *y,
                                   int max_tiles_hint, cudaStream_t stream) {
    // the tile's activation group scales are staged in SMEM: K <= 4096
    if (d % kBM || f % kBK || f > 4096 || E <= 0 || rows_cap <= 0) return -1;
    MoeGemmParams p{};
    const uint32_t prow = f / 2;
    if (!jt::make_tmap_2d_u8(&p.tmA0, wd, prow, (uint64_t)E * d, prow, Cfg<DN_ROUTED>::kPackedRow, kBM, false) ||
        !jt::make_tmap_2d_u8(&p.tmX, hq, f, rows_cap, f, kBK, kBN, true))
        return -2;
    p.tmA1 = p.tmA0;
    p.row_off = row_off;
    p.tile_off = tile_off;
    p.E = E;
    p.n_ch = d;
    p.K = f;
    p.gs0 = static_cast<const __half *>(ds);
    p.blk_scale = hs;
    p.y = y;
    p.row_tok = row_tok;
    p.row_w = row_w;
    p.y_accumulate = 1;
    return launch<DN_ROUTED>(p, max_tiles_hint, stream);
}

// Shared gate/up (one shared expert): wsg, wsu int8 [fs][d] with per-channel
// ssg, ssu; x int8 [T][d], xs [T]; writes hq [T][fs], hs [T][fs/64].
// row_off = {0, T}, tile_off = {0, ceil(T/64)} (device, 2 entries each).
extern "C" int jtk_moe_gateup_shared(const int8_t *wsg, const int8_t *wsu, const float *ssg,
                                     const float *ssu, int fs, int d, const int8_t *xq, int T,
                                     const float *xs, const int32_t *row_off,
                                     const int32_t *tile_off, int8_t *hq, float *hs,
                                     cudaStream_t stream) {
    if (fs % 64 || d % kBK || T <= 0) return -1;
    MoeGemmParams p{};
    if (!jt::make_tmap_2d_u8(&p.tmA0, wsg, d, fs, d, kBK, 64, true) ||
        !jt::make_tmap_2d_u8(&p.tmA1, wsu, d, fs, d, kBK, 64, true) ||
        !jt::make_tmap_2d_u8(&p.tmX, xq, d, T, d, kBK, kBN, true))
        return -2;
    p.row_off = row_off;
    p.tile_off = tile_off;
    p.E = 1;
    p.n_ch = fs;
    p.K = d;
    p.cs0 = ssg;
    p.cs1 = ssu;
    p.row_scale = xs;
    p.hq = hq;
    p.hs = hs;
    return launch<GU_SHARED>(p, ((T + kBN - 1) / kBN) * (fs / 64), stream);
}

// Shared down: wsd int8 [d][fs] with per-channel ssd; hq [T][fs], hs [T][fs/64];
// y[t][d] = (accumulate ? y + v : v).
extern "C" int jtk_moe_down_shared(const int8_t *wsd, const float *ssd, int d, int fs,
                                   const int8_t *hq, int T, const float *hs,
                                   const int32_t *row_off, const int32_t *tile_off, float *y,
                                   int accumulate, cudaStream_t stream) {
    if (d % kBM || fs % kBK || fs > 4096 || T <= 0) return -1;
    MoeGemmParams p{};
    if (!jt::make_tmap_2d_u8(&p.tmA0, wsd, fs, d, fs, kBK, kBM, true) ||
        !jt::make_tmap_2d_u8(&p.tmX, hq, fs, T, fs, kBK, kBN, true))
        return -2;
    p.tmA1 = p.tmA0;
    p.row_off = row_off;
    p.tile_off = tile_off;
    p.E = 1;
    p.n_ch = d;
    p.K = fs;
    p.cs0 = ssd;
    p.blk_scale = hs;
    p.y = y;
    p.y_accumulate = accumulate;
    return launch<DN_SHARED>(p, ((T + kBN - 1) / kBN) * (d / kBM), stream);
}
