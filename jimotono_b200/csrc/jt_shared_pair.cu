// jt_shared_pair.cu - gate/up projection of a shared expert, fused with
// SwiGLU, on the CTA-pair tensor-core pipeline (jt_pair.cuh, tcgen05
// cta_group::2).  h leaves as bf16 with the running maximum of |h| of every
// token row (the row's requantization scale, jt_shared.cu).
//
// Arithmetic (identical to the dense-GEMM form of jt_shared.cu used for
// T < 256: moe_layer.c:129-157 with the W8A8 projections of
// w8a8.c:1021-1072):
//   g[t][c] = ((float)acc_gate[t][c] * xs[t]) * sg[c]     (xs[t] = meta[t].x)
//   u[t][c] = ((float)acc_up[t][c]   * xs[t]) * su[c]
//   h[t][c] = SwiGLU(g, u)                      (jt_swiglu.cuh)
//   hb[t][c] = bf16_rn(h[t][c]);  rowmax[t] = max(rowmax[t], max_c |hb[t][c]|)
//
// Tiles: a pair covers 128 output channels x 256 tokens; rank r's 128 weight
// rows are gate rows c0 + 64r .. +63 over up rows c0 + 64r .. +63 (two
// 64-row TMA boxes), so its TMEM lanes 0-63 hold g and lanes 64-127 hold u of
// the same 64 channels, for all 256 tokens.  Per 128-K stage an SM reads
// 32 KB from L2 for 128 x 256 x 128 MACs, half the bytes per MAC of the
// single-CTA 128 x 128 tile.
//
// Epilogue, two groups of eight warps per CTA joined by a two-deep ring of
// 32-token chunks per token half (bounded mbarrier waits throughout):
//   readers (warps 2-9, TMEM lane quarter w%4, token half (w-2)/4): scale
//     their 32 channels of g or u for 32 tokens and store them to the
//     chunk's [32 tokens][64 channels] fp32 block in shared memory;
//   workers (warps 10-25, token half (w-10)/8): eight lanes per token form
//     h over 8 channels each, store them as bf16 (16 bytes per lane) and
//     fold the 64-channel max of |bf16 h| into the row maximum with one
//     atomic max per token; warp w takes tokens 4((w-10)%8) .. +3 of every
//     chunk of its half.
// The readers release the accumulator as soon as a tile is staged, so the
// SwiGLU of one tile overlaps the TMEM reads of the next.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_pair.cuh"
#include "jt_ptx.cuh"
#include "jt_quant.cuh"
#include "jt_runtime.cuh"
#include "jt_swiglu.cuh"

namespace {

namespace jp = jt::pair;

constexpr int kStages = 5;                       // 160 KB ring
constexpr int kThreads = 832;                    // 26 warps
constexpr int kWorkers = 16;                     // warps 10-25: 8 per token half
constexpr uint32_t kBlock = 32 * 64 * 4;         // one 32-token x 64-channel fp32 block
constexpr uint32_t kChunk = 2 * kBlock;          // g block, u block
constexpr uint32_t kStaging = 2 * 2 * kChunk;    // two chunks per token half
constexpr size_t kSmem = 1024 + kStages * jp::kStage + kStaging + jp::kBarBytes;
static_assert(kSmem <= 232448, "shared memory");

struct SharedGuParams {
    CUtensorMap tmG, tmU, tmX;  // gate / up weights [fs][d] (64-row boxes), tokens [T][d]
    int T, fs, d;
    const float4 *meta;         // per-token {activation scale, 1, t, 0} [T]
    const float *sg, *su;       // per-channel weight scales [fs]
    uint16_t *hb;               // [T][fs] bf16
    float *rowmax;              // [T], max |hb| of the row (atomic max on the bits; zero before)
    int *err;
};

__global__ void __launch_bounds__(kThreads, 1) k_shared_gu_pair(const __grid_constant__ SharedGuParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    float *staging = reinterpret_cast<float *>(smem + kStages * jp::kStage);
    uint8_t *bars = smem + kStages * jp::kStage + kStaging;
    // chunk ring per token half h and slot b: cfull (readers -> workers),
    // cempty (workers -> readers)
    uint64_t *cfull = reinterpret_cast<uint64_t *>(bars + 256);  // [h*2 + b]
    uint64_t *cempty = cfull + 4;
    jp::Ctx c;
    const CUtensorMap *maps[3] = {&p.tmG, &p.tmU, &p.tmX};
    if (threadIdx.x == 0)
        for (int i = 0; i < 4; ++i) {
            jt::mbar_init(&cfull[i], 4);
            jt::mbar_init(&cempty[i], kWorkers / 2);
        }
    jp::setup<kStages>(c, smem, bars, p.err, maps, 3);  // its __syncthreads publishes the inits
    const int n_ch_tiles = p.fs / 128;
    const int ntiles = n_ch_tiles * ((p.T + 255) / 256);
    const int nk = p.d / jp::kBK;

    if (c.warp == 0) {
        if (c.lane == 0)
            jp::producer<kStages>(
                c, &p.tmX, ntiles, nk,
                [&](uint8_t *dst, int kb, int tile, uint32_t bar) {
                    const int c0 = (tile % n_ch_tiles) * 128 + static_cast<int>(c.rank) * 64;
                    jt::tma_load_2d_pair(dst, &p.tmG, bar, kb * jp::kBK, c0);
                    jt::tma_load_2d_pair(dst + jp::kBox / 2, &p.tmU, bar, kb * jp::kBK, c0);
                },
                [&](int tile) { return tile / n_ch_tiles; });
    } else if (c.warp == 1) {
        if (c.lane == 0 && c.rank == 0) jp::mma<kStages>(c, ntiles, nk);
    } else if (c.warp < 2 + jp::kEpiWarps) {
        // readers
        const int q = c.warp & 3;                  // lane quarter: 0,1 gate, 2,3 up
        const int half = (c.warp - 2) >> 2;        // token columns 128*half .. +127
        const int lc = (q & 1) * 32 + c.lane;      // channel within the CTA's 64
        const bool is_up = q >= 2;
        uint32_t n = 0;                            // chunks of this half so far
        bool ok = true;
        int it = 0;
        for (int tile = c.pair; tile < ntiles && ok; tile += c.npairs, ++it) {
            if (!jp::epi_acquire(c, it)) break;
            const int cbase = (tile % n_ch_tiles) * 128 + static_cast<int>(c.rank) * 64;
            const int m0 = (tile / n_ch_tiles) * 256;
            const float cs = __ldg(is_up ? &p.su[cbase + lc] : &p.sg[cbase + lc]);
            const int cols = (p.T - m0) < 256 ? (p.T - m0) : 256;
            const int cb = half * 128, ce = (cb + 128) < cols ? (cb + 128) : cols;
            const uint32_t trow = jp::epi_row(c, it);
#pragma unroll 1
            for (int c0 = cb; c0 < ce && ok; c0 += 32) {
                // single-buffered TMEM loads: the register budget of 26 warps
                uint32_t v[32];
                jt::tmem_ld32(trow + c0, v);
                jt::tmem_wait_ld();
                const int slot = half * 2 + (n & 1);
                if (!jt::mbar_wait(&cempty[slot], ((n >> 1) & 1) ^ 1u, c.abort_flag, c.err)) {
                    ok = false;
                    break;
                }
                float *blk = staging + slot * (kChunk / 4) + (is_up ? kBlock / 4 : 0);
                const int tok0 = m0 + c0;
                const int nvalid = (p.T - tok0) < 32 ? (p.T - tok0) : 32;
                const float xl = c.lane < nvalid ? __ldg(&p.meta[tok0 + c.lane].x) : 0.0f;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float xj = __shfl_sync(0xffffffffu, xl, j);
                    blk[j * 64 + lc] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(v[j])), xj), cs);
                }
                __syncwarp();
                if (c.lane == 0) jt::mbar_arrive(&cfull[slot]);
                ++n;
            }
            jp::epi_release(c, it);
        }
    } else {
        // workers
        const int w2 = c.warp - 2 - jp::kEpiWarps;
        const int half = w2 >> 3, qq = w2 & 7;
        const int sl = c.lane & 7, gq = c.lane >> 3;
        uint32_t n = 0;
        bool ok = true;
        for (int tile = c.pair; tile < ntiles && ok; tile += c.npairs) {
            const int cbase = (tile % n_ch_tiles) * 128 + static_cast<int>(c.rank) * 64;
            const int m0 = (tile / n_ch_tiles) * 256;
            const int cols = (p.T - m0) < 256 ? (p.T - m0) : 256;
            const int cb = half * 128, ce = (cb + 128) < cols ? (cb + 128) : cols;
            for (int c0 = cb; c0 < ce && ok; c0 += 32, ++n) {
                const int slot = half * 2 + (n & 1);
                if (!jt::mbar_wait(&cfull[slot], (n >> 1) & 1, c.abort_flag, c.err)) {
                    ok = false;
                    break;
                }
                const float *gblk = staging + slot * (kChunk / 4);
                const float *ublk = gblk + kBlock / 4;
                const int tok0 = m0 + c0;
                const int nvalid = (p.T - tok0) < 32 ? (p.T - tok0) : 32;
                {
                    const int j = 4 * qq + gq;
                    const bool live = j < nvalid;
                    const float4 *gp = reinterpret_cast<const float4 *>(gblk + j * 64 + 8 * sl);
                    const float4 *up = reinterpret_cast<const float4 *>(ublk + j * 64 + 8 * sl);
                    const float4 g0 = gp[0], g1 = gp[1], u0 = up[0], u1 = up[1];
                    float h[8];
                    {
                        const float2 ha = jt::swiglu2(make_float2(g0.x, g0.y), make_float2(u0.x, u0.y));
                        const float2 hb = jt::swiglu2(make_float2(g0.z, g0.w), make_float2(u0.z, u0.w));
                        const float2 hc = jt::swiglu2(make_float2(g1.x, g1.y), make_float2(u1.x, u1.y));
                        const float2 hd = jt::swiglu2(make_float2(g1.z, g1.w), make_float2(u1.z, u1.w));
                        h[0] = ha.x, h[1] = ha.y, h[2] = hb.x, h[3] = hb.y;
                        h[4] = hc.x, h[5] = hc.y, h[6] = hd.x, h[7] = hd.y;
                    }
                    bool bad = false;
                    float m = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        if (!live) h[i] = 0.0f;
                        bad |= !isfinite(h[i]);
                        m = fmaxf(m, fabsf(h[i]));
                    }
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
                    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
                    if (__any_sync(0xffffffffu, bad) && c.lane == 0) atomicExch(p.err, JT_KERR_NONFINITE);
                    if (live) {
                        uint32_t hw[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const __nv_bfloat162 v = __floats2bfloat162_rn(h[2 * i], h[2 * i + 1]);
                            hw[i] = *reinterpret_cast<const uint32_t *>(&v);
                        }
                        const int tok = tok0 + j;
                        *reinterpret_cast<uint4 *>(p.hb + (size_t)tok * p.fs + cbase + 8 * sl) =
                            make_uint4(hw[0], hw[1], hw[2], hw[3]);
                        // |bf16(v)| is the bf16 rounding of |v|: the row maximum of the stored values
                        if (sl == 0)
                            atomicMax(reinterpret_cast<unsigned int *>(p.rowmax) + tok,
                                      __float_as_uint(__bfloat162float(__float2bfloat16_rn(m))));
                    }
                }
                __syncwarp();
                if (c.lane == 0) jt::mbar_arrive(&cempty[slot]);
            }
        }
    }
    jp::teardown(c);
}

}  // namespace

// Shared gate/up on the pair pipeline; -1 when the shape does not fit it
// (the caller then uses the single-CTA form).
extern "C" int jtk_shared_gu_pair(const int8_t *wsg, const int8_t *wsu, const float *ssg,
                                  const float *ssu, int fs, int d, const int8_t *xq,
                                  const float4 *sh_meta, int T, uint16_t *hb, float *rowmax,
                                  cudaStream_t stream) {
    if (fs % 128 || d % jp::kBK || T < 256 || fs <= 0 || d <= 0) return -1;
    SharedGuParams p{};
    if (!jt::make_tmap_2d_u8(&p.tmG, wsg, d, fs, d, jp::kBK, 64, true) ||
        !jt::make_tmap_2d_u8(&p.tmU, wsu, d, fs, d, jp::kBK, 64, true) ||
        !jt::make_tmap_2d_u8(&p.tmX, xq, d, T, d, jp::kBK, 128, true))
        return -2;
    p.T = T;
    p.fs = fs;
    p.d = d;
    p.meta = sh_meta;
    p.sg = ssg;
    p.su = ssu;
    p.hb = hb;
    p.rowmax = rowmax;
    p.err = jtk_error_word();
    static bool attr_done = false;
    if (!attr_done) {
        if (cudaFuncSetAttribute(k_shared_gu_pair, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kSmem)) != cudaSuccess)
            return -3;
        attr_done = true;
    }
    const int ntiles = (fs / 128) * ((T + 255) / 256);
    int pairs = jtk_num_sms() / 2;
    if (pairs > ntiles) pairs = ntiles;
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = jp::launch_config(pairs, kSmem, stream, attr, kThreads);
    return cudaLaunchKernelEx(&cfg, k_shared_gu_pair, p) == cudaSuccess ? 0 : -4;
}
