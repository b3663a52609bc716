// jt_pair.cuh - the CTA-pair (tcgen05 cta_group::2) GEMM pipeline shared by
// the dense int8 kernels whose tiles are 256 weight rows x 256 token rows.
//
// A 2-CTA cluster computes one tile with tcgen05.mma.cta_group::2 (M = 256,
// N = 256, K = 32).  Rank r holds rows 128r .. 128r+127 of A (its weight
// rows) and tokens 128r .. 128r+127 of B in its own shared memory, and D for
// its 128 weight rows x all 256 tokens in its TMEM.  Per 128-K stage each SM
// reads 32 KB from L2 (a single-CTA 128 x 256 tile reads 48 KB, a 128 x 128
// tile 32 KB for half the work), and each MMA reads 8 KB of its shared
// memory.
//
// Warp roles: w0 TMA producer of its rank's boxes, w1 TMEM allocator of both
// ranks and, on rank 0, the single MMA issuer, w2-9 read the accumulators
// (w reads TMEM lanes 32*(w%4) .. +31 and token columns 128*((w-2)/4) ..
// +127); a kernel may add warps of its own after them.
//
// Barriers: full[s] on rank 0 counts the bytes of both ranks' boxes of stage
// s (rank 1's loads report to it through the pair form of the TMA load; rank
// 0's producer posts the expected 64 KB); empty[s] and tfull[b] in both ranks
// are signalled by the MMA commit multicast to both ranks; tempty[b] on rank
// 0 counts the eight epilogue warps of each rank.  The TMA loads carry no
// multicast: each rank fetches its own boxes.  Every wait is bounded.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_ptx.cuh"

namespace jt {
namespace pair {

constexpr int kBK = 128;                       // K bytes per stage (one swizzle atom)
constexpr int kStages = 6;
constexpr uint32_t kBox = 128 * kBK;           // one 128-row x 128-byte box, 16 KB
constexpr uint32_t kStage = 2 * kBox;          // weight rows + token rows
constexpr uint32_t kCols = 512;                // two 256-column accumulators
constexpr int kThreads = 320;                  // 10 warps
constexpr int kEpiWarps = 8;                   // warps 2-9: the TMEM readers
constexpr uint32_t kRing = kStages * kStage;   // 192 KB
constexpr uint32_t kBarBytes = 512;            // barriers and flags after the ring

struct Ctx {
    uint8_t *smem;  // 1024-aligned base: the stage ring
    uint64_t *full, *empty, *tfull, *tempty, *drain;
    uint32_t *tmem_slot;
    volatile int *abort_flag;
    int *err;
    uint32_t rank;
    int pair, npairs, warp, lane;
    uint32_t tmem_base;
};

// Carves the barriers out of the `kBarBytes` at `bars` (the first 256 bytes),
// initialises them, allocates both ranks' TMEM and synchronises the
// cluster.  Every thread.  S: stages of the ring (S * kStage bytes at smem).
template <int S = kStages>
__device__ __forceinline__ void setup(Ctx &c, uint8_t *smem, uint8_t *bars, int *err,
                                      const CUtensorMap *const *maps, int nmaps) {
    c.smem = smem;
    c.full = reinterpret_cast<uint64_t *>(bars);
    c.empty = c.full + S;
    c.tfull = c.empty + S;
    c.tempty = c.tfull + 2;
    c.drain = c.tempty + 2;
    c.tmem_slot = reinterpret_cast<uint32_t *>(c.drain + 1);
    c.abort_flag = reinterpret_cast<volatile int *>(c.tmem_slot + 1);
    c.err = err;
    c.warp = warp_id();
    c.lane = lane_id();
    c.rank = cluster_ctarank();
    c.pair = static_cast<int>(cluster_id_x());
    c.npairs = static_cast<int>(ncluster_x());
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&c.full[s], 1);
            mbar_init(&c.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&c.tfull[b], 1);
            mbar_init(&c.tempty[b], 2 * kEpiWarps);
        }
        mbar_init(c.drain, 1);
        *c.abort_flag = 0;
        fence_mbar_init();
    }
    if (c.warp == 0 && c.lane == 0)
        for (int i = 0; i < nmaps; ++i) prefetch_tmap(maps[i]);
    if (c.warp == 1) {
        tmem_alloc_pair(c.tmem_slot, kCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    // both ranks' barriers are initialised before any cross-CTA signal
    cluster_sync();
    tc_fence_after();
    c.tmem_base = *c.tmem_slot;
}

// Warp 0, lane 0.  For every tile of this pair and every 128-K block: the
// weight box(es) through load_a(dst, kb, tile, bar) (16 KB in all, 128 rows
// in the 128-byte-swizzled K-major layout) and this rank's 128 token rows
// m0 = tile_tok(tile) * 256 + 128 * rank from tmX.
template <int S = kStages, typename LoadA, typename TileTok>
__device__ __forceinline__ void producer(Ctx &c, const CUtensorMap *tmX, int ntiles, int nk,
                                         LoadA &&load_a, TileTok &&tile_tok) {
    uint32_t stage = 0, phase = 0;
    uint32_t issued_mask = 0, issued_phase = 0;
    bool ok = true;
    for (int tile = c.pair; tile < ntiles && ok; tile += c.npairs) {
        const int m0 = tile_tok(tile) * 256 + static_cast<int>(c.rank) * 128;
        for (int kb = 0; kb < nk; ++kb) {
            if (!mbar_wait_cluster(&c.empty[stage], phase ^ 1u, c.abort_flag, c.err)) {
                ok = false;
                break;
            }
            uint8_t *sA = c.smem + stage * kStage;
            if (c.rank == 0) mbar_arrive_expect_tx(&c.full[stage], 2 * kStage);
            const uint32_t bar = cluster_addr(&c.full[stage], 0);
            load_a(sA, kb, tile, bar);
            tma_load_2d_pair(sA + kBox, tmX, bar, kb * kBK, m0);
            issued_mask |= 1u << stage;
            issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == S) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
    // Tail: the MMA commits that release the last stages arrive on this
    // CTA's barriers asynchronously; wait for every one of them so none
    // lands after the CTA has exited.
    for (int i = 0; i < S && ok; ++i) {
        if (!mbar_wait_cluster(&c.empty[stage], phase ^ 1u, c.abort_flag, c.err)) ok = false;
        if (++stage == S) {
            stage = 0;
            phase ^= 1u;
        }
    }
    if (!ok) {
        // Every issued box must land before the CTA exits.  Rank 0 waits
        // (bounded) for the last issued phase of each stage; rank 1 cannot
        // observe its boxes (they report to rank 0) and waits a fixed,
        // bounded interval instead.
        if (c.rank == 0) {
            for (int s = 0; s < S; ++s) {
                if (!(issued_mask & (1u << s))) continue;
                const uint32_t par = (issued_phase >> s) & 1u;
                const long long t0 = clock64();
                while (!mbar_try_wait(&c.full[s], par) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
                }
            }
        } else if (issued_mask) {
            const long long t0 = clock64();
            while (clock64() - t0 < JT_SPIN_CYCLES / 64) __nanosleep(1000);
        }
    }
}

// Warp 1, lane 0 of rank 0: the pair's MMAs, tile by tile into the two TMEM
// accumulators in turn.
template <int S = kStages>
__device__ __forceinline__ void mma(Ctx &c, int ntiles, int nk) {
    constexpr uint32_t kIdesc = idesc_i8(256, 256);
    uint32_t stage = 0, phase = 0;
    int it = 0;
    bool ok = true;
    for (int tile = c.pair; tile < ntiles && ok; tile += c.npairs, ++it) {
        const uint32_t buf = it & 1;
        const uint32_t use = (it >> 1) & 1;
        if (!mbar_wait_cluster(&c.tempty[buf], use ^ 1u, c.abort_flag, c.err)) {
            ok = false;
            break;
        }
        tc_fence_after();
        const uint32_t d_tmem = c.tmem_base + buf * 256;
        for (int kb = 0; kb < nk; ++kb) {
            if (!mbar_wait_cluster(&c.full[stage], phase, c.abort_flag, c.err)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t aA = smem_u32(c.smem + stage * kStage);
            const uint64_t da = umma_desc_sw128(aA);
            const uint64_t db = umma_desc_sw128(aA + kBox);
#pragma unroll
            for (int j = 0; j < kBK / 32; ++j)
                mma_i8_pair(d_tmem, da + 2u * j, db + 2u * j, kIdesc, (kb | j) != 0 ? 1u : 0u);
            mma_commit_pair(&c.empty[stage], 0x3);
            if (++stage == S) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if (!ok) break;
        mma_commit_pair(&c.tfull[buf], 0x3);
    }
    if (!ok) {
        mma_commit_pair(c.drain, 0x1);
        const long long t0 = clock64();
        while (!mbar_try_wait(c.drain, 0) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
        }
    }
}

// Epilogue warp: wait for tile `it`'s accumulator (false on abort).
__device__ __forceinline__ bool epi_acquire(Ctx &c, int it) {
    if (!mbar_wait_cluster(&c.tfull[it & 1], (it >> 1) & 1, c.abort_flag, c.err)) return false;
    tc_fence_after();
    return true;
}

// Epilogue warp: this warp is done reading tile `it`'s accumulator.
__device__ __forceinline__ void epi_release(Ctx &c, int it) {
    tc_fence_before();
    __syncwarp();
    if (c.lane == 0) {
        if (c.rank == 0)
            mbar_arrive(&c.tempty[it & 1]);
        else
            mbar_arrive_cluster(&c.tempty[it & 1], 0);
    }
}

// TMEM address of this epilogue warp's lane quarter in accumulator `it & 1`.
__device__ __forceinline__ uint32_t epi_row(const Ctx &c, int it) {
    return c.tmem_base + (static_cast<uint32_t>((c.warp & 3) * 32) << 16) + (it & 1) * 256;
}

// Every thread, at the end: no CTA of the pair releases TMEM or exits while
// its peer may still signal its barriers or read its shared memory.
__device__ __forceinline__ void teardown(Ctx &c) {
    __syncthreads();
    cluster_sync();
    if (c.warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(c.tmem_base, kCols);
    }
}

// Runs fn(v, c0) over the 32-column TMEM chunks c0 = cb, cb+32, .. < ce of
// this warp's lane quarter, the load of the next chunk in flight while fn
// processes the current one (warp-uniform bounds).
template <typename Fn>
__device__ __forceinline__ void tmem_columns(uint32_t trow, int cb, int ce, Fn &&fn) {
    if (cb >= ce) return;
    uint32_t va[32], vb[32];
    tmem_ld32(trow + cb, va);
#pragma unroll 1
    for (int c0 = cb; c0 < ce; c0 += 64) {
        tmem_wait_ld32(va);
        const bool more = c0 + 32 < ce;
        if (more) tmem_ld32(trow + c0 + 32, vb);
        fn(va, c0);
        if (!more) break;
        tmem_wait_ld32(vb);
        if (c0 + 64 < ce) tmem_ld32(trow + c0 + 64, va);
        fn(vb, c0 + 32);
    }
}

// Launch configuration of `pairs` 2-CTA clusters (attr: one attribute slot
// owned by the caller, alive until the launch).
inline cudaLaunchConfig_t launch_config(int pairs, size_t smem, cudaStream_t stream,
                                        cudaLaunchAttribute *attr, int threads = kThreads) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cfg;
}

}  // namespace pair
}  // namespace jt
