// jt_w8a8.cu - dense W8A8 int8 GEMM on the sm_100a tensor cores.
//
// Computes C[m][n] from int8 activations X [M][K] and int8 weights W [N][K]
// (both K-major, i.e. row-major with K innermost) with exact int32
// accumulation, the arithmetic of the reference jt_w8a8_gemm_per_channel
// (w8a8.c:1021-1072, scalar body w8a8.c:654-686):
//   acc[m][n] = sum_k X[m][k] * W[n][k]            (int32, exact)
// and one of three epilogues:
//   TOKEN_CHANNEL_F32 : C = ((float)acc * sx[m]) * sw[n]          (per-token x per-channel)
//   TOKEN_CHANNEL_F32_ACC: C += the same (the shared experts' down projections
//                      adding into the layer output)
//   TENSOR_CHANNEL_F64: C = (float)((double)acc * (sA * (double)sw[n]))  (w8a8.c:664,676-677)
//   RAW_I32           : C = acc
//
// Design (one CTA per SM, persistent over output tiles):
//   * "swap-AB" orientation: the MMA M side (128 lanes of TMEM) is 128 weight
//     channels, the MMA N side is a tile of BN tokens.  Small token counts
//     (decode, M=64) then waste no tensor-core rows, and in the epilogue each
//     thread owns one output channel, so per-channel scales are per-thread.
//   * warp 0: TMA producer (128x128 B weight box + BNx128 B token box per
//     stage, 128-byte swizzle), warp 1: TMEM allocator + single-thread
//     tcgen05.mma issuer, warps 2-5: epilogue (tcgen05.ld -> scale -> store).
//   * two TMEM accumulator buffers so the epilogue of tile i overlaps the
//     MMAs of tile i+1; S-stage SMEM ring between TMA and MMA.
//   * every mbarrier wait is bounded (jt_ptx.cuh).
//   * M >= 256: the CTA-pair kernel k_w8a8_pair (cta_group::2, 256 x 256
//     tiles per 2-CTA cluster), described above its definition.
#include <cuda.h>
#include <cuda_runtime.h>

#include "jt_internal.h"
#include "jt_pair.cuh"
#include "jt_ptx.cuh"
#include "jt_runtime.cuh"

namespace {

constexpr int kBM = 128;       // weight channels per tile (MMA M)
constexpr int kBK = 128;       // K bytes per pipeline stage (one swizzle atom)
constexpr int kThreads = 192;  // 6 warps

template <int BN>
struct W8A8Cfg {
    static constexpr uint32_t kWBytes = kBM * kBK;
    static constexpr uint32_t kXBytes = BN * kBK;
    static constexpr uint32_t kStage = kWBytes + kXBytes;
    static constexpr int kStages = (200 * 1024 / kStage) > 8 ? 8 : (200 * 1024 / kStage);
    static constexpr uint32_t kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;
    static constexpr int kChunk = BN < 32 ? BN : 32;
    static constexpr size_t kSmem = 1024 + kStages * kStage + 256;
};

template <int N>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld_chunk<16>(uint32_t taddr, uint32_t (&v)[16]) {
    jt::tmem_ld16(taddr, v);
}
template <>
__device__ __forceinline__ void tmem_ld_chunk<32>(uint32_t taddr, uint32_t (&v)[32]) {
    jt::tmem_ld32(taddr, v);
}

// Stores one TMEM chunk of the epilogue: NCOL consecutive tokens tok0.. of
// this thread's channel ch.  The chunk's token scales are fetched once,
// coalesced (lane j holds sx[tok0 + j]), and broadcast by shuffle, so no
// store waits on a per-element scale load.  Every lane of the warp calls it
// (the shuffles are warp-wide); stores are predicated on ch_ok and tok < M.
template <int EPI, int NCOL>
__device__ __forceinline__ void epi_chunk(const uint32_t (&v)[NCOL], int tok0, int M, int ch,
                                          bool ch_ok, float swf, double ss,
                                          const float *__restrict__ sx, void *__restrict__ out,
                                          int ldo, int lane) {
    const int nvalid = (M - tok0) < NCOL ? (M - tok0) : NCOL;
    float sxl = 0.f;
    constexpr bool kTC = EPI == JTK_EPI_TOKEN_CHANNEL_F32 || EPI == JTK_EPI_TOKEN_CHANNEL_F32_ACC;
    if (kTC && lane < nvalid) sxl = __ldg(&sx[tok0 + lane]);
    const size_t base = static_cast<size_t>(tok0) * ldo + ch;
#pragma unroll
    for (int j = 0; j < NCOL; ++j) {
        const int32_t acc = static_cast<int32_t>(v[j]);
        const bool live = ch_ok && j < nvalid;
        const size_t o = base + static_cast<size_t>(j) * ldo;
        if (kTC) {
            const float sj = __shfl_sync(0xffffffffu, sxl, j);
            const float r = __fmul_rn(__fmul_rn(__int2float_rn(acc), sj), swf);
            if (live) {
                float *dst = static_cast<float *>(out) + o;
                // the add happens in L2 (no load to wait for); one writer per
                // element, so it is the same single rounding as *dst + r
                if (EPI == JTK_EPI_TOKEN_CHANNEL_F32_ACC)
                    atomicAdd(dst, r);
                else
                    *dst = r;
            }
        } else if (EPI == JTK_EPI_TENSOR_CHANNEL_F64) {
            if (live) static_cast<float *>(out)[o] = __double2float_rn(__dmul_rn((double)acc, ss));
        } else {
            if (live) static_cast<int32_t *>(out)[o] = acc;
        }
    }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    k_w8a8_gemm(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                int M, int N, int K, const float *__restrict__ sx, const float *__restrict__ sw,
                double sA, void *__restrict__ out, int ldo, int *err) {
    using Cfg = W8A8Cfg<BN>;
    constexpr int S = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + S * Cfg::kStage);
    uint64_t *empty = full + S;
    uint64_t *tfull = empty + S;
    uint64_t *tempty = tfull + 2;
    uint64_t *drain = tempty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = jt::warp_id();
    const int lane = jt::lane_id();
    const int n_ch_tiles = (N + kBM - 1) / kBM;
    const int n_tok_tiles = (M + BN - 1) / BN;
    const int ntiles = n_ch_tiles * n_tok_tiles;
    const int nk = (K + kBK - 1) / kBK;
    // programmatic dependent launch: the next kernel of the stream may start
    // its own set-up on the SMs this grid leaves free
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            jt::mbar_init(&full[s], 1);
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
        jt::prefetch_tmap(&tmW);
        jt::prefetch_tmap(&tmX);
        // the first tile's first S k-blocks into L2 while the previous
        // kernel of the stream may still run (a hint: the loads below still
        // wait for that kernel and read what it wrote)
        if (static_cast<int>(blockIdx.x) < ntiles) {
            const int n0 = (blockIdx.x % n_ch_tiles) * kBM, m0 = (blockIdx.x / n_ch_tiles) * BN;
            for (int kb = 0; kb < nk && kb < S; ++kb) {
                jt::prefetch_tile_2d(&tmW, kb * kBK, n0);
                jt::prefetch_tile_2d(&tmX, kb * kBK, m0);
            }
        }
    }
    if (warp == 1) {
        jt::tmem_alloc(tmem_slot, Cfg::kTmemCols);
        jt::tmem_relinquish();
    }
    jt::tc_fence_before();
    __syncthreads();
    jt::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // the set-up above touches no global memory; everything below may read
    // what the previous kernel of the stream wrote, so it waits for that
    // grid to complete
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (warp == 0) {
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            uint32_t issued_mask = 0, issued_phase = 0;  // per stage: ever issued / parity of last issue
            bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
                const int n0 = (tile % n_ch_tiles) * kBM;
                const int m0 = (tile / n_ch_tiles) * BN;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!jt::mbar_wait(&empty[stage], phase ^ 1u, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    uint8_t *sW = smem + stage * Cfg::kStage;
                    uint8_t *sX = sW + Cfg::kWBytes;
                    jt::mbar_arrive_expect_tx(&full[stage], Cfg::kStage);
                    jt::tma_load_2d(sW, &tmW, &full[stage], kb * kBK, n0);
                    jt::tma_load_2d(sX, &tmX, &full[stage], kb * kBK, m0);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // On abort every issued TMA box must still land before the CTA
            // exits: wait (bounded) for the last issued phase of each stage.
            if (!ok) {
                for (int s = 0; s < S; ++s) {
                    if (!(issued_mask & (1u << s))) continue;
                    const uint32_t par = (issued_phase >> s) & 1u;
                    const long long t0 = clock64();
                    while (!jt::mbar_try_wait(&full[s], par) &&
                           clock64() - t0 < JT_SPIN_CYCLES / 16) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t kIdesc = jt::idesc_i8(kBM, BN);
            uint32_t stage = 0, phase = 0;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
                const uint32_t buf = it & 1;
                const uint32_t use = (it >> 1) & 1;
                if (!jt::mbar_wait(&tempty[buf], use ^ 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                jt::tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * BN;
                for (int kb = 0; kb < nk; ++kb) {
                    if (!jt::mbar_wait(&full[stage], phase, abort_flag, err)) {
                        ok = false;
                        break;
                    }
                    jt::tc_fence_after();
                    const uint32_t aW = jt::smem_u32(smem + stage * Cfg::kStage);
                    const uint32_t aX = aW + Cfg::kWBytes;
                    const uint64_t da = jt::umma_desc_sw128(aW);
                    const uint64_t db = jt::umma_desc_sw128(aX);
#pragma unroll
                    for (int j = 0; j < kBK / 32; ++j) {
                        // advance 32 bytes along K inside the swizzle atom (2 x 16 B units)
                        jt::mma_i8(d_tmem, da + 2u * j, db + 2u * j, kIdesc,
                                   (kb | j) != 0 ? 1u : 0u);
                    }
                    jt::mma_commit(&empty[stage]);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                jt::mma_commit(&tfull[buf]);
            }
            if (!ok) {
                // Let already-issued MMAs retire before TMEM is released.
                jt::mma_commit(drain);
                const long long t0 = clock64();
                while (!jt::mbar_try_wait(drain, 0) && clock64() - t0 < JT_SPIN_CYCLES / 16) {
                }
            }
        }
    } else {
        // Epilogue warps 2..5: warp w may only touch TMEM lanes 32*(w%4)..+31.
        const int q = warp & 3;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
            const uint32_t buf = it & 1;
            const uint32_t use = (it >> 1) & 1;
            if (!jt::mbar_wait(&tfull[buf], use, abort_flag, err)) break;
            jt::tc_fence_after();
            const int n0 = (tile % n_ch_tiles) * kBM;
            const int m0 = (tile / n_ch_tiles) * BN;
            const int ch = n0 + q * 32 + lane;
            const bool ch_ok = ch < N;
            float swf = 0.f;
            double ss = 0.0;
            if (EPI == JTK_EPI_TOKEN_CHANNEL_F32 || EPI == JTK_EPI_TOKEN_CHANNEL_F32_ACC) swf = ch_ok ? sw[ch] : 0.f;
            if (EPI == JTK_EPI_TENSOR_CHANNEL_F64) ss = ch_ok ? sA * (double)sw[ch] : 0.0;
            const uint32_t trow = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
            const int cols = (M - m0) < BN ? (M - m0) : BN;
#pragma unroll 1
            for (int c0 = 0; c0 < cols; c0 += Cfg::kChunk) {
                uint32_t v[Cfg::kChunk];
                tmem_ld_chunk<Cfg::kChunk>(trow + c0, v);
                jt::tmem_wait_ld();
                epi_chunk<EPI, Cfg::kChunk>(v, m0 + c0, M, ch, ch_ok, swf, ss, sx, out, ldo, lane);
            }
            jt::tc_fence_before();
            __syncwarp();
            if (lane == 0) jt::mbar_arrive(&tempty[buf]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        jt::tc_fence_after();
        jt::tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair form for M >= 256: 256 weight channels x 256 tokens per 2-CTA
// cluster on the jt_pair.cuh pipeline (tcgen05 cta_group::2).  Rank r's
// weight box is channels n0 + 128r .. +127; its epilogue writes those
// channels for all 256 tokens of the tile.
constexpr size_t kPairSmem = 1024 + jt::pair::kRing + jt::pair::kBarBytes;

template <int EPI>
__global__ void __launch_bounds__(jt::pair::kThreads, 1)
    k_w8a8_pair(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                int M, int N, int K, const float *__restrict__ sx, const float *__restrict__ sw,
                double sA, void *__restrict__ out, int ldo, int *err) {
    namespace jp = jt::pair;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    jp::Ctx c;
    const CUtensorMap *maps[2] = {&tmW, &tmX};
    // programmatic dependent launch, as in k_w8a8_gemm: the set-up (no
    // global memory) overlaps the previous kernel, the rest waits for it
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    jp::setup(c, smem, smem + jp::kRing, err, maps, 2);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int n_ch_tiles = (N + 255) / 256;
    const int ntiles = n_ch_tiles * ((M + 255) / 256);
    const int nk = (K + kBK - 1) / kBK;

    if (c.warp == 0) {
        if (c.lane == 0)
            jp::producer(
                c, &tmX, ntiles, nk,
                [&](uint8_t *dst, int kb, int tile, uint32_t bar) {
                    jt::tma_load_2d_pair(dst, &tmW, bar, kb * kBK,
                                         (tile % n_ch_tiles) * 256 + static_cast<int>(c.rank) * 128);
                },
                [&](int tile) { return tile / n_ch_tiles; });
    } else if (c.warp == 1) {
        if (c.lane == 0 && c.rank == 0) jp::mma(c, ntiles, nk);
    } else {
        const int cl = (c.warp & 3) * 32 + c.lane;  // channel within this rank's 128
        const int colh = ((c.warp - 2) >> 2) * 128;
        int it = 0;
        for (int tile = c.pair; tile < ntiles; tile += c.npairs, ++it) {
            if (!jp::epi_acquire(c, it)) break;
            const int ch = (tile % n_ch_tiles) * 256 + static_cast<int>(c.rank) * 128 + cl;
            const int m0 = (tile / n_ch_tiles) * 256;
            const bool ch_ok = ch < N;
            float swf = 0.f;
            double ss = 0.0;
            if (EPI == JTK_EPI_TOKEN_CHANNEL_F32 || EPI == JTK_EPI_TOKEN_CHANNEL_F32_ACC) swf = ch_ok ? sw[ch] : 0.f;
            if (EPI == JTK_EPI_TENSOR_CHANNEL_F64) ss = ch_ok ? sA * (double)sw[ch] : 0.0;
            const int cols = (M - m0) < 256 ? (M - m0) : 256;
            const int ce = (colh + 128) < cols ? (colh + 128) : cols;
            jp::tmem_columns(jp::epi_row(c, it), colh, ce, [&](uint32_t(&v)[32], int c0) {
                epi_chunk<EPI, 32>(v, m0 + c0, M, ch, ch_ok, swf, ss, sx, out, ldo, c.lane);
            });
            jp::epi_release(c, it);
        }
    }
    jp::teardown(c);
}

template <int EPI>
int launch_pair(const CUtensorMap &tmW, const int8_t *X, int ldx, int M, int N, int K,
                const float *sx, const float *sw, double sA, void *out, int ldo,
                cudaStream_t stream) {
    CUtensorMap tmX;
    if (!jt::make_tmap_2d_u8(&tmX, X, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                             static_cast<uint64_t>(ldx), kBK, 128, true))
        return -2;
    auto kern = k_w8a8_pair<EPI>;
    static bool attr_done = false;  // per template instance
    if (!attr_done) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kPairSmem)) != cudaSuccess)
            return -3;
        attr_done = true;
    }
    const int ntiles = ((N + 255) / 256) * ((M + 255) / 256);
    int pairs = jtk_num_sms() / 2;
    if (pairs > ntiles) pairs = ntiles;
    cudaLaunchAttribute attr[2];
    cudaLaunchConfig_t cfg = jt::pair::launch_config(pairs, kPairSmem, stream, attr);
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, kern, tmW, tmX, M, N, K, sx, sw, sA, out, ldo, jtk_error_word()) !=
        cudaSuccess)
        return -4;
    return 0;
}

template <int BN, int EPI>
int launch_bn(const CUtensorMap &tmW, const int8_t *X, int ldx, int M, int N, int K,
              const float *sx, const float *sw, double sA, void *out, int ldo,
              cudaStream_t stream) {
    using Cfg = W8A8Cfg<BN>;
    CUtensorMap tmX;
    if (!jt::make_tmap_2d_u8(&tmX, X, static_cast<uint64_t>(K), static_cast<uint64_t>(M),
                             static_cast<uint64_t>(ldx), kBK, BN, true))
        return -2;
    auto kern = k_w8a8_gemm<BN, EPI>;
    static bool attr_done = false;  // per template instance
    if (!attr_done) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(Cfg::kSmem)) != cudaSuccess)
            return -3;
        attr_done = true;
    }
    const int ntiles = ((N + kBM - 1) / kBM) * ((M + BN - 1) / BN);
    int grid = jtk_num_sms();
    if (grid > ntiles) grid = ntiles;
    int *err = jtk_error_word();
    // launched with programmatic stream serialization: the kernel's set-up
    // (barriers, TMEM, descriptor prefetch) overlaps the previous kernel's
    // tail; it waits for that kernel before its first global access
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tmW, tmX, M, N, K, sx, sw, sA, out, ldo, err) != cudaSuccess) return -4;
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

template <int EPI>
int launch_epi(const int8_t *X, int ldx, const int8_t *W, int ldw, int M, int N, int K,
               const float *sx, const float *sw, double sA, void *out, int ldo,
               cudaStream_t stream) {
    CUtensorMap tmW;
    if (!jt::make_tmap_2d_u8(&tmW, W, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                             static_cast<uint64_t>(ldw), kBK, kBM, true))
        return -2;
    if (M <= 16) return launch_bn<16, EPI>(tmW, X, ldx, M, N, K, sx, sw, sA, out, ldo, stream);
    if (M <= 32) return launch_bn<32, EPI>(tmW, X, ldx, M, N, K, sx, sw, sA, out, ldo, stream);
    if (M <= 64) return launch_bn<64, EPI>(tmW, X, ldx, M, N, K, sx, sw, sA, out, ldo, stream);
    if (M <= 128) return launch_bn<128, EPI>(tmW, X, ldx, M, N, K, sx, sw, sA, out, ldo, stream);
    if (M < 256) return launch_bn<256, EPI>(tmW, X, ldx, M, N, K, sx, sw, sA, out, ldo, stream);
    return launch_pair<EPI>(tmW, X, ldx, M, N, K, sx, sw, sA, out, ldo, stream);
}

}  // namespace

extern "C" int jtk_w8a8_gemm(const int8_t *X, int ldx, const int8_t *W, int ldw, int M, int N,
                             int K, const float *sx, const float *sw, double sA, void *out,
                             int ldo, int epi, cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || (K % 16) != 0 || (ldx % 16) != 0 || (ldw % 16) != 0 ||
        ldx < K || ldw < K || ldo < N)
        return -1;
    switch (epi) {
        case JTK_EPI_TOKEN_CHANNEL_F32:
            if (!sx || !sw) return -1;
            return launch_epi<JTK_EPI_TOKEN_CHANNEL_F32>(X, ldx, W, ldw, M, N, K, sx, sw, sA, out,
                                                         ldo, stream);
        case JTK_EPI_TOKEN_CHANNEL_F32_ACC:
            if (!sx || !sw) return -1;
            return launch_epi<JTK_EPI_TOKEN_CHANNEL_F32_ACC>(X, ldx, W, ldw, M, N, K, sx, sw, sA, out,
                                                             ldo, stream);
        case JTK_EPI_TENSOR_CHANNEL_F64:
            if (!sw) return -1;
            return launch_epi<JTK_EPI_TENSOR_CHANNEL_F64>(X, ldx, W, ldw, M, N, K, sx, sw, sA,
                                                          out, ldo, stream);
        case JTK_EPI_RAW_I32:
            return launch_epi<JTK_EPI_RAW_I32>(X, ldx, W, ldw, M, N, K, sx, sw, sA, out, ldo,
                                               stream);
        default:
            return -1;
    }
}
