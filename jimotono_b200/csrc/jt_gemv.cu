// jt_gemv.cu - batch-1 low-bit GEMV: y[n] = sa * fold_g(P[n][g] * s[n][g])
// over INT2 and INT4 weight rows packed little-endian along K with one fp16
// scale per 64 K (the decode replacement of the reference's LUT path,
// lowbit.c:158-267 / tmac.c:387-506):
//   P[n][g] = sum_{k in group g} a[k] * c[n][k]   (int32, exact)
//   c = 2*li - (2^bits - 1)
//   r = 0; for g ascending: r = fmaf((float)P[n][g], s[n][g], r); y[n] = r * sa
//
// HBM-bound, every weight byte read once.  Two CTAs per SM, each with a
// producer warp that streams chunks of consecutive rows (up to 10 KB of
// codes and scales) into an 8-stage shared-memory ring with bulk
// asynchronous copies, so up to 160 KB per SM are in flight; eight consumer
// warps per CTA take the chunks in turn.  Launched with programmatic
// dependent launch: a GEMV queued behind another kernel starts streaming its
// weights while that kernel drains, and waits for it only before reading the
// activations and writing y.  The weight and scale buffers must therefore
// not be written by work still running in the same stream (they are model
// parameters).  In a
// chunk, lane l owns 64-K group l of each row, masks the code bits of four K
// positions per byte lane in place (one logic op) and feeds them to an
// unsigned x signed dp4a against activation words permuted to match (built
// once per CTA); code j of a byte then carries a factor 4^j (INT2) or 16
// (INT4 high nibble), removed exactly by an arithmetic shift of its own
// accumulator:
//   P = 2 * sum(li * a) - (2^bits - 1) * sum(a)   (exact in int32).
// The group partials go through shared memory so that the sequential fp32
// fold runs lane-per-row.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

constexpr int kConsumers = 8;
constexpr int kThreads = (kConsumers + 1) * 32;
// One ring stage per consumer warp: stage i % 8 is always consumed by warp
// i % 8, so each warp waits for every fill of its stage in order and the
// mbarrier phase parity is never ambiguous.
constexpr int kStages = kConsumers;
constexpr uint32_t kStageBytes = 10240;
constexpr int kMaxG = 64;  // K <= 4096
constexpr int kSub = 16;   // rows per fold batch

// shared memory: ring (codes, then the chunk's scales when they are copied
// too) | activation words [2 formats][kMaxG][16] | group sums [kMaxG] |
// activations [K] | partials per consumer [kSub][33] (32 groups per pass) |
// barriers
constexpr size_t kOffAct = (size_t)kStages * kStageBytes;
constexpr size_t kOffSum = kOffAct + 2 * kMaxG * 16 * 4;
constexpr size_t kOffA = kOffSum + kMaxG * 4;          // activations, K bytes
constexpr size_t kOffP = kOffA + 64 * kMaxG;
constexpr int kPld = 36;  // partial-row stride (words): lane-per-row 16-byte reads without bank conflicts
constexpr size_t kOffBar = kOffP + (size_t)kConsumers * kSub * kPld * 4;
constexpr size_t kSmem = kOffBar + 2 * kStages * 8 + 16;
static_assert(kSmem <= 113 * 1024, "two CTAs per SM");

__device__ __forceinline__ uint32_t ubyte(const int8_t *a, int k) {
    return static_cast<uint32_t>(static_cast<uint8_t>(a[k]));
}

// Rows per chunk: as many as fit in a stage (codes + optional scales), a
// multiple of 8 when at least 8 fit, at most 64.
__host__ __device__ __forceinline__ int chunk_rows(int bytes_per_row) {
    int r = (int)(kStageBytes / (uint32_t)bytes_per_row);
    if (r >= 8) r &= ~7;
    return r < 1 ? 1 : (r > 64 ? 64 : r);
}

struct Chunk {
    int bits, row0, nrows;  // rows [row0, row0 + nrows) of segment `bits`
};

// Chunk c of the job: the INT2 segment first, then the INT4 segment.
__device__ __forceinline__ Chunk chunk_of(int c, int n2, int cr2, int c2, int cr4) {
    Chunk ch;
    if (c < c2) {
        ch.bits = 2;
        ch.row0 = c * cr2;
        ch.nrows = min(cr2, n2 - ch.row0);
    } else {
        ch.bits = 4;
        ch.row0 = (c - c2) * cr4;
        ch.nrows = cr4;  // clipped by the caller
    }
    return ch;
}

__device__ __forceinline__ int dp4a_us(uint32_t u, uint32_t s, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(u), "r"(s), "r"(c));
    return d;
}

template <int BITS>
__device__ __forceinline__ int group_partial(const uint8_t *codes, const uint32_t *ap, int asum) {
    if (BITS == 2) {
        const uint4 q = *reinterpret_cast<const uint4 *>(codes);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        int acc[4] = {0, 0, 0, 0};  // acc[j] = 4^j * sum(li_j * a)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] = dp4a_us(w[i] & (0x03030303u << (2 * j)), ap[4 * i + j], acc[j]);
        const int sum = acc[0] + (acc[1] >> 2) + (acc[2] >> 4) + (acc[3] >> 6);
        return 2 * sum - 3 * asum;
    } else {
        const uint4 q0 = *reinterpret_cast<const uint4 *>(codes);
        const uint4 q1 = *reinterpret_cast<const uint4 *>(codes + 16);
        const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        int lo = 0, hi = 0;  // hi = 16 * sum(li_odd * a)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo = dp4a_us(w[i] & 0x0F0F0F0Fu, ap[2 * i], lo);
            hi = dp4a_us(w[i] & 0xF0F0F0F0u, ap[2 * i + 1], hi);
        }
        return 2 * (lo + (hi >> 4)) - 15 * asum;
    }
}

// Specialization for K = 2048 (32 groups, lane = group) with the chunk's
// scales in shared memory: all R rows of the stage are processed with fixed
// trip counts (rows past nrows hold stale bytes and are not stored), the
// codes are masked in place into four (INT2) or two (INT4) independent
// unsigned x signed dp4a chains whose 4^j / 16 factors are shifted out.
template <int BITS, int R>
__device__ __forceinline__ void consume_k2048(const uint8_t *codes, int nrows, const uint32_t *act,
                                             const int *gsum, const uint16_t *sc, float sa, float *y,
                                             int32_t *Ps) {
    constexpr int kRowBytes = 2048 * BITS / 8;
    const int lane = jt::lane_id();
    const uint4 *a4 = reinterpret_cast<const uint4 *>(act + (BITS == 2 ? 0 : kMaxG * 16) + lane * 16);
    uint32_t ap[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = a4[i];
        ap[4 * i] = v.x;
        ap[4 * i + 1] = v.y;
        ap[4 * i + 2] = v.z;
        ap[4 * i + 3] = v.w;
    }
    const int asum = gsum[lane];
    const uint8_t *base = codes + lane * (64 * BITS / 8);
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        int p;
        if (BITS == 2) {
            const uint4 q = *reinterpret_cast<const uint4 *>(base + rr * kRowBytes);
            const uint32_t w[4] = {q.x, q.y, q.z, q.w};
            int acc[4] = {0, 0, 0, 0};  // acc[j] = 4^j * sum(li_j * a)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[j] = dp4a_us(w[i] & (0x03030303u << (2 * j)), ap[4 * i + j], acc[j]);
            p = 2 * ((acc[0] + (acc[1] >> 2)) + ((acc[2] >> 4) + (acc[3] >> 6))) - 3 * asum;
        } else {
            const uint4 q0 = *reinterpret_cast<const uint4 *>(base + rr * kRowBytes);
            const uint4 q1 = *reinterpret_cast<const uint4 *>(base + rr * kRowBytes + 16);
            const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {  // hi = 16 * sum(li_odd * a)
                lo = dp4a_us(w[i] & 0x0F0F0F0Fu, ap[2 * i], lo);
                hi = dp4a_us(w[i] & 0xF0F0F0F0u, ap[2 * i + 1], hi);
            }
            p = 2 * (lo + (hi >> 4)) - 15 * asum;
        }
        Ps[rr * kPld + lane] = p;
    }
    __syncwarp();
    if (lane < nrows) {
        // the row's 32 partials and 32 fp16 scales with 16-byte loads, then
        // the fold in ascending group order
        const uint4 *pp = reinterpret_cast<const uint4 *>(Ps + lane * kPld);
        const uint4 *sp = reinterpret_cast<const uint4 *>(sc + lane * 32);
        int32_t P[32];
        uint32_t hs[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint4 v = pp[i];
            P[4 * i] = (int32_t)v.x;
            P[4 * i + 1] = (int32_t)v.y;
            P[4 * i + 2] = (int32_t)v.z;
            P[4 * i + 3] = (int32_t)v.w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = sp[i];
            hs[4 * i] = v.x;
            hs[4 * i + 1] = v.y;
            hs[4 * i + 2] = v.z;
            hs[4 * i + 3] = v.w;
        }
        float r = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {  // two scales per conversion (low half = even group)
            __half2 h2;
            memcpy(&h2, &hs[i], 4);
            const float2 s2 = __half22float2(h2);
            r = __fmaf_rn((float)P[2 * i], s2.x, r);
            r = __fmaf_rn((float)P[2 * i + 1], s2.y, r);
        }
        y[lane] = __fmul_rn(r, sa);
    }
    __syncwarp();
}

// Rows [0, nrows) of one chunk in shared memory -> y.  Groups are taken 32
// at a time (lane = group); each pass's partials are folded lane-per-row
// into r, so the fold still runs over the groups in ascending order.
template <int BITS>
__device__ __forceinline__ void consume(const uint8_t *codes, int nrows, int K, const uint32_t *act,
                                       const int *gsum, const uint16_t *s, float sa, float *y,
                                       int32_t *Ps) {
    // s: the chunk's scales [nrows][G], in shared memory or in global memory
    const int lane = jt::lane_id();
    const int G = K / 64;
    const int rowbytes = K * BITS / 8;
    const uint32_t *actb = act + (BITS == 2 ? 0 : kMaxG * 16);
    for (int r0 = 0; r0 < nrows; r0 += kSub) {
        const int nr = min(kSub, nrows - r0);
        // 16-bit scale loads: a row's scales are only 2-byte aligned for odd G
        const uint16_t *sr = s + (size_t)(r0 + lane) * G;
        float r = 0.0f;
        for (int gp = 0; gp < G; gp += 32) {
            const int gc = min(32, G - gp);
            if (lane < gc) {
                const int g = gp + lane;
                uint32_t ap[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) ap[i] = actb[g * 16 + i];
                const int asum = gsum[g];
                const uint8_t *base = codes + (size_t)r0 * rowbytes + g * (64 * BITS / 8);
#pragma unroll 4
                for (int rr = 0; rr < nr; ++rr) Ps[rr * kPld + lane] = group_partial<BITS>(base + rr * rowbytes, ap, asum);
            }
            __syncwarp();
            if (lane < nr)
                for (int g = 0; g < gc; ++g)
                    r = __fmaf_rn((float)Ps[lane * kPld + g], __half2float(__ushort_as_half(sr[gp + g])), r);
            __syncwarp();
        }
        if (lane < nr) y[r0 + lane] = __fmul_rn(r, sa);
    }
}

__global__ void __launch_bounds__(kThreads, 2)
    k_lowbit_gemv(const int8_t *__restrict__ a, float sa, const uint8_t *__restrict__ w2,
                  const uint16_t *__restrict__ s2, int n2, const uint8_t *__restrict__ w4,
                  const uint16_t *__restrict__ s4, int n4, int K, int sbulk, float *__restrict__ y,
                  int *err) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint32_t *act = reinterpret_cast<uint32_t *>(smem + kOffAct);
    int *gsum = reinterpret_cast<int *>(smem + kOffSum);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t *empty = full + kStages;
    int *abort_flag = reinterpret_cast<int *>(empty + kStages);
    const int warp = jt::warp_id(), lane = jt::lane_id();
    const int G = K / 64;
    const int rb2 = K / 4, rb4 = K / 2;
    const int sb = sbulk ? 2 * G : 0;  // scale bytes per row copied with the codes
    const int cr2 = chunk_rows(rb2 + sb), cr4 = chunk_rows(rb4 + sb);  // rows per chunk
    const int c2 = (n2 + cr2 - 1) / cr2, c4 = (n4 + cr4 - 1) / cr4;
    const int nchunks = c2 + c4;

    // programmatic dependent launch: let the next kernel of the stream be
    // scheduled as our CTAs retire
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            jt::mbar_init(&full[s], 1);
            jt::mbar_init(&empty[s], 1);
        }
        *abort_flag = 0;
        jt::fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---------------- producer: one lane issues the bulk copies
        if (lane == 0) {
            uint32_t issued = 0, issued_ph = 0;
            int i = 0;
            bool ok = true;
            for (int c = blockIdx.x; c < nchunks; c += gridDim.x, ++i) {
                const int st = i % kStages;
                const uint32_t use = i / kStages;
                if (use > 0 && !jt::mbar_wait(&empty[st], (use - 1) & 1u, abort_flag, err)) {
                    ok = false;
                    break;
                }
                Chunk ch = chunk_of(c, n2, cr2, c2, cr4);
                if (ch.bits == 4) ch.nrows = min(cr4, n4 - ch.row0);
                const int rb = ch.bits == 2 ? rb2 : rb4;
                const uint8_t *src = (ch.bits == 2 ? w2 : w4) + (size_t)ch.row0 * rb;
                const uint32_t bytes = (uint32_t)(ch.nrows * rb);
                const uint32_t sbytes = (uint32_t)(ch.nrows * sb);
                uint8_t *dst = smem + (size_t)st * kStageBytes;
                jt::mbar_arrive_expect_tx(&full[st], bytes + sbytes);
                jt::bulk_load(dst, src, bytes, &full[st]);
                if (sbytes) {
                    const uint16_t *ssrc = (ch.bits == 2 ? s2 : s4) + (size_t)ch.row0 * G;
                    jt::bulk_load(dst + (ch.bits == 2 ? cr2 : cr4) * rb, ssrc, sbytes, &full[st]);
                }
                issued |= 1u << st;
                issued_ph = (issued_ph & ~(1u << st)) | ((use & 1u) << st);
            }
            if (!ok) {  // issued copies land before the CTA exits
                for (int s = 0; s < kStages; ++s) {
                    if (!(issued & (1u << s))) continue;
                    const long long t0 = clock64();
                    while (!jt::mbar_try_wait(&full[s], (issued_ph >> s) & 1u) &&
                           clock64() - t0 < JT_SPIN_CYCLES / 16) {
                    }
                }
            }
        }
    } else {
        // ---------------- consumers: chunk i of this CTA (stage i % 8) goes to warp i % 8
        // activation words permuted to the code order of the packed words
        // (built while the producer's first copies are in flight):
        // INT2 word w of a group holds k = 16w + 4b + j at bits 2j of byte b;
        // INT4 word w holds k = 8w + 2b (low nibble) and 8w + 2b + 1 (high)
        const int ct = threadIdx.x;  // consumer threads are 0..kConsumers*32-1
        // the activations (and y) may belong to the previous kernel of the
        // stream: wait for it here; the producer's weight copies (read-only
        // parameters) are already in flight
        asm volatile("griddepcontrol.wait;" ::: "memory");
        int8_t *as = reinterpret_cast<int8_t *>(smem + kOffA);
        for (int i = ct; i < K / 16; i += kConsumers * 32)
            reinterpret_cast<uint4 *>(as)[i] = __ldg(reinterpret_cast<const uint4 *>(a) + i);
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
        a = as;
        for (int i = ct; i < G * 16; i += kConsumers * 32) {
            const int g = i / 16, t = i % 16;
            const int k0 = 64 * g;
            {  // INT2: t = 4w + j
                const int b0 = k0 + 16 * (t / 4) + (t % 4);
                act[g * 16 + t] = ubyte(a, b0) | (ubyte(a, b0 + 4) << 8) | (ubyte(a, b0 + 8) << 16) | (ubyte(a, b0 + 12) << 24);
            }
            {  // INT4: t = 2w + h
                const int b0 = k0 + 8 * (t / 2) + (t % 2);
                act[kMaxG * 16 + g * 16 + t] =
                    ubyte(a, b0) | (ubyte(a, b0 + 2) << 8) | (ubyte(a, b0 + 4) << 16) | (ubyte(a, b0 + 6) << 24);
            }
        }
        for (int g = ct; g < G; g += kConsumers * 32) {
            int sum = 0;
#pragma unroll 8
            for (int i = 0; i < 64; ++i) sum += a[64 * g + i];
            gsum[g] = sum;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
        int32_t *Ps = reinterpret_cast<int32_t *>(smem + kOffP) + warp * kSub * kPld;
        int i = 0;
        for (int c = blockIdx.x; c < nchunks; c += gridDim.x, ++i) {
            if (i % kConsumers != warp) continue;
            const int st = i % kStages;
            const uint32_t use = i / kStages;
            if (!jt::mbar_wait(&full[st], use & 1u, abort_flag, err)) break;
            Chunk ch = chunk_of(c, n2, cr2, c2, cr4);
            const uint8_t *codes = smem + (size_t)st * kStageBytes;
            if (ch.bits == 2) {
                const uint16_t *sc = sb ? reinterpret_cast<const uint16_t *>(codes + cr2 * rb2)
                                        : s2 + (size_t)ch.row0 * G;
                if (K == 2048 && sb && cr2 == 16)
                    consume_k2048<2, 16>(codes, ch.nrows, act, gsum, sc, sa, y + ch.row0, Ps);
                else
                    consume<2>(codes, ch.nrows, K, act, gsum, sc, sa, y + ch.row0, Ps);
            } else {
                ch.nrows = min(cr4, n4 - ch.row0);
                const uint16_t *sc = sb ? reinterpret_cast<const uint16_t *>(codes + cr4 * rb4)
                                        : s4 + (size_t)ch.row0 * G;
                if (K == 2048 && sb && cr4 == 8)
                    consume_k2048<4, 8>(codes, ch.nrows, act, gsum, sc, sa, y + n2 + ch.row0, Ps);
                else
                    consume<4>(codes, ch.nrows, K, act, gsum, sc, sa, y + n2 + ch.row0, Ps);
            }
            __syncwarp();
            if (lane == 0) jt::mbar_arrive(&empty[st]);
        }
    }
}

}  // namespace

// y[0..n2) from the INT2 rows, y[n2..n2+n4) from the INT4 rows.  K % 64 == 0,
// K <= 4096, packed rows 16-byte aligned (K/4 and K/2 bytes per row).
extern "C" int jtk_lowbit_gemv(const int8_t *a, float sa, const uint8_t *w2, const uint16_t *s2,
                               int n2, const uint8_t *w4, const uint16_t *s4, int n4, int K,
                               float *y, cudaStream_t stream) {
    if (K <= 0 || K % 64 || K / 64 > kMaxG || n2 < 0 || n4 < 0 || (n2 > 0 && (!w2 || !s2)) ||
        (n4 > 0 && (!w4 || !s4)) || !a || !y)
        return -1;
    if (n2 + n4 == 0) return 0;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_lowbit_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) !=
            cudaSuccess)
            return -3;
        attr = true;
    }
    const int G = K / 64;
    // the scales travel with the codes when every chunk's scale block is a
    // whole number of 16-byte units starting on a 16-byte boundary
    const int sbulk = (G % 8 == 0) && (((uintptr_t)s2 | (uintptr_t)s4) & 15u) == 0;
    const int sb = sbulk ? 2 * G : 0;
    const int cr2 = chunk_rows(K / 4 + sb), cr4 = chunk_rows(K / 2 + sb);
    const int chunks = (n2 + cr2 - 1) / cr2 + (n4 + cr4 - 1) / cr4;
    int grid = 2 * jtk_num_sms();
    if (grid > chunks) grid = chunks;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr_pdl[1];
    attr_pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr_pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr_pdl;
    cfg.numAttrs = 1;
    int *errw = jtk_error_word();
    if (cudaLaunchKernelEx(&cfg, k_lowbit_gemv, a, sa, w2, s2, n2, w4, s4, n4, K, sbulk, y, errw) !=
        cudaSuccess)
        return -4;
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
