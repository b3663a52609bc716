// jt_gemv.cu - batch-1 low-bit GEMV: y[n] = sa * fold_g(P[n][g] * s[n][g])
// over INT2 and INT4 weight rows packed little-endian along K with one fp16
// scale per 64 K (the decode replacement of the reference's LUT path,
// lowbit.c:158-267 / tmac.c:387-506):
//   P[n][g] = sum_{k in group g} a[k] * c[n][k]   (int32, exact)
//   c = 2*li - (2^bits - 1)
//   r = 0; for g ascending: r = fmaf((float)P[n][g], s[n][g], r); y[n] = r * sa
//
// HBM-bound, every weight byte read once.  Two CTAs per SM, each with a
// producer warp that streams chunks of consecutive rows (up to 9 KB of
// codes and scales) into a 7-stage shared-memory ring with bulk
// asynchronous copies, so up to 129 KB per SM are in flight; seven consumer
// warps per CTA take the chunks in turn and, on the K = 2048 path, release
// a stage as soon as its codes and scales are copied out, so the refill
// streams while they compute.  Launched with programmatic
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
// The group partials go through shared memory (as exact fp32 on the
// K = 2048 path) so that the sequential fp32 fold runs lane-per-row.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

constexpr int kConsumers = 7;
constexpr int kThreads = (kConsumers + 1) * 32;
// One ring stage per consumer warp: stage i % kStages is always consumed by
// warp i % kConsumers, so each warp waits for every fill of its stage in
// order and the mbarrier phase parity is never ambiguous.
constexpr int kStages = kConsumers;
constexpr uint32_t kStageBytes = 9216;  // 16 INT2 or 8 INT4 rows of K = 2048 with their scales
constexpr int kMaxG = 64;  // K <= 4096
constexpr int kSub = 16;   // rows per fold batch

// shared memory: ring (codes, then the chunk's scales when they are copied
// too) | activation words [2 formats][kMaxG][16] | group sums [kMaxG] |
// partials per consumer [kSub][kPld] (32 groups per pass) | row scales per
// consumer, fp32 [kSub][kPld] (the K = 2048 path) | barriers
constexpr size_t kOffAct = (size_t)kStages * kStageBytes;
constexpr size_t kOffSum = kOffAct + 2 * kMaxG * 16 * 4;
constexpr size_t kOffP = kOffSum + kMaxG * 4;
constexpr int kPld = 36;  // partial-row stride (words): lane-per-row 16-byte reads without bank conflicts
constexpr size_t kOffS = kOffP + (size_t)kConsumers * kSub * kPld * 4;
constexpr size_t kOffBar = kOffS + (size_t)kConsumers * kSub * kPld * 4;
constexpr size_t kSmem = kOffBar + 2 * kStages * 8 + 16;
static_assert(kSmem <= 113 * 1024, "two CTAs per SM");

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
// The lane's codes of every row go to registers and the row scales of the
// fold, as fp32, to the warp's scale rows (Ss); then the stage is released
// (`empty`), so the producer refills it while this warp computes.  The
// partials are stored as fp32 (exact: |P| < 2^17) with every lane active:
// 0x4B400000 + P is the bit pattern of 1.5 * 2^23 + P for |P| < 2^22, and
// subtracting 1.5 * 2^23 leaves P, so the lane-per-row fold is FFMAs only.
template <int BITS, int R>
__device__ __forceinline__ void consume_k2048(const uint8_t *codes, int nrows, const uint32_t *act,
                                             const int *gsum, const uint16_t *sc, float sa, float *y,
                                             float *Ps, float *Ss, uint64_t *empty) {
    constexpr int kRowBytes = 2048 * BITS / 8;
    constexpr int kW = BITS / 2;  // 16-byte words per lane and row
    const int lane = jt::lane_id();
    uint4 q[R * kW];
    const uint8_t *base = codes + lane * (64 * BITS / 8);
#pragma unroll
    for (int rr = 0; rr < R; ++rr)
#pragma unroll
        for (int h = 0; h < kW; ++h) q[rr * kW + h] = *reinterpret_cast<const uint4 *>(base + rr * kRowBytes + 16 * h);
    // the R rows' 32 scales each, as fp32, to the scale rows (8 per step)
#pragma unroll
    for (int i = lane; i < R * 4; i += 32) {
        const uint4 v = reinterpret_cast<const uint4 *>(sc)[i];
        const uint32_t hv[4] = {v.x, v.y, v.z, v.w};
        float f[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h2;
            memcpy(&h2, &hv[j], 4);
            const float2 f2 = __half22float2(h2);
            f[2 * j] = f2.x;
            f[2 * j + 1] = f2.y;
        }
        float4 *dst = reinterpret_cast<float4 *>(Ss + (i / 4) * kPld + (i % 4) * 8);
        dst[0] = make_float4(f[0], f[1], f[2], f[3]);
        dst[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
    __syncwarp();
    if (lane == 0) jt::mbar_arrive(empty);
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
    // P = 2 sum(li a) - (2^BITS - 1) sum(a), carried as the biased pattern
    const int bias = 0x4B400000 - (BITS == 2 ? 3 : 15) * gsum[lane];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
        int p;
        if (BITS == 2) {
            const uint4 qq = q[rr * kW];
            const uint32_t w[4] = {qq.x, qq.y, qq.z, qq.w};
            int acc[4] = {0, 0, 0, 0};  // acc[j] = 4^j * sum(li_j * a)
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[j] = dp4a_us(w[i] & (0x03030303u << (2 * j)), ap[4 * i + j], acc[j]);
            p = 2 * ((acc[0] + (acc[1] >> 2)) + ((acc[2] >> 4) + (acc[3] >> 6))) + bias;
        } else {
            const uint4 q0 = q[rr * kW], q1 = q[rr * kW + kW - 1];
            const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
            int lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {  // hi = 16 * sum(li_odd * a)
                lo = dp4a_us(w[i] & 0x0F0F0F0Fu, ap[2 * i], lo);
                hi = dp4a_us(w[i] & 0xF0F0F0F0u, ap[2 * i + 1], hi);
            }
            p = 2 * (lo + (hi >> 4)) + bias;
        }
        Ps[rr * kPld + lane] = __fsub_rn(__int_as_float(p), 12582912.0f);
    }
    __syncwarp();
    if (lane < nrows) {
        // the row's 32 partials and 32 scales with 16-byte loads, then the
        // fold in ascending group order
        const float4 *pp = reinterpret_cast<const float4 *>(Ps + lane * kPld);
        const float4 *sp = reinterpret_cast<const float4 *>(Ss + lane * kPld);
        float r = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 pv = pp[i], sv = sp[i];
            r = __fmaf_rn(pv.x, sv.x, r);
            r = __fmaf_rn(pv.y, sv.y, r);
            r = __fmaf_rn(pv.z, sv.z, r);
            r = __fmaf_rn(pv.w, sv.w, r);
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
        // ---------------- consumers: chunk i of this CTA (stage i % kStages) goes to warp i % kConsumers
        // activation words permuted to the code order of the packed words:
        // INT2 word t = 4w + j of a group holds k = 16w + 4b + j at byte b;
        // INT4 word t = 2w + h holds k = 8w + h + 2b at byte b
        const int ct = threadIdx.x;  // consumer threads are 0..kConsumers*32-1
        // the activations (and y) may belong to the previous kernel of the
        // stream: wait for it here; the producer's weight copies (read-only
        // parameters) are already in flight
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // thread i: 16-byte segment i = quarter qd of group g, which holds
        // INT2 words 4 qd .. +3 (w = qd) and INT4 words 4 qd .. +3
        // (w = 2 qd, 2 qd + 1); the group sum from the four segments by
        // shuffles within the aligned lane quad (K / 16 is a multiple of 4
        // and so is the thread count, so a quad is always active together)
        for (int i = ct; i < K / 16; i += kConsumers * 32) {
            const uint4 v = __ldg(reinterpret_cast<const uint4 *>(a) + i);
            const int g = i >> 2, qd = i & 3;
            uint32_t w2[4], w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t sel = (uint32_t)j | ((4u + j) << 4);
                w2[j] = __byte_perm(__byte_perm(v.x, v.y, sel), __byte_perm(v.z, v.w, sel), 0x5410);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t sel = (uint32_t)h | ((2u + h) << 4) | ((4u + h) << 8) | ((6u + h) << 12);
                w4[h] = __byte_perm(v.x, v.y, sel);
                w4[2 + h] = __byte_perm(v.z, v.w, sel);
            }
            reinterpret_cast<uint4 *>(act + g * 16)[qd] = make_uint4(w2[0], w2[1], w2[2], w2[3]);
            reinterpret_cast<uint4 *>(act + kMaxG * 16 + g * 16)[qd] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            int sum = __dp4a((int)v.x, 0x01010101, __dp4a((int)v.y, 0x01010101,
                                                        __dp4a((int)v.z, 0x01010101, __dp4a((int)v.w, 0x01010101, 0))));
            const unsigned quad = 0xFu << (jt::lane_id() & ~3);
            sum += __shfl_xor_sync(quad, sum, 1);
            sum += __shfl_xor_sync(quad, sum, 2);
            if (qd == 0) gsum[g] = sum;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32) : "memory");
        int32_t *Ps = reinterpret_cast<int32_t *>(smem + kOffP) + warp * kSub * kPld;
        float *Pf = reinterpret_cast<float *>(Ps);  // the K = 2048 path's fp32 partials
        float *Ss = reinterpret_cast<float *>(smem + kOffS) + warp * kSub * kPld;
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
                if (K == 2048 && sb && cr2 == 16) {
                    consume_k2048<2, 16>(codes, ch.nrows, act, gsum, sc, sa, y + ch.row0, Pf, Ss, &empty[st]);
                    continue;
                }
                consume<2>(codes, ch.nrows, K, act, gsum, sc, sa, y + ch.row0, Ps);
            } else {
                ch.nrows = min(cr4, n4 - ch.row0);
                const uint16_t *sc = sb ? reinterpret_cast<const uint16_t *>(codes + cr4 * rb4)
                                        : s4 + (size_t)ch.row0 * G;
                if (K == 2048 && sb && cr4 == 8) {
                    consume_k2048<4, 8>(codes, ch.nrows, act, gsum, sc, sa, y + n2 + ch.row0, Pf, Ss, &empty[st]);
                    continue;
                }
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
