// jt_compat.cu - kernels behind the remaining reference-compatible host
// entry points (jt_api_compat.c): single-token top-k + softmax of any k,
// the exact fp32 GEMM / transpose of moe_gemm.c, and the low-bit level rule
// of lowbit.c (fake-quant values and bit-plane codes), and the T-MAC
// activation table, lookup and LUT GEMM of tmac.c / lowbit.c.  All arithmetic is
// the reference's: sequential k-order fp32 sums without fusion, double
// precision where the reference uses double.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"

namespace {

// ---------------------------------------------------------------- top-k
// One CTA: k passes of a block-wide (value, index) argmax over logits[0..n)
// with the selection rule of routing.c:38-52 (first index seeds `best`,
// then strictly greater values replace it, so ties go to the lowest index
// and taken entries count as -inf).  Then the softmax of routing.c:54-73 by
// thread 0: float max, double exp sum, w = (float)e * (float)(1/sum).
// flag[0] = 1 when the softmax sum is not finite and positive.  One CTA
// per token (blockIdx.x): logits [T][n], taken [T][ceil(n/32)], ids / w [T][k].
__global__ void __launch_bounds__(1024) k_topk_any(const float *__restrict__ logits, int n, int k,
                                                   uint32_t *__restrict__ taken, int32_t *__restrict__ ids,
                                                   float *__restrict__ w, int *flag) {
    __shared__ float sv[32];
    __shared__ int si[32];
    logits += (size_t)blockIdx.x * n;
    taken += (size_t)blockIdx.x * ((n + 31) / 32);
    ids += (size_t)blockIdx.x * k;
    w += (size_t)blockIdx.x * k;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int i = threadIdx.x; i < (n + 31) / 32; i += blockDim.x) taken[i] = 0;
    __syncthreads();
    for (int p = 0; p < k; ++p) {
        // per thread: best over its strided elements, "unset" = index n
        float bv = 0.0f;
        int bi = n;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const bool tk = (taken[i >> 5] >> (i & 31)) & 1u;
            const float v = tk ? -INFINITY : logits[i];
            if (bi == n || v > bv) {
                bv = v;
                bi = i;
            }
        }
        // combine candidates in index order semantics: a candidate (v, i)
        // wins over (v2, i2) when v > v2, or v == v2 and i < i2 (what the
        // sequential scan yields); an unset candidate never wins
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != n && (bi == n || ov > bv || (ov == bv && oi < bi))) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            sv[wid] = bv;
            si[wid] = bi;
        }
        __syncthreads();
        if (wid == 0) {
            bv = lane < nw ? sv[lane] : 0.0f;
            bi = lane < nw ? si[lane] : n;
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi != n && (bi == n || ov > bv || (ov == bv && oi < bi))) {
                    bv = ov;
                    bi = oi;
                }
            }
            if (lane == 0) {
                ids[p] = bi;
                taken[bi >> 5] |= 1u << (bi & 31);
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float mx = logits[ids[0]];
        for (int p = 1; p < k; ++p) {
            const float v = logits[ids[p]];
            mx = v > mx ? v : mx;
        }
        double sum = 0.0;
        for (int p = 0; p < k; ++p) {
            const double e = exp((double)logits[ids[p]] - (double)mx);
            sum += e;
            w[p] = (float)e;
        }
        if (!(sum > 0.0) || !isfinite(sum)) {
            flag[0] = 1;
            return;
        }
        const float inv = (float)(1.0 / sum);
        for (int p = 0; p < k; ++p) w[p] = __fmul_rn(w[p], inv);
    }
}

// ---------------------------------------------------------------- fp32 GEMM
// C[m][n] = sum_k A[m][k] * B[k][n] in ascending k, one rounding per
// multiply and per add (moe_gemm.c:44-170: no fused multiply-add).
__global__ void k_gemm_f32_seq(const float *__restrict__ A, const float *__restrict__ B,
                               float *__restrict__ C, int M, int N, int K) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (n >= N || m >= M) return;
    const float *a = A + (size_t)m * K;
    float acc = 0.0f;
    for (int kk = 0; kk < K; ++kk) acc = __fadd_rn(acc, __fmul_rn(a[kk], B[(size_t)kk * N + n]));
    C[(size_t)m * N + n] = acc;
}

__global__ void k_transpose_f32(const float *__restrict__ src, float *__restrict__ dst, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c = blockIdx.x * 32 + threadIdx.x, r = blockIdx.y * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (r + j < rows && c < cols) tile[threadIdx.y + j][threadIdx.x] = src[(size_t)(r + j) * cols + c];
    __syncthreads();
    const int c2 = blockIdx.y * 32 + threadIdx.x, r2 = blockIdx.x * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (r2 + j < cols && c2 < rows) dst[(size_t)(r2 + j) * rows + c2] = tile[threadIdx.x][threadIdx.y + j];
}

// ---------------------------------------------------------------- low-bit
// max |w| in double over n values (positive doubles order like their bits),
// bad = 1 on a non-finite value.
__global__ void k_absmax_d(const float *__restrict__ w, size_t n, unsigned long long *maxbits, int *bad) {
    double m = 0.0;
    int nf = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const double v = (double)w[i];
        nf |= !isfinite(v);
        m = fmax(m, fabs(v));
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        nf |= __shfl_xor_sync(0xffffffffu, nf, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(maxbits, (unsigned long long)__double_as_longlong(m));
        if (nf) atomicExch(bad, 1);
    }
}

// level index of lowbit.c:78-88: t = w / maxa (double), li = floor(t(n-1)/2
// + (n-1)/2 + 0.5) clamped to [0, n-1]
__device__ __forceinline__ int level(float wv, double maxa, int nl) {
    const double t = maxa == 0.0 ? 0.0 : __ddiv_rn((double)wv, maxa);
    const double li = floor(__dadd_rn(__dadd_rn(__ddiv_rn(__dmul_rn(t, (double)(nl - 1)), 2.0),
                                                 (double)(nl - 1) / 2.0),
                                      0.5));
    long l = (long)li;
    l = l < 0 ? 0 : l;
    l = l > nl - 1 ? nl - 1 : l;
    return (int)l;
}

// fq[i] = (float)(((2li - (n-1)) / (n-1)) * maxa), all-zero input -> 0
__global__ void k_lowbit_fq(const float *__restrict__ w, size_t n, int bits,
                            const unsigned long long *maxbits, float *__restrict__ fq) {
    const double maxa = __longlong_as_double((long long)*maxbits);
    const int nl = 1 << bits;
    const double nd = (double)(nl - 1);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        if (maxa == 0.0) {
            fq[i] = 0.0f;
            continue;
        }
        const int l = level(w[i], maxa, nl);
        const double lv = __ddiv_rn(__dsub_rn(2.0 * (double)l, nd), nd);
        fq[i] = (float)__dmul_rn(lv, maxa);
    }
}

// bit planes of lowbit.c:117-137: idx[b*(k/4) + g] bit j = bit b of li(4g+j)
__global__ void k_lowbit_idx(const float *__restrict__ col, size_t k, int bits,
                             const unsigned long long *maxbits, uint8_t *__restrict__ idx) {
    const double maxa = __longlong_as_double((long long)*maxbits);
    const int nl = 1 << bits;
    const size_t ng = k / 4;
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < ng; g += (size_t)gridDim.x * blockDim.x) {
        int li[4];
        for (int j = 0; j < 4; ++j) li[j] = level(col[g * 4 + j], maxa, nl);
        for (int b = 0; b < bits; ++b) {
            unsigned p = 0;
            for (int j = 0; j < 4; ++j)
                if (((unsigned)li[j] >> b) & 1u) p |= 1u << j;
            idx[(size_t)b * ng + g] = (uint8_t)p;
        }
    }
}

// ---------------------------------------------------------------- T-MAC LUT
// Error keys: the reference stops at its first failure, so every thread that
// fails posts (position << 1 | kind) with atomicMin and the host reads the
// smallest one (all ones = no error).  kind 0 = EINVAL, 1 = ERANGE.

// One thread per (row, 32-activation block) of tmac.c:274-376.  Patterns p
// of a 4-activation group: F(p) = sum_j (bit j of p ? +a_j : -a_j), summed
// in double in ascending j.  F(15-p) is the exact negation of F(p) (every
// partial sum flips sign and round-to-nearest is symmetric), so the maximum
// |F| over the 16 patterns is the maximum over p = 8..15, and the stored
// half-table holds q(p) for p = 8..15.
__global__ void k_tmac_ctor(const float *__restrict__ act, size_t nrows, size_t k, int8_t *__restrict__ qlut,
                            float *__restrict__ scales, float *__restrict__ biases,
                            unsigned long long *__restrict__ err) {
    const size_t nb = k / 32;
    const size_t L = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (L >= nrows * nb) return;
    const size_t r = L / nb, bb = L % nb;
    const float4 *src = reinterpret_cast<const float4 *>(act + r * k + bb * 32);
    float a[32];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = src[i];
        a[4 * i] = v.x;
        a[4 * i + 1] = v.y;
        a[4 * i + 2] = v.z;
        a[4 * i + 3] = v.w;
    }
    bool fin = true;
#pragma unroll
    for (int i = 0; i < 32; ++i) fin &= isfinite(a[i]);
    if (!fin) {
        atomicMin(err, (unsigned long long)L << 1);
        return;
    }
    double F[8][8];
    double maxabs = 0.0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
#pragma unroll
        for (int ii = 0; ii < 8; ++ii) {
            const int p = 8 + ii;
            double s = 0.0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const double av = (double)a[4 * g + j];
                s = __dadd_rn(s, ((p >> j) & 1) ? av : -av);
            }
            F[g][ii] = s;
            maxabs = fmax(maxabs, fabs(s));
        }
    }
    double asum = 0.0;
#pragma unroll
    for (int i = 0; i < 32; ++i) asum = __dadd_rn(asum, (double)a[i]);
    const float bias_f = (float)asum;
    if (!isfinite(bias_f)) {
        atomicMin(err, ((unsigned long long)L << 1) | 1ull);
        return;
    }
    uint32_t w[16];
    float scale_f = 1.0f;
    if (maxabs == 0.0) {
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = 0;
    } else {
        const double scale_d = __ddiv_rn(maxabs, 127.0);
        scale_f = (float)scale_d;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t word = 0;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    double qd = round(__ddiv_rn(F[g][4 * h + b], scale_d));
                    qd = qd > 127.0 ? 127.0 : (qd < -128.0 ? -128.0 : qd);
                    word |= ((uint32_t)(int)qd & 0xffu) << (8 * b);
                }
                w[2 * g + h] = word;
            }
        }
    }
    uint4 *dst = reinterpret_cast<uint4 *>(qlut + L * 64);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    scales[L] = scale_f;
    biases[L] = bias_f;
}

// plane_acc of tmac.c:80-93 over one block: nibble p of group g selects
// +q[g][p-8] (p >= 8) or -q[g][7-p] (p < 8); q8 holds the block's 64 bytes
// as 16 words and idx8 the block's 8 index bytes (low nibble used).
__device__ __forceinline__ int tmac_plane(const uint32_t (&q8)[16], uint2 idx8) {
    int acc = 0;
#pragma unroll
    for (int g = 0; g < 8; ++g) {
        const uint32_t byte = ((g < 4 ? idx8.x : idx8.y) >> (8 * (g & 3))) & 0xfu;
        const uint32_t hi = byte >> 3;                      // 1: p >= 8
        const uint32_t sel = (byte & 7u) ^ (hi ? 0u : 7u);  // p-8 or 7-p
        const uint32_t v = __byte_perm(q8[2 * g], q8[2 * g + 1], sel);
        const int qv = (int)(int8_t)(v & 0xffu);
        acc += hi ? qv : -qv;
    }
    return acc;
}

// ((sc*acc + bi)*0.5)*2^b, each operation rounded (tmac.c:482-487, no FMA)
__device__ __forceinline__ double tmac_contrib(double sc, double bi, int acc, int b) {
    return __dmul_rn(__dmul_rn(__dadd_rn(__dmul_rn(sc, (double)acc), bi), 0.5), (double)(1 << b));
}

// One dot product of tmac.c:387-506.  flag: 1 = a non-finite scale/bias
// (EINVAL), 2 = non-finite total or float result (ERANGE).  The reference
// checks the running total after every add; non-finite values are absorbing
// under addition, so one check at the end reports the same outcome.
__global__ void __launch_bounds__(256) k_tmac_lookup_one(const int8_t *__restrict__ qlut,
                                                          const uint8_t *__restrict__ idx,
                                                          const float *__restrict__ scales,
                                                          const float *__restrict__ biases, size_t ngroups,
                                                          size_t nblocks, int bits, float w_scale,
                                                          float *__restrict__ out, int *__restrict__ flag) {
    __shared__ double part[256][4];
    __shared__ int bad;
    if (threadIdx.x == 0) bad = 0;
    __syncthreads();
    for (size_t bb = threadIdx.x; bb < nblocks; bb += blockDim.x)
        if (!isfinite(scales[bb]) || !isfinite(biases[bb])) bad = 1;
    __syncthreads();
    if (bad) {
        if (threadIdx.x == 0) flag[0] = 1;
        return;
    }
    double total = 0.0;
    for (size_t c0 = 0; c0 < nblocks; c0 += blockDim.x) {
        const size_t bb = c0 + threadIdx.x;
        if (bb < nblocks) {
            const uint32_t *qw = reinterpret_cast<const uint32_t *>(qlut + bb * 64);
            uint32_t q8[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) q8[i] = qw[i];
            const double sc = (double)scales[bb], bi = (double)biases[bb];
            for (int b = 0; b < bits; ++b) {
                const uint8_t *pl = idx + (size_t)b * ngroups + bb * 8;
                uint2 i8;
                i8.x = pl[0] | (pl[1] << 8) | (pl[2] << 16) | ((uint32_t)pl[3] << 24);
                i8.y = pl[4] | (pl[5] << 8) | (pl[6] << 16) | ((uint32_t)pl[7] << 24);
                part[threadIdx.x][b] = tmac_contrib(sc, bi, tmac_plane(q8, i8), b);
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            const size_t n = nblocks - c0 < blockDim.x ? nblocks - c0 : blockDim.x;
            for (size_t i = 0; i < n; ++i)
                for (int b = 0; b < bits; ++b) total = __dadd_rn(total, part[i][b]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        total = __dmul_rn(total, (double)w_scale);
        const float f = (float)total;
        if (!isfinite(total) || !isfinite(f)) {
            flag[0] = 2;
            return;
        }
        out[0] = f;
    }
}

// Weight columns of the LUT GEMM.  Column j of expert e has k elements,
// element t at W + e*ws + t*st + j*sj: st = h, sj = 1 for a row-major
// [k][h] matrix (lowbit.c:228-231), st = 1, sj = k for a [h][k] matrix
// whose rows are the columns (the transposed gate/up weights of
// moe_layer.c:1301-1332).
struct WCols {
    const float *W;
    long long ws, st, sj;
    __device__ __forceinline__ float at(int e, int t, int j) const {
        return W[(long long)e * ws + (long long)t * st + (long long)j * sj];
    }
};

// Column max-abs in double for lowbit.c:103-115, one (32 columns x 8 row
// slices) CTA per column block and expert; a non-finite column posts key
// (e*h + j)*(me+1) (EINVAL).
__global__ void __launch_bounds__(256) k_col_absmax(WCols w, int k, int h, int me, double *__restrict__ maxa,
                                                     unsigned long long *__restrict__ err) {
    __shared__ double sm[8][32];
    __shared__ int sbad[8][32];
    const int j = blockIdx.x * 32 + threadIdx.x, e = blockIdx.y;
    double m = 0.0;
    int bad = 0;
    if (j < h)
        for (int t = threadIdx.y; t < k; t += 8) {
            const double v = (double)w.at(e, t, j);
            bad |= !isfinite(v);
            m = fmax(m, fabs(v));
        }
    sm[threadIdx.y][threadIdx.x] = m;
    sbad[threadIdx.y][threadIdx.x] = bad;
    __syncthreads();
    if (threadIdx.y == 0 && j < h) {
        for (int y = 1; y < 8; ++y) {
            m = fmax(m, sm[y][threadIdx.x]);
            bad |= sbad[y][threadIdx.x];
        }
        maxa[(size_t)e * h + j] = m;
        if (bad) atomicMin(err, ((unsigned long long)((long long)e * h + j) * (unsigned long long)(me + 1)) << 1);
    }
}

// Bit planes of every column (lowbit.c:117-137) in the layout the LUT GEMM
// reads: idxT[((e*bits + b)*nb + bb)*h + j] holds the 8 index bytes of
// groups bb*8 .. bb*8+7 of column j, plane b.  One thread per (bb, j).
__global__ void k_col_planes(WCols w, int k, int h, int bits, const double *__restrict__ maxa,
                             uint2 *__restrict__ idxT) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    const int bb = blockIdx.y, e = blockIdx.z;
    if (j >= h) return;
    const int nb = k / 32, nl = 1 << bits;
    const double m = maxa[(size_t)e * h + j];
    uint32_t pl[4][2] = {{0, 0}, {0, 0}, {0, 0}, {0, 0}};
    for (int t = 0; t < 32; ++t) {
        const int li = level(w.at(e, bb * 32 + t, j), m, nl);
        const int g = t >> 2, jj = t & 3;
        for (int b = 0; b < bits; ++b)
            if ((li >> b) & 1) pl[b][g >> 2] |= 1u << (8 * (g & 3) + jj);
    }
    for (int b = 0; b < bits; ++b)
        idxT[(((size_t)e * bits + b) * nb + bb) * h + j] = make_uint2(pl[b][0], pl[b][1]);
}

// Row sums of X in double, ascending t (lowbit.c:217-224).
__global__ void k_row_sum_d(const float *__restrict__ X, int me, int k, double *__restrict__ rowsum) {
    const int m = blockIdx.x * blockDim.x + threadIdx.x;
    if (m >= me) return;
    double s = 0.0;
    for (int t = 0; t < k; ++t) s = __dadd_rn(s, (double)X[(size_t)m * k + t]);
    rowsum[m] = s;
}

// The LUT GEMM of lowbit.c:226-257: thread (m, j) runs lookup_accum over
// row m's table and column j's planes of row m's expert (rexp[m], or 0),
// then the sign correction Y = (float)((2o - ((n-1)*ws)*rowsum) / (n-1)).
// A non-finite o posts key j*(me+1) + m + 1 (ERANGE), ordered after column
// j's own col_to_idx check.
__global__ void __launch_bounds__(256) k_lut_gemm(const int8_t *__restrict__ qlut, const float *__restrict__ scales,
                                                   const float *__restrict__ biases, const uint2 *__restrict__ idxT,
                                                   const double *__restrict__ maxa,
                                                   const double *__restrict__ rowsum,
                                                   const int32_t *__restrict__ rexp, float *__restrict__ Y, int me,
                                                   int h, int k, int bits, unsigned long long *__restrict__ err) {
    const int j = blockIdx.x * 32 + threadIdx.x;
    const int m = blockIdx.y * 8 + threadIdx.y;
    if (j >= h || m >= me) return;
    const int nb = k / 32;
    const int e = rexp ? rexp[m] : 0;
    const float ws = (float)maxa[(size_t)e * h + j];
    const uint2 *planes = idxT + (size_t)e * bits * nb * h;
    const uint4 *qrow = reinterpret_cast<const uint4 *>(qlut + (size_t)m * nb * 64);
    double total = 0.0;
    for (int bb = 0; bb < nb; ++bb) {
        uint32_t q8[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = __ldg(qrow + (size_t)bb * 4 + i);
            q8[4 * i] = v.x;
            q8[4 * i + 1] = v.y;
            q8[4 * i + 2] = v.z;
            q8[4 * i + 3] = v.w;
        }
        const double sc = (double)scales[(size_t)m * nb + bb], bi = (double)biases[(size_t)m * nb + bb];
        for (int b = 0; b < bits; ++b) {
            const uint2 i8 = planes[((size_t)b * nb + bb) * h + j];
            total = __dadd_rn(total, tmac_contrib(sc, bi, tmac_plane(q8, i8), b));
        }
    }
    total = __dmul_rn(total, (double)ws);
    const float o = (float)total;
    if (!isfinite(total) || !isfinite(o)) {
        atomicMin(err, (((unsigned long long)j * (unsigned long long)(me + 1) + (unsigned long long)m + 1ull) << 1) | 1ull);
        return;
    }
    const double n1 = (double)((1 << bits) - 1);
    const double corr = __dmul_rn(__dmul_rn(n1, (double)ws), rowsum[m]);
    Y[(size_t)m * h + j] = (float)__ddiv_rn(__dsub_rn(__dmul_rn(2.0, (double)o), corr), n1);
}

// lowbit.c:143-156: the k % 32 != 0 fallback, Y = (float) sum_t X*W in
// double, ascending t (products of floats are exact in double); W column j
// of row m's expert as in WCols.
__global__ void k_gemm_f64acc(const float *__restrict__ X, WCols w, const int32_t *__restrict__ rexp,
                              float *__restrict__ Y, int me, int h, int k) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= h) return;
    for (int m = blockIdx.y; m < me; m += gridDim.y) {
        const int e = rexp ? rexp[m] : 0;
        double acc = 0.0;
        for (int t = 0; t < k; ++t)
            acc = __dadd_rn(acc, __dmul_rn((double)X[(size_t)m * k + t], (double)w.at(e, t, j)));
        Y[(size_t)m * h + j] = (float)acc;
    }
}

int grid_for(size_t n, int threads) {
    size_t g = (n + threads - 1) / threads;
    const size_t cap = (size_t)jtk_num_sms() * 8;
    if (g > cap) g = cap;
    return g < 1 ? 1 : (int)g;
}

}  // namespace

extern "C" int jtk_tmac_ctor(const float *act, size_t n, size_t k, int8_t *qlut, float *scales, float *biases,
                             unsigned long long *err, cudaStream_t stream) {
    if (n == 0 || k == 0 || k % 32) return -1;
    const size_t units = n * (k / 32);
    const size_t grid = (units + 127) / 128;
    if (grid > 0x7fffffffull) return -1;
    if (cudaMemsetAsync(err, 0xff, sizeof(unsigned long long), stream) != cudaSuccess) return -4;
    k_tmac_ctor<<<(unsigned)grid, 128, 0, stream>>>(act, n, k, qlut, scales, biases, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_tmac_lookup_one(const int8_t *qlut, const uint8_t *idx, const float *scales,
                                   const float *biases, size_t ngroups, size_t nblocks, int bits, float w_scale,
                                   float *out, int *flag, cudaStream_t stream) {
    if (nblocks == 0 || ngroups != nblocks * 8 || bits < 1 || bits > 4) return -1;
    k_tmac_lookup_one<<<1, 256, 0, stream>>>(qlut, idx, scales, biases, ngroups, nblocks, bits, w_scale, out,
                                             flag);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

// LUT GEMM after the row tables are built (jtk_tmac_ctor): column
// max-abs and bit planes of every expert's columns, row sums, the lookups.
// *err is reset here and receives the first column / lookup error.  rexp
// [me] maps rows to experts (NULL: one expert).
extern "C" int jtk_lut_gemm(const float *X, const float *W, int E, long long ws, long long st, long long sj,
                            const int32_t *rexp, const int8_t *qlut, const float *scales, const float *biases,
                            double *maxa, void *idx_planes, double *rowsum, float *Y, int me, int h, int k,
                            int bits, unsigned long long *err, cudaStream_t stream) {
    if (me <= 0 || h <= 0 || k <= 0 || E <= 0 || E > 65535 || k % 32 || (bits != 2 && bits != 4) ||
        (me + 7) / 8 > 65535 || k / 32 > 65535)
        return -1;
    uint2 *idxT = static_cast<uint2 *>(idx_planes);
    const WCols w{W, ws, st, sj};
    if (cudaMemsetAsync(err, 0xff, sizeof(unsigned long long), stream) != cudaSuccess) return -4;
    const unsigned gx = (unsigned)((h + 31) / 32);
    k_col_absmax<<<dim3(gx, (unsigned)E), dim3(32, 8), 0, stream>>>(w, k, h, me, maxa, err);
    k_col_planes<<<dim3((unsigned)((h + 127) / 128), (unsigned)(k / 32), (unsigned)E), 128, 0, stream>>>(
        w, k, h, bits, maxa, idxT);
    k_row_sum_d<<<(me + 127) / 128, 128, 0, stream>>>(X, me, k, rowsum);
    k_lut_gemm<<<dim3(gx, (unsigned)((me + 7) / 8)), dim3(32, 8), 0, stream>>>(qlut, scales, biases, idxT, maxa,
                                                                              rowsum, rexp, Y, me, h, k, bits, err);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_gemm_f64acc(const float *X, const float *W, long long ws, long long st, long long sj,
                               const int32_t *rexp, float *Y, int me, int h, int k, cudaStream_t stream) {
    if (me <= 0 || h <= 0 || k <= 0) return -1;
    const unsigned gy = (unsigned)(me < 65535 ? me : 65535);
    k_gemm_f64acc<<<dim3((unsigned)((h + 127) / 128), gy), 128, 0, stream>>>(X, WCols{W, ws, st, sj}, rexp, Y,
                                                                            me, h, k);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_topk_any(const float *logits, int T, int n, int k, uint32_t *taken, int32_t *ids, float *w,
                            int *flag, cudaStream_t stream) {
    if (T <= 0 || n <= 0 || k <= 0 || k > n) return -1;
    k_topk_any<<<T, 1024, 0, stream>>>(logits, n, k, taken, ids, w, flag);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_gemm_f32_seq(const float *A, const float *B, float *C, int M, int N, int K,
                                cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M > 65535) return -1;
    dim3 grid((N + 127) / 128, M);
    k_gemm_f32_seq<<<grid, 128, 0, stream>>>(A, B, C, M, N, K);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_transpose_f32(const float *src, float *dst, int rows, int cols, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || (rows + 31) / 32 > 65535) return -1;
    dim3 grid((cols + 31) / 32, (rows + 31) / 32);
    k_transpose_f32<<<grid, dim3(32, 8), 0, stream>>>(src, dst, rows, cols);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_lowbit_absmax(const float *w, size_t n, unsigned long long *maxbits, int *bad,
                                 cudaStream_t stream) {
    if (n == 0) return -1;
    if (cudaMemsetAsync(maxbits, 0, sizeof(unsigned long long), stream) != cudaSuccess) return -4;
    k_absmax_d<<<grid_for(n, 256), 256, 0, stream>>>(w, n, maxbits, bad);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_lowbit_fq(const float *w, size_t n, int bits, const unsigned long long *maxbits, float *fq,
                             cudaStream_t stream) {
    k_lowbit_fq<<<grid_for(n, 256), 256, 0, stream>>>(w, n, bits, maxbits, fq);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

extern "C" int jtk_lowbit_idx(const float *col, size_t k, int bits, const unsigned long long *maxbits,
                              uint8_t *idx, cudaStream_t stream) {
    k_lowbit_idx<<<grid_for(k / 4, 256), 256, 0, stream>>>(col, k, bits, maxbits, idx);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
}
