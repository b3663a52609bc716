// jt_layer_ref.cu - kernels of the reference-signature MoE layer entry
// points (jt_api_layer.c): jt_moe_fwd_batch[_unchecked] (moe_layer.c:980-1663)
// and jt_moe_fwd[_unchecked] (moe_layer.c:304-545).  They take the
// reference's fp32 weights and reproduce its arithmetic: the 4-lane double
// dot of the gate logits and of the single-token SwiGLU, fp32 GEMMs with one
// rounding per multiply and add in ascending k, double SwiGLU, the double
// combine in slot order.  The int8 and LUT modes reuse the exact W8A8 and
// T-MAC kernels.
//
// Error flags: flags[i] = 1 (EINVAL) or 2 (ERANGE), set with atomicExch.
#include <cuda_runtime.h>
#include <stdint.h>

#include "jt_internal.h"

namespace {

// The 4-lane double dot of moe_layer.c:74-94 / train_bwd.c:150-169: lane l
// sums x[j]*y[j] for j = l mod 4 below n & ~3 in ascending j, the lanes
// combine as (l0 + l1) + (l2 + l3), then the tail adds in order.  Products
// of two floats are exact in double.
__device__ __forceinline__ double dot4(const float *__restrict__ x, const float *__restrict__ y, int n) {
    double l0 = 0.0, l1 = 0.0, l2 = 0.0, l3 = 0.0;
    const int n4 = n & ~3;
    int j = 0;
    for (; j < n4; j += 4) {
        l0 = __dadd_rn(l0, __dmul_rn((double)x[j], (double)y[j]));
        l1 = __dadd_rn(l1, __dmul_rn((double)x[j + 1], (double)y[j + 1]));
        l2 = __dadd_rn(l2, __dmul_rn((double)x[j + 2], (double)y[j + 2]));
        l3 = __dadd_rn(l3, __dmul_rn((double)x[j + 3], (double)y[j + 3]));
    }
    double s = __dadd_rn(__dadd_rn(l0, l1), __dadd_rn(l2, l3));
    for (; j < n; ++j) s = __dadd_rn(s, __dmul_rn((double)x[j], (double)y[j]));
    return s;
}

// Gate logits (moe_layer.c:1117-1135): logits[t][e] = (float)dot4(X[t],
// Wgate[e]); a non-finite dot or float -> EINVAL.
__global__ void k_logits(const float *__restrict__ X, const float *__restrict__ Wgate, int T, int n, int E,
                         float *__restrict__ logits, int *flags) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (e >= E || t >= T) return;
    const double acc = dot4(X + (size_t)t * n, Wgate + (size_t)e * n, n);
    const float f = (float)acc;
    if (!isfinite(acc) || !isfinite(f)) atomicExch(&flags[0], 1);
    logits[(size_t)t * E + e] = f;
}

// Xe[r] = X[perm[r] / k] (moe_layer.c:1265-1271).
__global__ void k_gather_rows(const float *__restrict__ X, const int32_t *__restrict__ perm, int k, int R, int n,
                              float *__restrict__ Xe) {
    const int r = blockIdx.y;
    if (r >= R) return;
    const float *src = X + (size_t)(perm[r] / k) * n;
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
        Xe[(size_t)r * n + j] = src[j];
}

// rexp[r] = expert of sorted row r, from off [E+1].
__global__ void k_row_expert(const int32_t *__restrict__ off, int E, int32_t *__restrict__ rexp) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= E) return;
    for (int r = off[e]; r < off[e + 1]; ++r) rexp[r] = e;
}

// fp32 GEMM of moe_gemm.c:92-170 over 32-row tiles of one expert each:
// C[r][j] = sum_kk A[r][kk] * B_e[kk][j], acc = fl(acc + fl(a*b)) in
// ascending kk from 0.0f.  B_e = W + e*ws, row-major [K][N] (wt 0) or the
// transpose of a row-major [N][K] (wt 1, an exact transpose like
// moe_layer.c:1285-1297).  tiles[y] = {e, row0, row_end, 0}.
constexpr int kT = 32;
__global__ void __launch_bounds__(256) k_gemm_f32_tiles(const float *__restrict__ A, int lda,
                                                         const float *__restrict__ W, long long ws, int wt,
                                                         const int4 *__restrict__ tiles, float *__restrict__ C,
                                                         int ldc, int N, int K) {
    __shared__ float As[kT][kT + 1];
    __shared__ float Bs[kT][kT + 1];
    const int4 tl = tiles[blockIdx.y];
    const int r0 = tl.y, r1 = tl.z;
    const int j0 = blockIdx.x * kT;
    const int tx = threadIdx.x, ty = threadIdx.y;
    const float *We = W + (long long)tl.x * ws;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int k0 = 0; k0 < K; k0 += kT) {
        const int kn = min(kT, K - k0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 8 * i;
            As[r][tx] = (r0 + r < r1 && tx < kn) ? A[(size_t)(r0 + r) * lda + k0 + tx] : 0.0f;
            if (wt == 0)
                Bs[r][tx] = (r < kn && j0 + tx < N) ? We[(size_t)(k0 + r) * N + j0 + tx] : 0.0f;
            else
                Bs[tx][r] = (tx < kn && j0 + r < N) ? We[(size_t)(j0 + r) * K + k0 + tx] : 0.0f;
        }
        __syncthreads();
        for (int kk = 0; kk < kn; ++kk) {
            const float b = Bs[kk][tx];
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(As[ty + 8 * i][kk], b));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = ty + 8 * i;
        if (r0 + r < r1 && j0 + tx < N) C[(size_t)(r0 + r) * ldc + j0 + tx] = acc[i];
    }
}

// SwiGLU tile of moe_layer.c:129-157 / :1528-1540: sig = 1/(1+exp(-g)),
// silu = g*sig, s = silu*u in double, S = (float)s; non-finite -> EINVAL.
__global__ void k_silu(const float *__restrict__ G, const float *__restrict__ U, float *__restrict__ S,
                       size_t count, int *flags) {
    int bad = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        const double g = (double)G[i], u = (double)U[i];
        const double sig = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-g)));
        const double silu = __dmul_rn(g, sig);
        const double s = __dmul_rn(silu, u);
        bad |= !isfinite(s) || !isfinite(sig) || !isfinite(silu);
        S[i] = (float)s;
    }
    if (bad) atomicExch(&flags[0], 1);
}

// Low-bit level index and value of lowbit.c:78-90.
__device__ __forceinline__ float lowbit_fq(float wv, double maxa, int nl) {
    if (maxa == 0.0) return 0.0f;
    const double t = __ddiv_rn((double)wv, maxa);
    const double li = floor(__dadd_rn(__dadd_rn(__ddiv_rn(__dmul_rn(t, (double)(nl - 1)), 2.0),
                                                 (double)(nl - 1) / 2.0),
                                      0.5));
    long l = (long)li;
    l = l < 0 ? 0 : l;
    l = l > nl - 1 ? nl - 1 : l;
    const double nd = (double)(nl - 1);
    const double lv = __ddiv_rn(__dsub_rn(2.0 * (double)l, nd), nd);
    return (float)__dmul_rn(lv, maxa);
}

// Fake-quant of every row of W [rows][cols] with its own max-abs: the
// per-column fake-quant of the transposed gate/up weights
// (moe_layer.c:24-53 on Wgt = Wg^T).  One CTA per row.
__global__ void __launch_bounds__(256) k_fq_rows(const float *__restrict__ W, int cols, int bits,
                                                  float *__restrict__ out, int *flags) {
    __shared__ double sm[8];
    __shared__ int sb[8];
    const float *row = W + (size_t)blockIdx.x * cols;
    double m = 0.0;
    int bad = 0;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) {
        const double v = (double)row[i];
        bad |= !isfinite(v);
        m = fmax(m, fabs(v));
    }
    for (int o = 16; o > 0; o >>= 1) {
        m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if ((threadIdx.x & 31) == 0) {
        sm[threadIdx.x >> 5] = m;
        sb[threadIdx.x >> 5] = bad;
    }
    __syncthreads();
    m = 0.0;
    bad = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
        m = fmax(m, sm[w]);
        bad |= sb[w];
    }
    if (bad) {
        if (threadIdx.x == 0) atomicExch(&flags[0], 1);
        return;
    }
    const int nl = 1 << bits;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) out[(size_t)blockIdx.x * cols + i] = lowbit_fq(row[i], m, nl);
}

// Fake-quant of every column of each expert's W [h][n] (moe_layer.c:24-53
// on the down weights): thread per (expert, column).
__global__ void k_fq_cols(const float *__restrict__ W, int E, int h, int n, int bits, float *__restrict__ out,
                          int *flags) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x, e = blockIdx.y;
    if (j >= n || e >= E) return;
    const float *col = W + (size_t)e * h * n + j;
    double m = 0.0;
    int bad = 0;
    for (int t = 0; t < h; ++t) {
        const double v = (double)col[(size_t)t * n];
        bad |= !isfinite(v);
        m = fmax(m, fabs(v));
    }
    if (bad) {
        atomicExch(&flags[0], 1);
        return;
    }
    const int nl = 1 << bits;
    for (int t = 0; t < h; ++t) out[(size_t)e * h * n + (size_t)t * n + j] = lowbit_fq(col[(size_t)t * n], m, nl);
}

// dst[e][j] = src[e] (per-tensor down scale spread over the output channels).
__global__ void k_fill_rows(const float *__restrict__ src, int E, int n, float *__restrict__ dst) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x, e = blockIdx.y;
    if (j < n && e < E) dst[(size_t)e * n + j] = src[e];
}

// Combine of moe_layer.c:1443-1463 and :1543-1552: per (t, j) the double
// sum over kept slots p of (double)w*(double)Ye[pos[q]][j], then the shared
// rows Ys[s][t][j]; non-finite -> EINVAL; Y = (float)sum.
__global__ void k_combine(const float *__restrict__ Ye, const int32_t *__restrict__ pos,
                          const float *__restrict__ w, const uint8_t *__restrict__ drop, int T, int t_base, int k,
                          int n, const float *__restrict__ Ys, int S, float *__restrict__ Y, int *flags) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x, t = t_base + (int)blockIdx.y;
    if (j >= n || t >= T) return;
    double ya = 0.0;
    for (int p = 0; p < k; ++p) {
        const size_t q = (size_t)t * k + p;
        if (drop[q]) continue;
        ya = __dadd_rn(ya, __dmul_rn((double)w[q], (double)Ye[(size_t)pos[q] * n + j]));
    }
    for (int s = 0; s < S; ++s) ya = __dadd_rn(ya, (double)Ys[((size_t)s * T + t) * n + j]);
    if (!isfinite(ya)) atomicExch(&flags[0], 1);
    Y[(size_t)t * n + j] = (float)ya;
}

// Per (token, slot) cache rows (moe_layer.c:1400-1438): kept slots copy
// their sorted row, dropped slots are zero.
__global__ void k_scatter_rows(const float *__restrict__ src, const int32_t *__restrict__ pos,
                               const uint8_t *__restrict__ drop, int cols, float *__restrict__ dst) {
    const size_t q = blockIdx.y;
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= cols) return;
    dst[q * cols + j] = drop[q] ? 0.0f : src[(size_t)pos[q] * cols + j];
}

// Single-token SwiGLU of train_bwd.c:926-1043 for P experts: thread (p, i)
// computes g, u = dot4(x, W_e[i]), s = silu(g)*u in double (kept in
// double), G/U = (float)g/(float)u.  ids[p] selects the expert (NULL: p).
__global__ void k_tok_gateup(const float *__restrict__ x, const float *__restrict__ Wg,
                             const float *__restrict__ Wu, const int32_t *__restrict__ ids, int P, int n, int h,
                             double *__restrict__ s, float *__restrict__ G, float *__restrict__ U, int *flags) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x, p = blockIdx.y;
    if (i >= h || p >= P) return;
    const size_t e = ids ? (size_t)ids[p] : (size_t)p;
    const double g = dot4(x, Wg + (e * h + i) * n, n);
    const double u = dot4(x, Wu + (e * h + i) * n, n);
    const double sig = __ddiv_rn(1.0, __dadd_rn(1.0, exp(-g)));
    const double v = __dmul_rn(__dmul_rn(g, sig), u);
    if (!isfinite(g) || !isfinite(u) || !isfinite(v)) atomicExch(&flags[0], 1);
    s[(size_t)p * h + i] = v;
    G[(size_t)p * h + i] = (float)g;
    U[(size_t)p * h + i] = (float)u;
}

// y[p][j] = (float) sum_i s[p][i] * (double)Wd_e[i][j], ascending i.
__global__ void k_tok_down(const double *__restrict__ s, const float *__restrict__ Wd,
                           const int32_t *__restrict__ ids, int P, int n, int h, float *__restrict__ y, int *flags) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x, p = blockIdx.y;
    if (j >= n || p >= P) return;
    const size_t e = ids ? (size_t)ids[p] : (size_t)p;
    const float *wd = Wd + e * h * n + j;
    const double *sp = s + (size_t)p * h;
    double acc = 0.0;
    for (int i = 0; i < h; ++i) acc = __dadd_rn(acc, __dmul_rn(sp[i], (double)wd[(size_t)i * n]));
    if (!isfinite(acc)) atomicExch(&flags[0], 1);
    y[(size_t)p * n + j] = (float)acc;
}

// Single-token combine (moe_layer.c:443-490): sum_p (double)w_p*(double)Yr[p][j]
// then + (double)Ys[s][j]; non-finite -> EINVAL.
__global__ void k_tok_combine(const float *__restrict__ Yr, const float *__restrict__ w, int P,
                              const float *__restrict__ Ys, int S, int n, float *__restrict__ Y, int *flags) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n) return;
    double ya = 0.0;
    for (int p = 0; p < P; ++p) ya = __dadd_rn(ya, __dmul_rn((double)w[p], (double)Yr[(size_t)p * n + j]));
    for (int s = 0; s < S; ++s) ya = __dadd_rn(ya, (double)Ys[(size_t)s * n + j]);
    if (!isfinite(ya)) atomicExch(&flags[0], 1);
    Y[j] = (float)ya;
}

inline int ok() { return cudaGetLastError() == cudaSuccess ? 0 : -4; }
inline unsigned cdiv(long long a, long long b) { return (unsigned)((a + b - 1) / b); }

}  // namespace

extern "C" {

int jtk_ref_logits(const float *X, const float *Wgate, int T, int n, int E, float *logits, int *flags,
                   cudaStream_t st) {
    if (T <= 0 || T > 65535 * 64 || n <= 0 || E <= 0) return -1;
    for (int t0 = 0; t0 < T; t0 += 65535) {
        const int tn = T - t0 < 65535 ? T - t0 : 65535;
        k_logits<<<dim3(cdiv(E, 128), tn), 128, 0, st>>>(X + (size_t)t0 * n, Wgate, tn, n, E,
                                                         logits + (size_t)t0 * E, flags);
    }
    return ok();
}

int jtk_ref_gather(const float *X, const int32_t *perm, int k, int R, int n, float *Xe, cudaStream_t st) {
    if (R <= 0) return 0;
    for (int r0 = 0; r0 < R; r0 += 65535) {
        const int rn = R - r0 < 65535 ? R - r0 : 65535;
        k_gather_rows<<<dim3(cdiv(n, 256) < 4 ? cdiv(n, 256) : 4, rn), 256, 0, st>>>(X, perm + r0, k, rn, n,
                                                                                     Xe + (size_t)r0 * n);
    }
    return ok();
}

int jtk_ref_row_expert(const int32_t *off, int E, int32_t *rexp, cudaStream_t st) {
    k_row_expert<<<cdiv(E, 128), 128, 0, st>>>(off, E, rexp);
    return ok();
}

int jtk_ref_gemm_f32(const float *A, int lda, const float *W, long long ws, int wt, const int4 *tiles, int ntiles,
                     float *C, int ldc, int N, int K, cudaStream_t st) {
    if (ntiles <= 0) return 0;
    if (ntiles > 65535 || N <= 0 || K <= 0) return -1;
    k_gemm_f32_tiles<<<dim3(cdiv(N, kT), ntiles), dim3(32, 8), 0, st>>>(A, lda, W, ws, wt, tiles, C, ldc, N, K);
    return ok();
}

int jtk_ref_silu(const float *G, const float *U, float *S, size_t count, int *flags, cudaStream_t st) {
    if (count == 0) return 0;
    const long long g = (long long)cdiv((long long)count, 256);
    const long long cap = (long long)jtk_num_sms() * 8;
    k_silu<<<(unsigned)(g < cap ? g : cap), 256, 0, st>>>(G, U, S, count, flags);
    return ok();
}

int jtk_ref_fq_rows(const float *W, int rows, int cols, int bits, float *out, int *flags, cudaStream_t st) {
    if (rows <= 0) return 0;
    k_fq_rows<<<rows, 256, 0, st>>>(W, cols, bits, out, flags);
    return ok();
}

int jtk_ref_fq_cols(const float *W, int E, int h, int n, int bits, float *out, int *flags, cudaStream_t st) {
    if (E <= 0 || E > 65535) return -1;
    k_fq_cols<<<dim3(cdiv(n, 128), E), 128, 0, st>>>(W, E, h, n, bits, out, flags);
    return ok();
}

int jtk_ref_fill_rows(const float *src, int E, int n, float *dst, cudaStream_t st) {
    if (E <= 0 || E > 65535) return -1;
    k_fill_rows<<<dim3(cdiv(n, 128), E), 128, 0, st>>>(src, E, n, dst);
    return ok();
}

int jtk_ref_combine(const float *Ye, const int32_t *pos, const float *w, const uint8_t *drop, int T, int k, int n,
                    const float *Ys, int S, float *Y, int *flags, cudaStream_t st) {
    for (int t0 = 0; t0 < T; t0 += 65535) {
        const int tn = T - t0 < 65535 ? T - t0 : 65535;
        k_combine<<<dim3(cdiv(n, 128), tn), 128, 0, st>>>(Ye, pos, w, drop, T, t0, k, n, Ys, S, Y, flags);
    }
    return ok();
}

int jtk_ref_scatter_rows(const float *src, const int32_t *pos, const uint8_t *drop, size_t Tk, int cols, float *dst,
                         cudaStream_t st) {
    for (size_t q0 = 0; q0 < Tk; q0 += 65535) {
        const size_t qn = Tk - q0 < 65535 ? Tk - q0 : 65535;
        k_scatter_rows<<<dim3(cdiv(cols, 128), (unsigned)qn), 128, 0, st>>>(src, pos + q0, drop + q0, cols,
                                                                              dst + q0 * cols);
    }
    return ok();
}

int jtk_ref_tok_gateup(const float *x, const float *Wg, const float *Wu, const int32_t *ids, int P, int n, int h,
                       double *s, float *G, float *U, int *flags, cudaStream_t st) {
    if (P <= 0) return 0;
    k_tok_gateup<<<dim3(cdiv(h, 128), P), 128, 0, st>>>(x, Wg, Wu, ids, P, n, h, s, G, U, flags);
    return ok();
}

int jtk_ref_tok_down(const double *s, const float *Wd, const int32_t *ids, int P, int n, int h, float *y,
                     int *flags, cudaStream_t st) {
    if (P <= 0) return 0;
    k_tok_down<<<dim3(cdiv(n, 128), P), 128, 0, st>>>(s, Wd, ids, P, n, h, y, flags);
    return ok();
}

int jtk_ref_tok_combine(const float *Yr, const float *w, int P, const float *Ys, int S, int n, float *Y, int *flags,
                        cudaStream_t st) {
    k_tok_combine<<<cdiv(n, 128), 128, 0, st>>>(Yr, w, P, Ys, S, n, Y, flags);
    return ok();
}

}  // extern "C"
