// jt_topk.cuh - top-k + softmax of one token's router logits by one warp,
// shared by the batched router (jt_route.cu) and the batch-1 layer
// (jt_decode.cu).
//
// Lane l holds logits l, l+32, ...  Each of the k passes takes the maximum
// of (taken ? -inf : logit [+ bias]) with ties to the lowest index, exactly
// the strict '>' scan of routing.c:38-52 (including its behaviour when only
// -inf values remain); then the softmax of routing.c:54-73: float max,
// double exps (one slot per lane) summed in slot order, w = (float)e *
// (float)(1/sum).  A NaN logit raises err 0x81 (nothing is written), a bad
// softmax sum 0x82.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace jt {

// Shared-memory words a warp passes as `taken` to warp_topk_softmax.
__host__ __device__ inline int topk_scratch_words(int E) { return E <= 64 ? 128 : (E + 31) / 32; }

// Selection for E <= 64 logits without the k dependent passes: lane l holds
// logits l and l + 32 (+ bias) and counts the logits that a pass would take
// before each of them - the larger ones, and the equal ones of lower index -
// which is its pass number (routing.c:38-52 takes, at every pass, the
// largest remaining logit with ties to the lowest index).  All counts are
// formed at once, from the 64 logits staged in shared memory (scratch, 128
// words owned by the warp) and read back as broadcasts.  The ranking equals
// the passes' order whenever no logit is -inf (a pass that finds only -inf
// left may take an index again, which a ranking cannot express); in that
// case, or for a NaN, it returns false before touching scratch and the
// caller runs the passes.  Every lane writes sel/selv entries 0..k-1 (the
// same values), as the passes do.
__device__ __forceinline__ bool small_select(float v0, float v1, bool ok0, bool ok1, int k, uint32_t *scratch,
                                             int32_t *sel, float *selv) {
    const int lane = threadIdx.x & 31;
    const bool odd = (ok0 && (v0 != v0 || v0 == -INFINITY)) || (ok1 && (v1 != v1 || v1 == -INFINITY));
    if (__any_sync(0xffffffffu, odd)) return false;
    // missing logits (E < 64) read as -inf, which beats no present logit
    // (none is -inf here), so the counts need no bound
    float *val = reinterpret_cast<float *>(scratch);
    int32_t *slot = reinterpret_cast<int32_t *>(scratch) + 64;
    const float w0 = ok0 ? v0 : -INFINITY, w1 = ok1 ? v1 : -INFINITY;
    val[lane] = w0;
    val[lane + 32] = w1;
    __syncwarp();
    int c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
        const float4 a = reinterpret_cast<const float4 *>(val)[j4];      // logits 4 j4 ..
        const float4 b = reinterpret_cast<const float4 *>(val + 32)[j4]; // logits 32 + 4 j4 ..
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = 4 * j4 + t;
            c0[t] += (av[t] > w0) || (av[t] == w0 && j < lane);  // logit j against lane
            c1[t] += (av[t] >= w1);                              // j < lane + 32: ties count
            c0[t] += (bv[t] > w0);                               // 32 + j > lane: ties do not count
            c1[t] += (bv[t] > w1) || (bv[t] == w1 && j < lane);  // 32 + j against lane + 32
        }
    }
    const int r0 = (c0[0] + c0[1]) + (c0[2] + c0[3]);
    const int r1 = (c1[0] + c1[1]) + (c1[2] + c1[3]);
    // the logit of count q goes to slot q
    if (ok0 && r0 < k) slot[r0] = lane;
    if (ok1 && r1 < k) slot[r1] = lane + 32;
    __syncwarp();
    for (int q = 0; q < k; ++q) {
        const int id = slot[q];
        sel[q] = id;
        selv[q] = val[id];
    }
    __syncwarp();
    return true;
}

// taken: max(ceil(E/32), 128 if E <= 64) words of shared memory owned by
// this warp (the selection for E <= 64 uses 128 words of it as scratch); sel/selv: k
// entries of scratch written identically by every lane; ids_out/w_out
// entry p is written by lane p mod 32 with the softmax, by lane 0 without
// it (nothing on a bad softmax sum).  With softmax == false only the ids
// are produced (w_out is not touched), for callers that need the experts
// before the weights.  Returns false on a NaN logit.
__device__ __forceinline__ bool warp_topk_softmax(const float *__restrict__ row, const float *__restrict__ bias,
                                                  int E, int k, uint32_t *taken, int32_t *sel, float *selv,
                                                  int32_t *ids_out, float *w_out, int *err,
                                                  bool softmax = true) {
    const int lane = threadIdx.x & 31;
    const int nw = (E + 31) / 32;
    for (int i = lane; i < nw; i += 32) taken[i] = 0;
    __syncwarp();
    bool selected = false;
    if (E <= 64) {
        // lane l holds logits l and l + 32 (+ bias), read once
        const bool ok0 = lane < E, ok1 = lane + 32 < E;
        float v0 = 0.0f, v1 = 0.0f;
        if (ok0) v0 = bias ? __fadd_rn(row[lane], bias[lane]) : row[lane];
        if (ok1) v1 = bias ? __fadd_rn(row[lane + 32], bias[lane + 32]) : row[lane + 32];
        if (__any_sync(0xffffffffu, (ok0 && v0 != v0) || (ok1 && v1 != v1))) {
            if (lane == 0) atomicExch(err, 0x81);
            return false;
        }
        selected = small_select(v0, v1, ok0, ok1, k, taken, sel, selv);
    } else {
        int nan_seen = 0;
        for (int i = lane; i < E; i += 32) {
            float v = row[i];
            if (bias) v = __fadd_rn(v, bias[i]);
            nan_seen |= (v != v);
        }
        if (__any_sync(0xffffffffu, nan_seen)) {
            if (lane == 0) atomicExch(err, 0x81);
            return false;
        }
    }
    if (!selected) {
        for (int p = 0; p < k; ++p) {
            float best = 0.0f;
            int bi = E;  // sentinel: "not set", like best == n in routing.c:40
            for (int i = lane; i < E; i += 32) {
                float v = row[i];
                if (bias) v = __fadd_rn(v, bias[i]);
                if ((taken[i >> 5] >> (i & 31)) & 1u) v = -INFINITY;
                if (bi == E || v > best) {
                    best = v;
                    bi = i;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                // candidate with lower index wins unless the other is strictly larger
                bool take;
                if (oi == E) take = false;
                else if (bi == E) take = true;
                else if (oi < bi) take = !(best > ov);
                else take = ov > best;
                if (take) {
                    best = ov;
                    bi = oi;
                }
            }
            sel[p] = bi;
            if (lane == 0) atomicOr(&taken[bi >> 5], 1u << (bi & 31));
            __syncwarp();
            float lv = row[bi];
            if (bias) lv = __fadd_rn(lv, bias[bi]);
            selv[p] = lv;
        }
    }
    if (!softmax) {
        if (lane == 0)
            for (int p = 0; p < k; ++p) ids_out[p] = sel[p];
        return true;
    }
    // softmax (routing.c:54-73): every lane takes the exp of its slots
    // (lane p: slots p and p + 32); the sum is formed in slot order (on
    // every lane, from the shuffled terms), as the reference's loop adds
    float mx = selv[0];
    for (int p = 1; p < k; ++p) mx = (selv[p] > mx) ? selv[p] : mx;
    double e0 = 0.0, e1 = 0.0;
    if (lane < k) e0 = exp((double)selv[lane] - (double)mx);
    if (lane + 32 < k) e1 = exp((double)selv[lane + 32] - (double)mx);
    double sum = 0.0;
    for (int p = 0; p < k; ++p) sum += __shfl_sync(0xffffffffu, p < 32 ? e0 : e1, p & 31);
    // every lane holds the same sum (the same adds in the same order)
    if (!(sum > 0.0) || !isfinite(sum)) {
        if (lane == 0) atomicExch(err, 0x82);
        return true;
    }
    const float inv = (float)(1.0 / sum);
    if (lane < k) {
        ids_out[lane] = sel[lane];
        w_out[lane] = __fmul_rn((float)e0, inv);
    }
    if (lane + 32 < k) {
        ids_out[lane + 32] = sel[lane + 32];
        w_out[lane + 32] = __fmul_rn((float)e1, inv);
    }
    return true;
}

}  // namespace jt
