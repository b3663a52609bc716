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

// taken: ceil(E/32) words of shared memory owned by this warp; sel/selv: k
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
