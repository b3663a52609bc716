/* jt_ep_layout.c - host-side bookkeeping of the expert-parallel MoE layer.
 *
 * N ranks, each holding a contiguous slice of the tokens (rank r has the
 * tokens that come before rank r+1's in the global order) and the experts
 * [r*E/N, (r+1)*E/N).  The reference keeps, per expert, the first `cap`
 * (token, slot) pairs in the global q = t*k + p order and drops the rest
 * (moe_layer.c:931-970).  With the per-rank expert counts cnt[s][e] of all
 * ranks (one all-gather), every rank derives the same global decision:
 *
 *   kept(s, e) = clamp(cap - sum_{s' < s} cnt[s'][e], 0, cnt[s][e])
 *
 * i.e. rank s keeps the first kept(s, e) of its own pairs of expert e in
 * its local q order.  From kept() this file computes what rank `rank`
 * sends to each owner, receives from each source, and where every received
 * row goes in its expert-contiguous matrix.  Pure integer code, no device
 * calls: the same function is tested on the CPU.
 */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"

static int64_t kept_of(const int32_t *cnt, int E, int s, int e, int64_t cap) {
    int64_t before = 0;
    for (int s2 = 0; s2 < s; s2++) before += cnt[(size_t)s2 * E + e];
    int64_t k = cap - before;
    if (k < 0) k = 0;
    if (k > cnt[(size_t)s * E + e]) k = cnt[(size_t)s * E + e];
    return k;
}

int jt_b200_ep_capacity(long long T_global, int k, int E, float cap_factor) {
    if (T_global <= 0 || k <= 0 || E <= 0 || !(cap_factor > 0.0f)) return -1;
    /* capacity of moe_layer.c:931-943 (double arithmetic) */
    const double capd = ceil((double)cap_factor * (double)(T_global * (long long)k) / (double)E);
    if (!isfinite(capd) || capd < 1.0 || capd > 2147483647.0) return -1;
    return (int)capd;
}

int jt_b200_ep_layout(const int32_t *cnt, int N, int E, int rank, int cap, int32_t *gbase,
                      int32_t *send_cnt, int32_t *recv_cnt, int32_t *own_off,
                      int32_t *own_tile_off, int32_t *gather) {
    if (cnt == NULL || N <= 0 || E <= 0 || E % N != 0 || rank < 0 || rank >= N || cap <= 0 ||
        gbase == NULL || send_cnt == NULL || recv_cnt == NULL || own_off == NULL ||
        own_tile_off == NULL || gather == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const int El = E / N, e0 = rank * El;
    for (int e = 0; e < E; e++) {
        int64_t before = 0;
        for (int s = 0; s < rank; s++) before += cnt[(size_t)s * E + e];
        if (before > INT32_MAX) before = INT32_MAX;
        gbase[e] = (int32_t)before;
    }
    for (int o = 0; o < N; o++) {
        int64_t n = 0;
        for (int e = o * El; e < (o + 1) * El; e++) n += kept_of(cnt, E, rank, e, cap);
        send_cnt[o] = (int32_t)n;
    }
    for (int s = 0; s < N; s++) {
        int64_t n = 0;
        for (int e = e0; e < e0 + El; e++) n += kept_of(cnt, E, s, e, cap);
        recv_cnt[s] = (int32_t)n;
    }
    /* expert-contiguous rows of the owned experts, and their token tiles */
    own_off[0] = 0;
    own_tile_off[0] = 0;
    for (int el = 0; el < El; el++) {
        int64_t n = 0;
        for (int s = 0; s < N; s++) n += kept_of(cnt, E, s, e0 + el, cap);
        own_off[el + 1] = own_off[el] + (int32_t)n;
        own_tile_off[el + 1] = own_tile_off[el] + (int32_t)((n + JT_TILE_ROWS - 1) / JT_TILE_ROWS);
    }
    /* received rows: source segments in rank order, each sorted by expert.
     * gather[(s*El + el)*4 + {0,1,2}] = {first received row, first owned
     * row, rows} of expert e0+el from source s. */
    int64_t seg = 0;
    for (int s = 0; s < N; s++) {
        int64_t src = seg;
        for (int el = 0; el < El; el++) {
            const int e = e0 + el;
            int64_t dst = own_off[el];
            for (int s2 = 0; s2 < s; s2++) dst += kept_of(cnt, E, s2, e, cap);
            const int64_t n = kept_of(cnt, E, s, e, cap);
            int32_t *g = gather + ((size_t)s * El + el) * 4;
            g[0] = (int32_t)src;
            g[1] = (int32_t)dst;
            g[2] = (int32_t)n;
            g[3] = 0;
            src += n;
        }
        seg += recv_cnt[s];
    }
    return JT_OK;
}
