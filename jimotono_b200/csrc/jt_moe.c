/* jt_moe.c - C11 host runtime of the quantized MoE layer on the B200.
 *
 * A plan owns the device workspace of one layer shape (allocated once, so a
 * forward call allocates nothing) and enqueues the layer as a fixed chain of
 * kernels on the caller's stream:
 *
 *   1. top-k + softmax over the router logits        (routing.c:16-76)
 *   2. stable capacity sort, drop, renormalization   (moe_layer.c:895-978, :1171-1201)
 *   3. per-token int8 quantization + dispatch of each kept (token, slot)
 *      row into expert order                         (w8a8.c:688-747, moe_layer.c:1283-1288)
 *   4. shared experts: gate/up + SwiGLU + requant, down (stores, then adds)
 *                                                     (moe_layer.c:1469-1560)
 *   5. routed experts: grouped gate/up + SwiGLU + requant, grouped down
 *      with the weighted combine fused into its epilogue
 *                                                     (moe_layer.c:1265-1463)
 *   6. optional fp32 -> bf16 of the layer output.
 *
 * Every kernel is sized from device-side counts (kept pairs, per-expert token
 * tiles), so the host never waits for the routing result. */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <stdio.h>
#include <string.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"

/* Description of the last failed launch (per thread): which launcher and
 * the CUDA runtime's message. */
static _Thread_local char g_last_error[512];

void jt_set_last_error(const char *what, int code) {
    const cudaError_t e = cudaPeekAtLastError();
    snprintf(g_last_error, sizeof(g_last_error), "%.300s -> %d (%s)", what, code,
             cudaGetErrorString(e));
}

const char *jt_b200_last_error(void) { return g_last_error; }

struct jt_b200_moe_plan {
    jt_b200_moe_dims dm;
    int dev;
    void *arena;
    size_t arena_bytes;
    int32_t *ids, *perm, *pos, *hist, *off, *tile_off, *meta;
    int4 *tiles;     /* JT_TILE_ROWS-row token tiles (routed down) */
    int4 *sub_tiles; /* JT_SUB_ROWS-row token tiles (routed gate/up) */
    int32_t *nsub;   /* entries of sub_tiles */
    float4 *row_meta, *sh_meta;
    float *w_raw, *w_fin, *xs, *hs_s, *y32;
    uint8_t *drop;
    int8_t *xq, *hq_s;
    uint16_t *hb_s;    /* shared experts' SwiGLU output, bf16 [T][fs] */
    float *g32, *u32;  /* shared gate / up in fp32 [min(T, 255)][fs] (T < 256 only) */
    uint16_t *h;  /* routed SwiGLU output, bf16 [kept][f] */
    uint16_t *xd; /* kept token rows, fp16, expert order (jtk_quant_dispatch) */
    /* batch-1 path: h codes and scales of every shared expert at once */
    uint16_t *hb_d;    /* batch-1 path: shared h of every shared expert, bf16 [S][fs] */
    int32_t *dec_acc, *dec_cnt; /* K-split partial dots of the shared experts (zero between calls) */
    /* optional per-stage profiling: events[step][JT_B200_MOE_NSTAGE + 1] */
    cudaEvent_t *prof_ev;
    int prof_max, prof_used;
};

/* Row stride (floats) of the per-(row, 64-channel group) h scales: padded to
 * 16 bytes so a token tile's scales are one TMA box. */

static size_t align_up(size_t v) { return (v + 255u) & ~(size_t)255u; }

static int dims_valid(const jt_b200_moe_dims *d) {
    if (d->T <= 0 || d->d <= 0 || d->f <= 0) return 0;
    if (d->d % 128 || d->f % 128 || d->f > 4096) return 0;
    if (d->E <= 0 || d->E > 4096 || d->k <= 0 || d->k > d->E || d->k > 64) return 0;
    if (d->S < 0 || d->S > 8) return 0;
    if (d->S > 0 && (d->fs <= 0 || d->fs % 128 || d->fs > 4096)) return 0;
    if (!(d->cap_factor >= 1.0f) || !(d->cap_factor <= 1.5f) || !isfinite((double)d->cap_factor))
        return 0;
    return 1;
}

int jt_b200_moe_plan_create(const jt_b200_moe_dims *dims, jt_b200_moe_plan **out) {
    if (dims == NULL || out == NULL || !dims_valid(dims)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    jt_b200_moe_plan *p = (jt_b200_moe_plan *)calloc(1, sizeof(*p));
    if (!p) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    p->dm = *dims;
    const size_t T = (size_t)dims->T, k = (size_t)dims->k, E = (size_t)dims->E;
    const size_t d = (size_t)dims->d, f = (size_t)dims->f;
    const size_t fs = dims->S > 0 ? (size_t)dims->fs : 64;
    const size_t Tk = T * k;
    const size_t nch = (size_t)jtk_sort_chunks(dims->T);
    const size_t max_tiles = Tk / JT_TILE_ROWS + E + 1;
    struct {
        void **dst;
        size_t bytes;
    } parts[] = {
        {(void **)&p->ids, Tk * 4},          {(void **)&p->perm, Tk * 4},
        {(void **)&p->pos, Tk * 4},          {(void **)&p->hist, nch * E * 4},
        {(void **)&p->off, (E + 1) * 4},     {(void **)&p->tile_off, (E + 1) * 4},
        {(void **)&p->meta, 64},
        {(void **)&p->tiles, max_tiles * 16},
        {(void **)&p->sub_tiles, (Tk / JT_SUB_ROWS + E + 1) * 16}, {(void **)&p->nsub, 16},
        {(void **)&p->row_meta, Tk * 16},    {(void **)&p->sh_meta, T * 16},
        {(void **)&p->w_raw, Tk * 4},        {(void **)&p->w_fin, Tk * 4},
        {(void **)&p->xs, T * 4},
        {(void **)&p->hs_s, T * 4},
        {(void **)&p->hb_s, T * fs * 2},
        {(void **)&p->g32, (T < 255 ? T : 255) * fs * 4}, {(void **)&p->u32, (T < 255 ? T : 255) * fs * 4},
        {(void **)&p->y32, T * d * 4},       {(void **)&p->drop, Tk},
        {(void **)&p->xq, T * d},            {(void **)&p->xd, Tk * d * 2},
        {(void **)&p->h, Tk * f * 2},        {(void **)&p->hq_s, T * fs},
        {(void **)&p->hb_d, (size_t)(dims->S > 0 ? dims->S : 1) * fs * 2},
        {(void **)&p->dec_acc, (size_t)(dims->S > 0 ? dims->S : 1) * 2 * fs * 4},
        {(void **)&p->dec_cnt, (size_t)(dims->S > 0 ? dims->S : 1) * (fs / 64) * 4},
    };
    const size_t nparts = sizeof(parts) / sizeof(parts[0]);
    size_t total = 0;
    for (size_t i = 0; i < nparts; i++) total += align_up(parts[i].bytes);
    if (cudaGetDevice(&p->dev) != cudaSuccess || cudaMalloc(&p->arena, total) != cudaSuccess) {
        cudaGetLastError();
        free(p);
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    /* Zero once: rows past the kept count are read by full token tiles. */
    if (cudaMemset(p->arena, 0, total) != cudaSuccess) {
        cudaFree(p->arena);
        free(p);
        errno = EIO;
        return JT_ERR_CUDA;
    }
    p->arena_bytes = total;
    size_t offb = 0;
    for (size_t i = 0; i < nparts; i++) {
        *parts[i].dst = (char *)p->arena + offb;
        offb += align_up(parts[i].bytes);
    }
    *out = p;
    return JT_OK;
}

static void prof_free(jt_b200_moe_plan *p) {
    if (!p->prof_ev) return;
    for (int i = 0; i < p->prof_max * (JT_B200_MOE_NSTAGE + 1); i++) cudaEventDestroy(p->prof_ev[i]);
    free(p->prof_ev);
    p->prof_ev = NULL;
    p->prof_max = p->prof_used = 0;
}

int jt_b200_moe_profile_begin(jt_b200_moe_plan *plan, int max_steps) {
    if (plan == NULL || max_steps <= 0 || max_steps > 4096) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    prof_free(plan);
    const int n = max_steps * (JT_B200_MOE_NSTAGE + 1);
    plan->prof_ev = (cudaEvent_t *)calloc((size_t)n, sizeof(cudaEvent_t));
    if (!plan->prof_ev) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    for (int i = 0; i < n; i++) {
        if (cudaEventCreate(&plan->prof_ev[i]) != cudaSuccess) {
            plan->prof_max = i / (JT_B200_MOE_NSTAGE + 1);
            prof_free(plan);
            errno = EIO;
            return JT_ERR_CUDA;
        }
    }
    plan->prof_max = max_steps;
    plan->prof_used = 0;
    return JT_OK;
}

int jt_b200_moe_profile_end(jt_b200_moe_plan *plan, float *stage_ms, int nstage, int *steps) {
    if (plan == NULL || stage_ms == NULL || nstage < JT_B200_MOE_NSTAGE || !plan->prof_ev) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    for (int s = 0; s < JT_B200_MOE_NSTAGE; s++) stage_ms[s] = 0.0f;
    int rc = JT_OK;
    for (int i = 0; i < plan->prof_used && rc == JT_OK; i++) {
        cudaEvent_t *ev = plan->prof_ev + (size_t)i * (JT_B200_MOE_NSTAGE + 1);
        if (cudaEventSynchronize(ev[JT_B200_MOE_NSTAGE]) != cudaSuccess) {
            rc = JT_ERR_CUDA;
            break;
        }
        for (int s = 0; s < JT_B200_MOE_NSTAGE; s++) {
            float ms = 0.0f;
            if (cudaEventElapsedTime(&ms, ev[s], ev[s + 1]) != cudaSuccess) {
                rc = JT_ERR_CUDA;
                break;
            }
            stage_ms[s] += ms;
        }
    }
    if (steps) *steps = plan->prof_used;
    prof_free(plan);
    if (rc != JT_OK) errno = EIO;
    return rc;
}

int jt_b200_moe_plan_destroy(jt_b200_moe_plan *plan) {
    if (plan == NULL) return JT_OK;
    prof_free(plan);
    if (plan->arena) cudaFree(plan->arena);
    free(plan);
    return JT_OK;
}

size_t jt_b200_moe_plan_bytes(const jt_b200_moe_plan *plan) {
    return plan ? plan->arena_bytes : 0;
}

int jt_b200_moe_router_logits(const float *x, const float *wgate, int T, int d, int E,
                              float *logits, void *stream) {
    if (x == NULL || wgate == NULL || logits == NULL || T <= 0 || T > 2097120 || d <= 0 ||
        d % 32 != 0 || E <= 0 || (((uintptr_t)x | (uintptr_t)wgate) & 15u) != 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const int r = jtk_router_logits(x, wgate, T, d, E, logits, (cudaStream_t)stream);
    if (r == -1) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (r != 0) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}

static int weights_valid(const jt_b200_moe_weights *w, int S) {
    if (!w->wg || !w->wu || !w->sg || !w->su || !w->wd || !w->sd) return 0;
    if (S > 0 && (!w->wsg || !w->wsu || !w->ssg || !w->ssu || !w->wsd || !w->ssd)) return 0;
    return 1;
}

#define LAUNCH(expr)                                                          \
    do {                                                                      \
        int _r = (expr);                                                      \
        if (_r != 0) {                                                        \
            jt_set_last_error(#expr, _r);                                     \
            errno = _r == -1 ? EINVAL : EIO;                                  \
            return _r == -1 ? JT_ERR_INVAL : JT_ERR_CUDA;                     \
        }                                                                     \
    } while (0)

int jt_b200_moe_forward(jt_b200_moe_plan *plan, const jt_b200_moe_weights *w, const float *x,
                        const float *logits, const float *bias, int T, void *y, int y_bf16,
                        void *stream) {
    if (plan == NULL || w == NULL || x == NULL || logits == NULL || y == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const jt_b200_moe_dims *dm = &plan->dm;
    if (T <= 0 || T > dm->T || !weights_valid(w, dm->S)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    cudaStream_t st = (cudaStream_t)stream;
    const int k = dm->k, E = dm->E, d = dm->d, f = dm->f, S = dm->S, fs = dm->fs;
    const int rows_cap = dm->T * k;
    /* capacity of moe_layer.c:931-943 (double arithmetic on the host) */
    const double capd = ceil((double)dm->cap_factor * (double)((size_t)T * k) / (double)E);
    if (!isfinite(capd) || capd < 1.0 || capd > 2147483647.0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const int cap = (int)capd;
    int gu_hint = 0, dn_hint = 0;
    float *yf = y_bf16 ? plan->y32 : (float *)y;
    cudaEvent_t *ev = NULL;
    if (plan->prof_ev && plan->prof_used < plan->prof_max)
        ev = plan->prof_ev + (size_t)(plan->prof_used++) * (JT_B200_MOE_NSTAGE + 1);
#define MARK(i) \
    do { \
        if (ev) cudaEventRecord(ev[(i)], st); \
    } while (0)

    MARK(JT_B200_STAGE_ROUTE);
    if (T == 1) {
        /* one token: nothing can be dropped (cap >= 1, k distinct experts);
         * router, gate/up and down as matrix-vector kernels (jt_decode.cu) */
        MARK(JT_B200_STAGE_SORT);
        MARK(JT_B200_STAGE_DISPATCH);
        MARK(JT_B200_STAGE_SHARED);
        MARK(JT_B200_STAGE_GATEUP);
        const int r = jtk_moe_decode(x, logits, bias, plan->ids, plan->w_raw, w->wg, w->wu, w->sg, w->su, w->wd, w->sd,
                                     w->wsg, w->wsu, w->ssg, w->ssu, w->wsd, w->ssd, d, f, E, k, S, fs,
                                     plan->xq, plan->xs, plan->h, plan->hb_d, plan->dec_acc, plan->dec_cnt,
                                     plan->perm, plan->pos, plan->off,
                                     plan->tile_off, plan->meta, plan->drop, plan->w_fin,
                                     y_bf16 ? NULL : (float *)y, y_bf16 ? (uint16_t *)y : NULL, st);
        if (r == 0) {
            MARK(JT_B200_STAGE_DOWN);
            MARK(JT_B200_STAGE_OUTPUT);
            MARK(JT_B200_MOE_NSTAGE);
            return JT_OK;
        }
        if (r != -1) {
            jt_set_last_error("jtk_moe_decode", r);
            errno = EIO;
            return JT_ERR_CUDA;
        }
        /* shape outside the batch-1 kernels: the batched chain below */
    }
    LAUNCH(jtk_route_topk(logits, bias, T, E, k, plan->ids, plan->w_raw, st));
    MARK(JT_B200_STAGE_SORT);
    LAUNCH(jtk_moe_sort(plan->ids, plan->w_raw, T, k, E, cap, NULL, plan->hist, plan->off,
                        plan->tile_off, plan->tiles, plan->meta, plan->perm, plan->pos, plan->drop,
                        plan->w_fin, st));
    LAUNCH(jtk_split_tiles(plan->tiles, plan->tile_off + E, plan->sub_tiles, plan->nsub, st));
    MARK(JT_B200_STAGE_DISPATCH);
    LAUNCH(jtk_quant_dispatch(x, T, d, k, plan->pos, plan->w_fin, plan->xq, plan->xs, plan->xd,
                              plan->row_meta, S > 0 ? plan->sh_meta : NULL, st));
    MARK(JT_B200_STAGE_SHARED);
    if (S > 0) {
        LAUNCH(jtk_moe_shared(w->wsg, w->wsu, w->ssg, w->ssu, w->wsd, w->ssd, S, fs, d, plan->xq, plan->xs,
                              plan->sh_meta, T, plan->hb_s, plan->hq_s, plan->hs_s, plan->g32, plan->u32, yf,
                              st));
    } else {
        if (cudaMemsetAsync(yf, 0, (size_t)T * d * sizeof(float), st) != cudaSuccess) {
            errno = EIO;
            return JT_ERR_CUDA;
        }
    }
    /* Upper bounds of the device-side token-tile counts: every non-empty
     * expert adds at most one partial tile to (kept pairs)/(tile rows) full ones. */
    {
        const long long pairs = (long long)T * k;
        const long long ne = pairs < E ? pairs : E;
        const long long tl = ne + pairs / JT_TILE_ROWS, ts = ne + pairs / JT_SUB_ROWS;
        gu_hint = ts * (f / 128) > 0x7fffffffLL ? 0 : (int)(ts * (f / 128));
        dn_hint = tl * ((d + 255) / 256) > 0x7fffffffLL ? 0 : (int)(tl * ((d + 255) / 256));
    }
    MARK(JT_B200_STAGE_GATEUP);
    LAUNCH(jtk_moe_gateup_routed(w->wg, w->wu, w->sg, w->su, E, f, d, plan->xd, rows_cap,
                                 plan->row_meta, plan->sub_tiles, plan->nsub, plan->h, gu_hint, st));
    MARK(JT_B200_STAGE_DOWN);
    LAUNCH(jtk_moe_down_routed(w->wd, w->sd, E, d, f, plan->h, rows_cap, plan->row_meta, plan->tiles,
                               plan->tile_off + E, yf, 1, dn_hint, st));
    MARK(JT_B200_STAGE_OUTPUT);
    if (y_bf16) LAUNCH(jtk_f32_to_bf16(yf, (uint16_t *)y, (size_t)T * d, st));
    MARK(JT_B200_MOE_NSTAGE);
#undef MARK
    return JT_OK;
}

int jt_b200_moe_debug_copy(jt_b200_moe_plan *plan, int what, void *host_dst, size_t bytes) {
    if (plan == NULL || host_dst == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t T = (size_t)plan->dm.T, k = (size_t)plan->dm.k, E = (size_t)plan->dm.E;
    const size_t d = (size_t)plan->dm.d, f = (size_t)plan->dm.f;
    const void *src = NULL;
    size_t cap = 0;
    switch (what) {
        case JT_B200_DBG_IDS: src = plan->ids; cap = T * k * 4; break;
        case JT_B200_DBG_WEIGHTS: src = plan->w_fin; cap = T * k * 4; break;
        case JT_B200_DBG_PERM: src = plan->perm; cap = T * k * 4; break;
        case JT_B200_DBG_OFF: src = plan->off; cap = (E + 1) * 4; break;
        case JT_B200_DBG_DROP: src = plan->drop; cap = T * k; break;
        case JT_B200_DBG_XQ: src = plan->xq; cap = T * d; break;
        case JT_B200_DBG_XS: src = plan->xs; cap = T * 4; break;
        case JT_B200_DBG_H: src = plan->h; cap = T * k * f * 2; break;
        case JT_B200_DBG_META: src = plan->meta; cap = 16; break;
        default:
            errno = EINVAL;
            return JT_ERR_INVAL;
    }
    if (bytes > cap) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (cudaDeviceSynchronize() != cudaSuccess ||
        cudaMemcpy(host_dst, src, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}
