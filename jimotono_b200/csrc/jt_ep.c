/* jt_ep.c - expert-parallel MoE layer over NCCL (one process per GPU).
 *
 * Rank r of N holds tokens [r*T, (r+1)*T) of the global batch (T per rank,
 * the same on every rank) and the routed experts [r*E/N, (r+1)*E/N); the
 * shared experts are replicated.  One forward:
 *
 *   1. top-k routing of the local tokens (routing.c:16-76), local counts
 *      per expert, NCCL all-gather of the counts;
 *   2. the global capacity decision (moe_layer.c:931-970) from the gathered
 *      counts (jt_ep_layout.c), local stable sort with the other ranks'
 *      pairs as a per-expert base, drop + renormalization at the source
 *      (moe_layer.c:1171-1201);
 *   3. per-token int8 quantization; each token's codes sent ONCE to every
 *      owner holding at least one of its routed slots, plus 16 bytes of
 *      metadata per kept (token, slot) pair {scale, weight, token row};
 *   4. on the owner: pairs expanded into expert-contiguous rows (codes
 *      copied from the received token row), routed gate/up + SwiGLU +
 *      requant, down projection adding each pair's weighted fp32 row into
 *      the row of its token: one summed row per received token;
 *   5. token rows sent back to their sources and added, owner by owner in
 *      rank order, into the layer output, which already holds the shared
 *      experts' contribution of the local tokens.
 *
 * Sending tokens instead of pairs divides both exchanges by the mean number
 * of a token's slots that land on one owner (about k/N for k >= N).
 *
 * The host learns the exchange sizes from the gathered counts (one
 * device-to-host copy per forward, waited on through an event while the
 * token quantization and the shared experts, which need no layout, run on
 * the device); everything else is stream-ordered.  No device-side remote loads, no multicast.
 */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"
#include "jt_nccl.h"

void jt_set_last_error(const char *what, int code);

struct jt_b200_ep_comm {
    jt_nccl_comm comm;
    int nranks, rank, dev;
    int timeout_ms; /* deadline of the forward's host wait */
    int failed;     /* aborted by the watchdog */
};

struct jt_b200_moe_ep_plan {
    jt_b200_moe_dims dm; /* T = tokens per rank, E = global experts */
    jt_b200_ep_comm *comm;
    int El, R_max, cap;
    void *arena;
    size_t arena_bytes;
    /* local routing and dispatch */
    int32_t *ids, *perm, *pos, *hist, *off, *tile_off, *meta;
    int4 *tiles;
    float4 *row_meta, *sh_meta;
    float *w_raw, *w_fin, *xs, *hs_s, *y32;
    uint8_t *drop;
    int8_t *xq, *hq_s;
    uint16_t *hb_s;   /* shared experts' SwiGLU output, bf16 [T][fs] */
    float *g32, *u32; /* shared gate / up in fp32 [min(T, 255)][fs] (T < 256 only) */
    /* exchange: cnt = E expert counts then N token-row counts */
    int32_t *cnt, *cnt_all, *gbase, *own_off, *own_tile_off, *trow, *tsoff;
    int4 *gather, *own_tiles, *own_sub_tiles; /* JT_TILE_ROWS- / JT_SUB_ROWS-row token tiles */
    int32_t *own_nsub;
    int8_t *send_tok, *rtok;
    uint16_t *own_h; /* owned pairs' routed SwiGLU output, bf16 */
    uint16_t *own_x; /* owned pairs' token rows, fp16, expert order (jtk_ep_gather) */
    float4 *rmeta, *own_meta;
    float *ret, *back;
    int R_tok; /* received token rows capacity (T * N) */
    cudaEvent_t ev_counts; /* the gathered counts reached the host buffer */
    /* host (pinned) */
    int32_t *h_ext, *h_cnt_all, *h_gbase, *h_send, *h_recv, *h_own_off, *h_own_tile_off, *h_gather;
    int32_t *h_tsend, *h_trecv, *h_tsoff;
};

static size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

static int nccl_fail(const char *what, int r) {
    const jt_nccl_api *nc = jt_nccl();
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, nc ? nc->error_string(r) : "nccl unavailable");
    jt_set_last_error(buf, 0);
    errno = EIO;
    return JT_ERR_CUDA;
}

int jt_b200_ep_unique_id(void *id128) {
    const jt_nccl_api *nc = jt_nccl();
    if (id128 == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (nc == NULL) {
        jt_set_last_error("libnccl.so.2 not found", 0);
        errno = ENOSYS;
        return JT_ERR_NOSUP;
    }
    jt_nccl_id id;
    const int r = nc->get_unique_id(&id);
    if (r != 0) return nccl_fail("ncclGetUniqueId", r);
    memcpy(id128, &id, sizeof id);
    return JT_OK;
}

int jt_b200_ep_comm_create(const void *id128, int nranks, int rank, jt_b200_ep_comm **out) {
    if (id128 == NULL || out == NULL || nranks <= 0 || rank < 0 || rank >= nranks) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const jt_nccl_api *nc = jt_nccl();
    if (nc == NULL) {
        jt_set_last_error("libnccl.so.2 not found", 0);
        errno = ENOSYS;
        return JT_ERR_NOSUP;
    }
    jt_b200_ep_comm *c = (jt_b200_ep_comm *)calloc(1, sizeof *c);
    if (c == NULL) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    jt_nccl_id id;
    memcpy(&id, id128, sizeof id);
    if (cudaGetDevice(&c->dev) != cudaSuccess) {
        free(c);
        errno = EIO;
        return JT_ERR_CUDA;
    }
    const int r = nc->comm_init_rank(&c->comm, nranks, id, rank);
    if (r != 0) {
        free(c);
        return nccl_fail("ncclCommInitRank", r);
    }
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_ms = 60000;
    const char *env = getenv("JT_B200_EP_TIMEOUT_MS");
    if (env && atoi(env) > 0) c->timeout_ms = atoi(env);
    *out = c;
    return JT_OK;
}

int jt_b200_ep_comm_set_timeout(jt_b200_ep_comm *c, int timeout_ms) {
    if (c == NULL || timeout_ms <= 0) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    c->timeout_ms = timeout_ms;
    return JT_OK;
}

int jt_b200_ep_comm_failed(const jt_b200_ep_comm *c) { return c != NULL && c->failed; }

/* watchdog operations of one forward: the counts' event, the communicator */
typedef struct {
    cudaEvent_t ev;
    jt_b200_ep_comm *c;
} wd_ctx;

static int wd_done(void *p) {
    const cudaError_t e = cudaEventQuery(((wd_ctx *)p)->ev);
    return e == cudaSuccess ? 1 : (e == cudaErrorNotReady ? 0 : -1);
}

static int wd_async_error(void *p) {
    const jt_nccl_api *nc = jt_nccl();
    int err = 0;
    if (nc && nc->comm_get_async_error && nc->comm_get_async_error(((wd_ctx *)p)->c->comm, &err) != 0)
        return 1;
    return err != 0 && err != 7; /* 7: ncclInProgress */
}

static void wd_abort(void *p) {
    jt_b200_ep_comm *c = ((wd_ctx *)p)->c;
    const jt_nccl_api *nc = jt_nccl();
    if (nc && nc->comm_abort && c->comm) nc->comm_abort(c->comm);
    c->comm = NULL; /* aborted: destroy must not touch it again */
    c->failed = 1;
}

int jt_b200_ep_comm_destroy(jt_b200_ep_comm *c) {
    if (c == NULL) return JT_OK;
    const jt_nccl_api *nc = jt_nccl();
    if (nc && c->comm) nc->comm_destroy(c->comm);
    free(c);
    return JT_OK;
}

int jt_b200_moe_ep_plan_create(const jt_b200_moe_dims *dims, jt_b200_ep_comm *comm,
                               jt_b200_moe_ep_plan **out) {
    if (dims == NULL || comm == NULL || out == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const int N = comm->nranks;
    if (dims->T <= 0 || dims->d <= 0 || dims->d % 128 || dims->f <= 0 || dims->f % 128 ||
        dims->E <= 0 || dims->E > 4096 || dims->E % N || dims->k <= 0 || dims->k > dims->E ||
        dims->k > 64 || dims->S < 0 || dims->S > 8 || (dims->S > 0 && (dims->fs <= 0 || dims->fs % 128)) ||
        !(dims->cap_factor >= 1.0f && dims->cap_factor <= 1.5f)) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    jt_b200_moe_ep_plan *p = (jt_b200_moe_ep_plan *)calloc(1, sizeof *p);
    if (p == NULL) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    p->dm = *dims;
    p->comm = comm;
    p->El = dims->E / N;
    const long long Tg = (long long)dims->T * N;
    p->cap = jt_b200_ep_capacity(Tg, dims->k, dims->E, dims->cap_factor);
    if (p->cap <= 0) {
        free(p);
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    long long rmax = (long long)p->El * p->cap;
    if (rmax > Tg * dims->k) rmax = Tg * dims->k;
    p->R_max = (int)rmax;
    const size_t T = (size_t)dims->T, k = (size_t)dims->k, E = (size_t)dims->E, El = (size_t)p->El;
    const size_t d = (size_t)dims->d, f = (size_t)dims->f, R = (size_t)p->R_max;
    const size_t fs = dims->S > 0 ? (size_t)dims->fs : 64;
    const size_t Tk = T * k, nch = (size_t)jtk_sort_chunks(dims->T), Nn = (size_t)N;
    const size_t Tdst = T * (Nn < k ? Nn : k); /* token rows sent: <= min(N, k) per token */
    p->R_tok = (int)(T * Nn);
    const size_t RT = (size_t)p->R_tok;
    struct {
        void **dst;
        size_t bytes;
    } parts[] = {
        {(void **)&p->ids, Tk * 4},          {(void **)&p->perm, Tk * 4},
        {(void **)&p->pos, Tk * 4},          {(void **)&p->hist, nch * E * 4},
        {(void **)&p->off, (E + 1) * 4},     {(void **)&p->tile_off, (E + 1) * 4},
        {(void **)&p->meta, 64},
        {(void **)&p->tiles, (Tk / JT_TILE_ROWS + E + 1) * 16},
        {(void **)&p->row_meta, Tk * 16},    {(void **)&p->sh_meta, T * 16},
        {(void **)&p->w_raw, Tk * 4},        {(void **)&p->w_fin, Tk * 4},
        {(void **)&p->xs, T * 4},            {(void **)&p->hs_s, T * 4},
        {(void **)&p->hb_s, T * fs * 2},
        {(void **)&p->g32, (T < 255 ? T : 255) * fs * 4}, {(void **)&p->u32, (T < 255 ? T : 255) * fs * 4},
        {(void **)&p->y32, T * d * 4},       {(void **)&p->drop, Tk},
        {(void **)&p->xq, T * d},            {(void **)&p->send_tok, Tdst * d},
        {(void **)&p->hq_s, T * fs},
        {(void **)&p->cnt, (E + Nn) * 4},    {(void **)&p->cnt_all, Nn * (E + Nn) * 4},
        {(void **)&p->trow, T * Nn * 4},     {(void **)&p->tsoff, (Nn + 1) * 4},
        {(void **)&p->gbase, E * 4},         {(void **)&p->own_off, (El + 1) * 4},
        {(void **)&p->own_tile_off, (El + 1) * 4},
        {(void **)&p->gather, Nn * El * 16}, {(void **)&p->own_tiles, (R / JT_TILE_ROWS + El + 1) * 16},
        {(void **)&p->own_sub_tiles, (R / JT_SUB_ROWS + El + 1) * 16}, {(void **)&p->own_nsub, 16},
        {(void **)&p->rtok, RT * d},         {(void **)&p->own_x, R * d * 2},
        {(void **)&p->own_h, R * f * 2},     {(void **)&p->rmeta, R * 16},
        {(void **)&p->own_meta, R * 16},
        {(void **)&p->ret, RT * d * 4},      {(void **)&p->back, Tdst * d * 4},
    };
    const size_t nparts = sizeof(parts) / sizeof(parts[0]);
    size_t total = 0;
    for (size_t i = 0; i < nparts; i++) total += align_up(parts[i].bytes);
    if (cudaMalloc(&p->arena, total) != cudaSuccess) {
        cudaGetLastError();
        free(p);
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    /* zero once: rows past the kept counts are read by full token tiles */
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
    const size_t hbytes = (Nn * (E + Nn) + Nn * E + E + 2 * Nn + 2 * (El + 1) + Nn * El * 4 +
                           3 * (Nn + 1)) * sizeof(int32_t);
    int32_t *h = NULL;
    if (cudaMallocHost((void **)&h, hbytes) != cudaSuccess) {
        cudaFree(p->arena);
        free(p);
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    p->h_ext = h;
    p->h_cnt_all = p->h_ext + Nn * (E + Nn);
    p->h_gbase = p->h_cnt_all + Nn * E;
    p->h_send = p->h_gbase + E;
    p->h_recv = p->h_send + Nn;
    p->h_own_off = p->h_recv + Nn;
    p->h_own_tile_off = p->h_own_off + El + 1;
    p->h_gather = p->h_own_tile_off + El + 1;
    p->h_tsend = p->h_gather + Nn * El * 4;
    p->h_trecv = p->h_tsend + Nn + 1;
    p->h_tsoff = p->h_trecv + Nn + 1;
    if (cudaEventCreateWithFlags(&p->ev_counts, cudaEventDisableTiming) != cudaSuccess) {
        cudaFreeHost(h);
        cudaFree(p->arena);
        free(p);
        errno = EIO;
        return JT_ERR_CUDA;
    }
    *out = p;
    return JT_OK;
}

int jt_b200_moe_ep_plan_destroy(jt_b200_moe_ep_plan *p) {
    if (p == NULL) return JT_OK;
    if (p->ev_counts) cudaEventDestroy(p->ev_counts);
    cudaFree(p->arena);
    cudaFreeHost(p->h_ext);
    free(p);
    return JT_OK;
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

#define CUDA(expr)                                                            \
    do {                                                                      \
        if ((expr) != cudaSuccess) {                                          \
            jt_set_last_error(#expr, -4);                                     \
            errno = EIO;                                                      \
            return JT_ERR_CUDA;                                               \
        }                                                                     \
    } while (0)

#define NCCL(expr)                                                            \
    do {                                                                      \
        int _r = (expr);                                                      \
        if (_r != 0) return nccl_fail(#expr, _r);                             \
    } while (0)

int jt_b200_moe_ep_forward(jt_b200_moe_ep_plan *p, const jt_b200_moe_weights *w, const float *x,
                           const float *logits, const float *bias, void *y, int y_bf16,
                           void *stream) {
    if (p == NULL || w == NULL || x == NULL || logits == NULL || y == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const jt_nccl_api *nc = jt_nccl();
    if (nc == NULL) {
        errno = ENOSYS;
        return JT_ERR_NOSUP;
    }
    const jt_b200_moe_dims *dm = &p->dm;
    const int T = dm->T, k = dm->k, E = dm->E, d = dm->d, f = dm->f, S = dm->S, fs = dm->fs;
    const int N = p->comm->nranks, rank = p->comm->rank, El = p->El;
    if (!w->wg || !w->wu || !w->sg || !w->su || !w->wd || !w->sd ||
        (S > 0 && (!w->wsg || !w->wsu || !w->ssg || !w->ssu || !w->wsd || !w->ssd))) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (p->comm->failed) {
        jt_set_last_error("expert-parallel communicator aborted by the watchdog", 0);
        errno = EIO;
        return JT_ERR_CUDA;
    }
    cudaStream_t st = (cudaStream_t)stream;
    jt_nccl_comm comm = p->comm->comm;
    float *yf = y_bf16 ? p->y32 : (float *)y;

    /* 1. routing, the expert counts and the token-row counts of every rank */
    LAUNCH(jtk_route_topk(logits, bias, T, E, k, p->ids, p->w_raw, st));
    LAUNCH(jtk_ep_count(p->ids, T * k, E, p->cnt, st));
    LAUNCH(jtk_ep_tokens(p->ids, T, k, El, N, p->trow, p->cnt + E, st));
    NCCL(nc->all_gather(p->cnt, p->cnt_all, (size_t)(E + N), JT_NCCL_INT32, comm, st));
    CUDA(cudaMemcpyAsync(p->h_ext, p->cnt_all, (size_t)N * (E + N) * sizeof(int32_t),
                         cudaMemcpyDeviceToHost, st));
    CUDA(cudaEventRecord(p->ev_counts, st));

    /* the quantization and the shared experts need no exchange layout: they
     * run while the host waits for the counts and computes the layout */
    LAUNCH(jtk_quant_dispatch(x, T, d, k, NULL, p->w_raw, p->xq, p->xs, NULL, NULL,
                              S > 0 ? p->sh_meta : NULL, st));
    if (S > 0) {
        LAUNCH(jtk_moe_shared(w->wsg, w->wsu, w->ssg, w->ssu, w->wsd, w->ssd, S, fs, d, p->xq, p->xs,
                              p->sh_meta, T, p->hb_s, p->hq_s, p->hs_s, p->g32, p->u32, yf, st));
    } else {
        CUDA(cudaMemsetAsync(yf, 0, (size_t)T * d * sizeof(float), st));
    }
    {   /* bounded wait for the gathered counts (jt_watchdog.c) */
        wd_ctx wc = {p->ev_counts, p->comm};
        const jt_watchdog_ops ops = {wd_done, wd_async_error, wd_abort, &wc};
        const int wr = jt_watchdog_wait(&ops, p->comm->timeout_ms, NULL);
        if (wr != JT_WD_DONE) {
            jt_set_last_error(wr == JT_WD_TIMEOUT ? "expert counts all-gather: deadline passed, communicator aborted"
                                                  : "expert counts all-gather: NCCL error, communicator aborted",
                              wr);
            errno = wr == JT_WD_TIMEOUT ? ETIMEDOUT : EIO;
            return JT_ERR_CUDA;
        }
    }
    for (int s = 0; s < N; s++)
        memcpy(p->h_cnt_all + (size_t)s * E, p->h_ext + (size_t)s * (E + N), (size_t)E * sizeof(int32_t));

    /* 2. global capacity decision, exchange layout */
    if (jt_b200_ep_layout(p->h_cnt_all, N, E, rank, p->cap, p->h_gbase, p->h_send, p->h_recv,
                          p->h_own_off, p->h_own_tile_off, p->h_gather) != JT_OK)
        return JT_ERR_INVAL;
    /* token rows: sent to owner o = ext[rank][E + o], received from source
     * s = ext[s][E + rank]; gather entries carry their source's first
     * received token row */
    long long tsoff[64 + 1], rtoff[64 + 1];
    if (N > 64) return JT_ERR_INVAL;
    tsoff[0] = rtoff[0] = 0;
    for (int i = 0; i < N; i++) {
        p->h_tsend[i] = p->h_ext[(size_t)rank * (E + N) + E + i];
        p->h_trecv[i] = p->h_ext[(size_t)i * (E + N) + E + rank];
        tsoff[i + 1] = tsoff[i] + p->h_tsend[i];
        rtoff[i + 1] = rtoff[i] + p->h_trecv[i];
        p->h_tsoff[i] = (int32_t)tsoff[i];
    }
    if (rtoff[N] > p->R_tok) {
        jt_set_last_error("expert-parallel received token rows exceed the plan capacity", 0);
        errno = ERANGE;
        return JT_ERR_INVAL;
    }
    for (int s = 0; s < N; s++)
        for (int el = 0; el < El; el++) p->h_gather[((size_t)s * El + el) * 4 + 3] = (int32_t)rtoff[s];
    CUDA(cudaMemcpyAsync(p->gbase, p->h_gbase, (size_t)E * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    CUDA(cudaMemcpyAsync(p->own_off, p->h_own_off, (size_t)(El + 1) * sizeof(int32_t),
                         cudaMemcpyHostToDevice, st));
    CUDA(cudaMemcpyAsync(p->own_tile_off, p->h_own_tile_off, (size_t)(El + 1) * sizeof(int32_t),
                         cudaMemcpyHostToDevice, st));
    CUDA(cudaMemcpyAsync(p->gather, p->h_gather, (size_t)N * El * 4 * sizeof(int32_t),
                         cudaMemcpyHostToDevice, st));
    CUDA(cudaMemcpyAsync(p->tsoff, p->h_tsoff, (size_t)N * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    LAUNCH(jtk_moe_sort(p->ids, p->w_raw, T, k, E, p->cap, p->gbase, p->hist, p->off, p->tile_off,
                        p->tiles, p->meta, p->perm, p->pos, p->drop, p->w_fin, st));

    /* 3. the send buffers: token rows per owner and the kept pairs'
     * metadata in send (expert) order */
    LAUNCH(jtk_ep_pack(p->xq, p->xs, T, d, k, El, N, p->ids, p->pos, p->w_fin, p->trow, p->tsoff,
                       p->send_tok, p->row_meta, st));

    /* dispatch: token rows and pair metadata to the experts' owners */
    long long soff[64 + 1], roff[64 + 1];
    soff[0] = roff[0] = 0;
    for (int i = 0; i < N; i++) {
        soff[i + 1] = soff[i] + p->h_send[i];
        roff[i + 1] = roff[i] + p->h_recv[i];
    }
    if (roff[N] > p->R_max) {
        jt_set_last_error("expert-parallel receive rows exceed the plan capacity", 0);
        errno = ERANGE;
        return JT_ERR_INVAL;
    }
    NCCL(nc->group_start());
    for (int o = 0; o < N; o++) {
        if (p->h_tsend[o])
            NCCL(nc->send(p->send_tok + (size_t)tsoff[o] * d, (size_t)p->h_tsend[o] * d, JT_NCCL_INT8, o, comm, st));
        if (p->h_send[o])
            NCCL(nc->send(p->row_meta + soff[o], (size_t)p->h_send[o] * 4, JT_NCCL_FLOAT32, o, comm, st));
        if (p->h_trecv[o])
            NCCL(nc->recv(p->rtok + (size_t)rtoff[o] * d, (size_t)p->h_trecv[o] * d, JT_NCCL_INT8, o, comm, st));
        if (p->h_recv[o])
            NCCL(nc->recv(p->rmeta + roff[o], (size_t)p->h_recv[o] * 4, JT_NCCL_FLOAT32, o, comm, st));
    }
    NCCL(nc->group_end());

    /* 4. owned experts; each pair's weighted row is added into its token's
     * returned row */
    const int own_rows = p->h_own_off[El];
    const int own_tiles = p->h_own_tile_off[El];
    if (rtoff[N] > 0)
        CUDA(cudaMemsetAsync(p->ret, 0, (size_t)rtoff[N] * d * sizeof(float), st));
    if (own_rows > 0) {
        LAUNCH(jtk_ep_gather(p->gather, N * El, p->rtok, p->rmeta, d, p->own_x, p->own_meta, st));
        LAUNCH(jtk_build_tiles(p->own_off, p->own_tile_off, El, p->own_tiles, st));
        LAUNCH(jtk_split_tiles(p->own_tiles, p->own_tile_off + El, p->own_sub_tiles, p->own_nsub, st));
        /* each JT_TILE_ROWS-row tile is at most two JT_SUB_ROWS-row ones */
        const int gu_hint = 2 * own_tiles * (f / 128), dn_hint = own_tiles * ((d + 255) / 256);
        LAUNCH(jtk_moe_gateup_routed(w->wg, w->wu, w->sg, w->su, El, f, d, p->own_x, p->R_max,
                                     p->own_meta, p->own_sub_tiles, p->own_nsub, p->own_h, gu_hint, st));
        LAUNCH(jtk_moe_down_routed(w->wd, w->sd, El, d, f, p->own_h, p->R_max, p->own_meta,
                                   p->own_tiles, p->own_tile_off + El, p->ret, 1, dn_hint, st));
    }

    /* 5. combine: token rows back to their sources, added into y */
    NCCL(nc->group_start());
    for (int o = 0; o < N; o++) {
        if (p->h_trecv[o])
            NCCL(nc->send(p->ret + (size_t)rtoff[o] * d, (size_t)p->h_trecv[o] * d, JT_NCCL_FLOAT32, o, comm, st));
        if (p->h_tsend[o])
            NCCL(nc->recv(p->back + (size_t)tsoff[o] * d, (size_t)p->h_tsend[o] * d, JT_NCCL_FLOAT32, o, comm, st));
    }
    NCCL(nc->group_end());
    LAUNCH(jtk_ep_combine(p->trow, p->tsoff, T, N, p->back, d, yf, st));
    if (y_bf16) LAUNCH(jtk_f32_to_bf16(yf, (uint16_t *)y, (size_t)T * d, st));
    return JT_OK;
}

int jt_b200_moe_ep_debug_copy(jt_b200_moe_ep_plan *p, int what, void *host_dst, size_t bytes) {
    if (p == NULL || host_dst == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t Tk = (size_t)p->dm.T * p->dm.k;
    const void *src = NULL;
    size_t have = 0;
    switch (what) {
    case JT_B200_DBG_IDS: src = p->ids; have = Tk * 4; break;
    case JT_B200_DBG_WEIGHTS: src = p->w_fin; have = Tk * 4; break;
    case JT_B200_DBG_DROP: src = p->drop; have = Tk; break;
    case JT_B200_DBG_XQ: src = p->xq; have = (size_t)p->dm.T * p->dm.d; break;
    case JT_B200_DBG_XS: src = p->xs; have = (size_t)p->dm.T * 4; break;
    case JT_B200_DBG_PERM: src = p->perm; have = Tk * 4; break;
    case JT_B200_DBG_H: src = p->own_h; have = (size_t)p->R_max * p->dm.f * 2; break;
    case JT_B200_DBG_META: {
        /* kept local pairs, owned rows, owned token tiles, capacity */
        int32_t m[4] = {0, 0, 0, p->cap};
        for (int i = 0; i < p->comm->nranks; i++) m[0] += p->h_send[i];
        m[1] = p->h_own_off[p->El];
        m[2] = p->h_own_tile_off[p->El];
        if (bytes > sizeof m) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
        memcpy(host_dst, m, bytes);
        return JT_OK;
    }
    default: errno = EINVAL; return JT_ERR_INVAL;
    }
    if (bytes > have) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    if (cudaMemcpy(host_dst, src, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}
