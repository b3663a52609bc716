/* jt_wfile.c - on-disk form of the prepared MoE weights.
 *
 * The reference keeps fp32 masters and re-derives its quantized forms on
 * every call (moe_layer.c:185-274, lowbit.c:228-237); its expert streaming
 * path (esmoe) reads raw tensors from files.  The prepared layer's packed
 * INT2/INT4 codes, fp16 group scales and int8 shared experts are the form
 * worth storing, so this file defines one:
 *
 *   bytes 0..4095  header, little-endian:
 *     char     magic[8]     "JTB2MOE1"
 *     uint32   version      1
 *     uint32   header_bytes 4096
 *     int32    d, f, E, S, fs
 *     uint32   nfields      12
 *     uint64   offset[12], size[12], fnv1a64[12]   per array, in the field
 *              order of jt_b200_moe_weights (wg wu sg su wd sd wsg wsu ssg
 *              ssu wsd ssd)
 *   then every array at a 4096-byte aligned offset (so a reader can stream
 *   an expert's rows with direct I/O), zero padding between them.
 *
 * The checksum is FNV-1a 64 over each array's bytes; a reader rejects a
 * file whose header does not match the expected dims or whose data does not
 * match its checksums.  Host-pointer forms do the file work; the device
 * forms stage each array through one pinned host buffer. */
#include <errno.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "../../include/jimotono_b200.h"

void jt_set_last_error(const char *what, int code);

#define WF_HDR 4096u
#define WF_ALIGN 4096u
#define WF_N 12
static const char kMagic[8] = {'J', 'T', 'B', '2', 'M', 'O', 'E', '1'};

typedef struct {
    char magic[8];
    uint32_t version, header_bytes;
    int32_t d, f, E, S, fs;
    uint32_t nfields;
    uint64_t offset[WF_N], size[WF_N], fnv[WF_N];
} wf_header;

static uint64_t fnv1a64(uint64_t h, const unsigned char *p, size_t n) {
    for (size_t i = 0; i < n; i++) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}
#define FNV_INIT 14695981039346656037ull

int jt_b200_moe_weights_sizes(const jt_b200_moe_dims *dm, size_t sizes[12]) {
    if (dm == NULL || sizes == NULL || dm->d <= 0 || dm->d % 128 || dm->f <= 0 || dm->f % 128 ||
        dm->E <= 0 || dm->S < 0 || (dm->S > 0 && (dm->fs <= 0 || dm->fs % 128))) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    const size_t E = (size_t)dm->E, d = (size_t)dm->d, f = (size_t)dm->f, S = (size_t)dm->S,
                 fs = dm->S > 0 ? (size_t)dm->fs : 0;
    sizes[0] = sizes[1] = E * f * (d / 4);           /* wg, wu: INT2 [E][f][d/4] */
    sizes[2] = sizes[3] = E * (d / 64) * f * 2;      /* sg, su: fp16 [E][d/64][f] */
    sizes[4] = E * d * (f / 2);                      /* wd: INT4 [E][d][f/2] */
    sizes[5] = E * (f / 64) * d * 2;                 /* sd: fp16 [E][f/64][d] */
    sizes[6] = sizes[7] = S * fs * d;                /* wsg, wsu: int8 [S][fs][d] */
    sizes[8] = sizes[9] = S * fs * 4;                /* ssg, ssu: fp32 [S][fs] */
    sizes[10] = S * d * fs;                          /* wsd: int8 [S][d][fs] */
    sizes[11] = S * d * 4;                           /* ssd: fp32 [S][d] */
    return JT_OK;
}

static uint64_t align_up(uint64_t v) { return (v + WF_ALIGN - 1) / WF_ALIGN * WF_ALIGN; }

static void fill_header(wf_header *h, const jt_b200_moe_dims *dm, const size_t sizes[WF_N]) {
    memset(h, 0, sizeof *h);
    memcpy(h->magic, kMagic, 8);
    h->version = 1;
    h->header_bytes = WF_HDR;
    h->d = dm->d;
    h->f = dm->f;
    h->E = dm->E;
    h->S = dm->S;
    h->fs = dm->S > 0 ? dm->fs : 0;
    h->nfields = WF_N;
    uint64_t off = WF_HDR;
    for (int i = 0; i < WF_N; i++) {
        h->offset[i] = off;
        h->size[i] = sizes[i];
        off = align_up(off + sizes[i]);
    }
}

static int io_fail(const char *what, FILE *fp) {
    if (fp) fclose(fp);
    jt_set_last_error(what, 0);
    errno = EIO;
    return JT_ERR_IO;
}

/* get(i, buf, off, n) provides n bytes of array i starting at byte off. */
typedef int (*wf_get_fn)(void *ctx, int i, void *buf, size_t off, size_t n);
typedef int (*wf_put_fn)(void *ctx, int i, const void *buf, size_t off, size_t n);

static int write_file(const char *path, const jt_b200_moe_dims *dm, wf_get_fn get, void *ctx,
                      unsigned char *buf, size_t bufsz) {
    size_t sizes[WF_N];
    int r = jt_b200_moe_weights_sizes(dm, sizes);
    if (r != JT_OK) return r;
    wf_header h;
    fill_header(&h, dm, sizes);
    FILE *fp = fopen(path, "wb");
    if (fp == NULL) return io_fail("cannot create the weight file", NULL);
    unsigned char zero[WF_ALIGN];
    memset(zero, 0, sizeof zero);
    /* header placeholder first; the checksums are known after the data */
    if (fwrite(zero, 1, WF_HDR, fp) != WF_HDR) return io_fail("write failed", fp);
    uint64_t pos = WF_HDR;
    for (int i = 0; i < WF_N; i++) {
        uint64_t hsum = FNV_INIT;
        for (size_t o = 0; o < sizes[i]; o += bufsz) {
            const size_t n = sizes[i] - o < bufsz ? sizes[i] - o : bufsz;
            if (get(ctx, i, buf, o, n) != 0) {
                fclose(fp);
                errno = EIO;
                return JT_ERR_CUDA;
            }
            hsum = fnv1a64(hsum, buf, n);
            if (fwrite(buf, 1, n, fp) != n) return io_fail("write failed", fp);
        }
        h.fnv[i] = hsum;
        pos += sizes[i];
        const uint64_t pad = (i + 1 < WF_N ? h.offset[i + 1] : align_up(pos)) - pos;
        if (pad && fwrite(zero, 1, (size_t)pad, fp) != pad) return io_fail("write failed", fp);
        pos += pad;
    }
    unsigned char hb[WF_HDR];
    memset(hb, 0, sizeof hb);
    memcpy(hb, &h, sizeof h);
    if (fseek(fp, 0, SEEK_SET) != 0 || fwrite(hb, 1, WF_HDR, fp) != WF_HDR) return io_fail("write failed", fp);
    if (fclose(fp) != 0) return io_fail("close failed", NULL);
    return JT_OK;
}

static int read_file(const char *path, const jt_b200_moe_dims *dm, wf_put_fn put, void *ctx,
                     unsigned char *buf, size_t bufsz) {
    size_t sizes[WF_N];
    int r = jt_b200_moe_weights_sizes(dm, sizes);
    if (r != JT_OK) return r;
    FILE *fp = fopen(path, "rb");
    if (fp == NULL) return io_fail("cannot open the weight file", NULL);
    unsigned char hb[WF_HDR];
    if (fread(hb, 1, WF_HDR, fp) != WF_HDR) return io_fail("truncated header", fp);
    wf_header h, want;
    memcpy(&h, hb, sizeof h);
    fill_header(&want, dm, sizes);
    if (memcmp(h.magic, kMagic, 8) != 0 || h.version != 1 || h.header_bytes != WF_HDR || h.nfields != WF_N ||
        h.d != want.d || h.f != want.f || h.E != want.E || h.S != want.S || h.fs != want.fs ||
        memcmp(h.offset, want.offset, sizeof h.offset) != 0 || memcmp(h.size, want.size, sizeof h.size) != 0) {
        fclose(fp);
        jt_set_last_error("weight file header does not match the layer dims", 0);
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    /* Pass 1 checks every array against its checksum without writing
     * anything; pass 2 copies into the destinations.  So a corrupt or
     * truncated file leaves the caller's arrays untouched.  Pass 2 hashes
     * again and reports a file changed between the passes (the destinations
     * then hold part of the new contents). */
    for (int pass = 0; pass < 2; pass++) {
        for (int i = 0; i < WF_N; i++) {
            if (fseek(fp, (long)h.offset[i], SEEK_SET) != 0) return io_fail("seek failed", fp);
            uint64_t hsum = FNV_INIT;
            for (size_t o = 0; o < sizes[i]; o += bufsz) {
                const size_t n = sizes[i] - o < bufsz ? sizes[i] - o : bufsz;
                if (fread(buf, 1, n, fp) != n) return io_fail("truncated weight file", fp);
                hsum = fnv1a64(hsum, buf, n);
                if (pass == 1 && put(ctx, i, buf, o, n) != 0) {
                    fclose(fp);
                    errno = EIO;
                    return JT_ERR_CUDA;
                }
            }
            if (hsum != h.fnv[i]) {
                fclose(fp);
                jt_set_last_error(pass == 0 ? "weight file checksum mismatch"
                                            : "weight file changed while it was read", 0);
                errno = EIO;
                return JT_ERR_IO;
            }
        }
    }
    fclose(fp);
    return JT_OK;
}

/* ---- host arrays ---- */
static int host_get(void *ctx, int i, void *buf, size_t off, size_t n) {
    const unsigned char *const *a = (const unsigned char *const *)ctx;
    memcpy(buf, a[i] + off, n);
    return 0;
}
static int host_put(void *ctx, int i, const void *buf, size_t off, size_t n) {
    unsigned char *const *a = (unsigned char *const *)ctx;
    memcpy(a[i] + off, buf, n);
    return 0;
}

#define WF_BUF (8u << 20)

int jt_b200_moe_weights_write_host(const char *path, const jt_b200_moe_dims *dims, const void *const arrays[12]) {
    if (path == NULL || arrays == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    size_t sizes[WF_N];
    int r = jt_b200_moe_weights_sizes(dims, sizes);
    if (r != JT_OK) return r;
    for (int i = 0; i < WF_N; i++)
        if (sizes[i] && arrays[i] == NULL) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    unsigned char *buf = (unsigned char *)malloc(WF_BUF);
    if (buf == NULL) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    r = write_file(path, dims, host_get, (void *)arrays, buf, WF_BUF);
    free(buf);
    return r;
}

int jt_b200_moe_weights_read_host(const char *path, const jt_b200_moe_dims *dims, void *const arrays[12]) {
    if (path == NULL || arrays == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    size_t sizes[WF_N];
    int r = jt_b200_moe_weights_sizes(dims, sizes);
    if (r != JT_OK) return r;
    for (int i = 0; i < WF_N; i++)
        if (sizes[i] && arrays[i] == NULL) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    unsigned char *buf = (unsigned char *)malloc(WF_BUF);
    if (buf == NULL) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    r = read_file(path, dims, host_put, (void *)arrays, buf, WF_BUF);
    free(buf);
    return r;
}

/* ---- device arrays (the fields of jt_b200_moe_weights) ---- */
static void fields_of(const jt_b200_moe_weights *w, const void *a[WF_N]) {
    a[0] = w->wg, a[1] = w->wu, a[2] = w->sg, a[3] = w->su, a[4] = w->wd, a[5] = w->sd;
    a[6] = w->wsg, a[7] = w->wsu, a[8] = w->ssg, a[9] = w->ssu, a[10] = w->wsd, a[11] = w->ssd;
}
static int dev_get(void *ctx, int i, void *buf, size_t off, size_t n) {
    const unsigned char *const *a = (const unsigned char *const *)ctx;
    return cudaMemcpy(buf, a[i] + off, n, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}
static int dev_put(void *ctx, int i, const void *buf, size_t off, size_t n) {
    unsigned char *const *a = (unsigned char *const *)ctx;
    return cudaMemcpy(a[i] + off, buf, n, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -1;
}

static int dev_file(const char *path, const jt_b200_moe_dims *dims, const jt_b200_moe_weights *w, int writing) {
    if (path == NULL || w == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    size_t sizes[WF_N];
    int r = jt_b200_moe_weights_sizes(dims, sizes);
    if (r != JT_OK) return r;
    const void *a[WF_N];
    fields_of(w, a);
    for (int i = 0; i < WF_N; i++)
        if (sizes[i] && a[i] == NULL) {
            errno = EINVAL;
            return JT_ERR_INVAL;
        }
    /* The copies below run on the legacy default stream; work that is still
     * producing or consuming the weights on other streams (a packer on a
     * non-blocking stream, a forward) finishes first. */
    if (cudaDeviceSynchronize() != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    unsigned char *buf = NULL;
    if (cudaMallocHost((void **)&buf, WF_BUF) != cudaSuccess) {
        errno = ENOMEM;
        return JT_ERR_NOMEM;
    }
    r = writing ? write_file(path, dims, dev_get, (void *)a, buf, WF_BUF)
                : read_file(path, dims, dev_put, (void *)a, buf, WF_BUF);
    cudaFreeHost(buf);
    return r;
}

int jt_b200_moe_weights_save(const char *path, const jt_b200_moe_dims *dims, const jt_b200_moe_weights *w) {
    return dev_file(path, dims, w, 1);
}

int jt_b200_moe_weights_load(const char *path, const jt_b200_moe_dims *dims, const jt_b200_moe_weights *w) {
    return dev_file(path, dims, w, 0);
}
