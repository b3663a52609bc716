/* jt_stage.c - staging area for the reference-compatible (host pointer)
 * entry points: a small set of grow-only device buffers reused across
 * calls, one stream, and a lock.  The reference API is single-threaded
 * (moe_layer.h fail-closed notes; w8a8.c:53 process globals); the lock only
 * keeps concurrent callers from sharing a slot. */
#include "jt_stage.h"

#include <errno.h>
#include <pthread.h>
#include <string.h>

static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;
static void *g_buf[JT_STAGE_SLOTS];
static size_t g_cap[JT_STAGE_SLOTS];
static int g_dev = -1;
static cudaStream_t g_stream;
static int g_stream_ok;

void jt_stage_lock(void) { pthread_mutex_lock(&g_lock); }
void jt_stage_unlock(void) { pthread_mutex_unlock(&g_lock); }

static int ensure_device(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (dev != g_dev) {
        /* Device changed: drop buffers that belong to the old device. */
        for (int i = 0; i < JT_STAGE_SLOTS; i++) {
            g_buf[i] = NULL;
            g_cap[i] = 0;
        }
        g_stream_ok = 0;
        g_dev = dev;
    }
    if (!g_stream_ok) {
        if (cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) != cudaSuccess) return -1;
        g_stream_ok = 1;
    }
    return 0;
}

void *jt_stage_buf(int slot, size_t bytes) {
    if (slot < 0 || slot >= JT_STAGE_SLOTS) return NULL;
    if (ensure_device() != 0) return NULL;
    if (bytes == 0) bytes = 16;
    if (g_cap[slot] < bytes) {
        if (g_buf[slot]) cudaFree(g_buf[slot]);
        g_buf[slot] = NULL;
        g_cap[slot] = 0;
        size_t want = bytes + (bytes >> 2);
        want = (want + 255u) & ~(size_t)255u;
        if (cudaMalloc(&g_buf[slot], want) != cudaSuccess) {
            cudaGetLastError();
            return NULL;
        }
        g_cap[slot] = want;
    }
    return g_buf[slot];
}

cudaStream_t jt_stage_stream(void) {
    if (ensure_device() != 0) return 0;
    return g_stream;
}

int jt_stage_h2d(void *dst, const void *src, size_t bytes) {
    if (bytes == 0) return 0;
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, jt_stage_stream()) !=
        cudaSuccess)
        return -1;
    return 0;
}

int jt_stage_d2h(void *dst, const void *src, size_t bytes) {
    if (bytes == 0) return 0;
    if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, jt_stage_stream()) !=
        cudaSuccess)
        return -1;
    return 0;
}

int jt_stage_sync(void) {
    if (cudaStreamSynchronize(jt_stage_stream()) != cudaSuccess) return -1;
    int code = 0;
    if (jtk_read_and_clear_error(&code) != 0 || code != 0) return -1;
    return 0;
}
