/* jt_nccl.c - run-time binding of NCCL (see jt_nccl.h). */
#include "jt_nccl.h"

#include <dlfcn.h>
#include <pthread.h>
#include <stddef.h>

static jt_nccl_api g_api;
static int g_ok = 0;
static pthread_once_t g_once = PTHREAD_ONCE_INIT;

static void load(void) {
    /* prefer a copy already in the process (e.g. the one PyTorch loaded) */
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
#define SYM(field, name)                                      \
    do {                                                      \
        *(void **)(&g_api.field) = dlsym(h, name);            \
        if (!g_api.field) return;                             \
    } while (0)
    SYM(get_unique_id, "ncclGetUniqueId");
    SYM(comm_init_rank, "ncclCommInitRank");
    SYM(comm_destroy, "ncclCommDestroy");
    SYM(all_gather, "ncclAllGather");
    SYM(group_start, "ncclGroupStart");
    SYM(group_end, "ncclGroupEnd");
    SYM(send, "ncclSend");
    SYM(recv, "ncclRecv");
    SYM(error_string, "ncclGetErrorString");
#undef SYM
    *(void **)(&g_api.comm_get_async_error) = dlsym(h, "ncclCommGetAsyncError");
    *(void **)(&g_api.comm_abort) = dlsym(h, "ncclCommAbort");
    g_ok = 1;
}

const jt_nccl_api *jt_nccl(void) {
    pthread_once(&g_once, load);
    return g_ok ? &g_api : NULL;
}
