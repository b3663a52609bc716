/* jt_nccl.h - the few NCCL entry points the expert-parallel layer uses,
 * resolved at run time from the process's libnccl.so.2 (the one the
 * application already loaded, else the system's), so the library builds
 * and loads without NCCL headers or a link-time dependency. */
#ifndef JT_NCCL_H
#define JT_NCCL_H

#include <stddef.h>
#include <cuda_runtime_api.h>

typedef struct {
    char internal[128];
} jt_nccl_id;

typedef void *jt_nccl_comm;

/* data types of the NCCL C API (nccl.h) */
enum { JT_NCCL_INT8 = 0, JT_NCCL_INT32 = 2, JT_NCCL_FLOAT32 = 7 };

typedef struct {
    int (*get_unique_id)(jt_nccl_id *);
    int (*comm_init_rank)(jt_nccl_comm *, int, jt_nccl_id, int);
    int (*comm_destroy)(jt_nccl_comm);
    int (*all_gather)(const void *, void *, size_t, int, jt_nccl_comm, cudaStream_t);
    int (*group_start)(void);
    int (*group_end)(void);
    int (*send)(const void *, size_t, int, int, jt_nccl_comm, cudaStream_t);
    int (*recv)(void *, size_t, int, int, jt_nccl_comm, cudaStream_t);
    const char *(*error_string)(int);
    int (*comm_get_async_error)(jt_nccl_comm, int *);  /* may be NULL (old NCCL) */
    int (*comm_abort)(jt_nccl_comm);                   /* may be NULL (old NCCL) */
} jt_nccl_api;

/* NULL when no NCCL library can be loaded. */
const jt_nccl_api *jt_nccl(void);

#endif
