/* jt_stage.h - device staging used by the host-pointer entry points. */
#ifndef JT_STAGE_H
#define JT_STAGE_H

#include <stddef.h>
#include <cuda_runtime_api.h>

#include "jt_internal.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Staging slots (one grow-only device buffer each). */
enum {
    JT_SLOT_A = 0,
    JT_SLOT_B,
    JT_SLOT_A2,
    JT_SLOT_B2,
    JT_SLOT_C,
    JT_SLOT_SCALE,
    JT_SLOT_FLAGS,
    JT_SLOT_X,
    JT_SLOT_Y,
    JT_SLOT_W1,
    JT_SLOT_W2,
    JT_SLOT_W3,
    JT_SLOT_AUX1,
    JT_SLOT_AUX2,
    JT_SLOT_AUX3,
    JT_SLOT_AUX4,
    JT_SLOT_L0 /* first of the slots private to the layer entry points */
};

#define JT_STAGE_SLOTS 96

void jt_stage_lock(void);
void jt_stage_unlock(void);
void *jt_stage_buf(int slot, size_t bytes);
cudaStream_t jt_stage_stream(void);
int jt_stage_h2d(void *dst, const void *src, size_t bytes);
int jt_stage_d2h(void *dst, const void *src, size_t bytes);
/* Synchronize the staging stream and fold kernel-reported faults: 0 ok. */
int jt_stage_sync(void);

#ifdef __cplusplus
}
#endif

#endif
