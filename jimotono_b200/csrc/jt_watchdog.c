/* jt_watchdog.c - bounded host waits of the expert-parallel layer.
 *
 * The expert-parallel forward blocks on the host once per step: for the
 * gathered expert counts, which need every rank's all-gather.  A rank that
 * died or stopped calling leaves that collective unfinished forever.  The
 * watchdog replaces the blocking wait by a poll with a deadline: it checks
 * completion (a CUDA event), and the communicator's asynchronous error
 * (ncclCommGetAsyncError); on an error or when the deadline passes it aborts
 * the communicator (ncclCommAbort, which ends the rank's in-flight NCCL
 * kernels so the GPU stays usable) and the call returns an error; the
 * communicator is dead from then on and later calls fail at once.
 *
 * The polling loop takes its three operations as callbacks, so the same
 * code is checked without a GPU by jt_b200_watchdog_selftest (fake
 * operations: completion after some polls, a reported error, or nothing). */
#include <errno.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#include "jimotono_b200.h"
#include "jt_internal.h"

static double now_ms(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

int jt_watchdog_wait(const jt_watchdog_ops *ops, int timeout_ms, int *polls) {
    const double t0 = now_ms();
    int n = 0, rc = JT_WD_TIMEOUT;
    for (;;) {
        ++n;
        const int d = ops->done(ops->ctx);
        if (d > 0) {
            rc = JT_WD_DONE;
            break;
        }
        if (d < 0 || ops->async_error(ops->ctx) != 0) {
            rc = JT_WD_ERROR;
            break;
        }
        if (now_ms() - t0 > (double)timeout_ms) break;
        /* short sleeps: the counts usually land within tens of microseconds */
        const struct timespec nap = {0, n < 1000 ? 2000 : 200000};
        nanosleep(&nap, NULL);
    }
    if (rc != JT_WD_DONE && ops->abort_comm) ops->abort_comm(ops->ctx);
    if (polls) *polls = n;
    return rc;
}

/* ---------------------------------------------------------------- self-test */

typedef struct {
    int scenario, polls, aborted;
} fake_ctx;

static int fake_done(void *c) {
    fake_ctx *f = (fake_ctx *)c;
    ++f->polls;
    return f->scenario == 0 && f->polls >= 5 ? 1 : 0;
}

static int fake_error(void *c) {
    fake_ctx *f = (fake_ctx *)c;
    return f->scenario == 1 && f->polls >= 3 ? 1 : 0;
}

static void fake_abort(void *c) { ((fake_ctx *)c)->aborted = 1; }

int jt_b200_watchdog_selftest(int scenario, int timeout_ms, int *out_aborted) {
    if (scenario < 0 || scenario > 2 || timeout_ms < 0 || out_aborted == NULL) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    fake_ctx f = {scenario, 0, 0};
    const jt_watchdog_ops ops = {fake_done, fake_error, fake_abort, &f};
    const int rc = jt_watchdog_wait(&ops, timeout_ms, NULL);
    *out_aborted = f.aborted;
    return rc;
}
