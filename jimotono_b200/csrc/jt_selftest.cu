// jt_selftest.cu - diagnostic entry points of the failure-detection path.
//
// Every wait of the library's kernels on an mbarrier (a TMA landing, an MMA
// commit, a role handing a buffer on) is bounded: when its budget runs out
// the kernel raises its CTA abort flag and the device error word
// (JT_KERR_TIMEOUT), drains and returns, so the context stays usable and
// the host learns of it from jt_b200_sync.  jt_b200_selftest_bounded_wait
// runs that exact wait on a barrier that nothing ever completes, with a
// short budget chosen by the caller, so a test can check the whole path
// without hanging or faulting a GPU.
#include <cuda_runtime.h>
#include <errno.h>

#include "../../include/jimotono_b200.h"
#include "jt_internal.h"
#include "jt_ptx.cuh"

namespace {

__global__ void k_selftest_wait(long long budget, int *err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        jt::mbar_init(&bar, 1);
        jt::fence_mbar_init();
    }
    __syncthreads();
    // no thread ever arrives on bar
    jt::mbar_wait_budget(&bar, 0, &abort_flag, err, budget);
}

}  // namespace

extern "C" int jt_b200_selftest_bounded_wait(long long budget_cycles, void *stream) {
    if (budget_cycles <= 0 || budget_cycles > JT_SPIN_CYCLES) {
        errno = EINVAL;
        return JT_ERR_INVAL;
    }
    k_selftest_wait<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(budget_cycles, jtk_error_word());
    if (cudaGetLastError() != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}

extern "C" int jt_b200_sync_code(int *kernel_code) {
    if (kernel_code) *kernel_code = 0;
    if (cudaDeviceSynchronize() != cudaSuccess) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    int code = 0;
    if (jtk_read_and_clear_error(&code) != 0) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    if (kernel_code) *kernel_code = code;
    if (code != 0) {
        errno = EIO;
        return JT_ERR_CUDA;
    }
    return JT_OK;
}
