// cm_selftest.cu -- device-side wait expiry, made on purpose without a fault.
//
// The kernel waits on an mbarrier that nothing ever arrives on, through the
// same bounded wait the GEMM and pool pipelines use.  When the limit runs out
// it records CM_ETIMEOUT in the device status word and returns; the host reads
// the status like any other call's, and the context stays usable.
#include "cm_async.cuh"

namespace cm {
namespace {

__global__ void selftest_wait_kernel(int* status, uint64_t timeout_ns) {
    griddep_wait();
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const WaitCtl wc{&abort_flag, status, timeout_ns};
        mbar_wait(smem_u32(&bar), 0, wc);   // phase 0 never completes: no arrival is pending
    }
    __syncthreads();
}

}  // namespace
}  // namespace cm

using namespace cm;

extern "C" int cm_selftest_wait_timeout(unsigned timeout_ms) {
    const Context* cx;
    int rc = enter(&cx);
    if (rc) return rc;
    if (timeout_ms == 0 || timeout_ms > 10000) return set_error(CM_EINVAL, "cm_selftest_wait_timeout: 1..10000 ms");
    launch_k(selftest_wait_kernel, 1, 32, 0, (cudaStream_t)0, cx->status, (uint64_t)timeout_ms * 1000000ull);
    count_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, "selftest launch");
    return finish_sync(nullptr);
}
