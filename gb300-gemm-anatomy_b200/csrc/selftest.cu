// Failure-detection self-test: one kernel whose bounded wait must run out.
//
// The reference's device waits spin forever (src/memory/tma.cu:404-408,
// src/compute/umma_1sm.cu:466-467); every wait in this library is bounded
// instead (ptx.cuh mbar_wait). This entry point exercises that path on the
// GPU without faulting or hanging it: one thread initialises an mbarrier that
// nothing ever arrives on, waits on it with the given budget, records
// B200_DEV_TIMEOUT_SELFTEST in the caller's status word and returns normally,
// so the context stays usable.
#include "internal.h"
#include "ptx.cuh"

namespace b200 {

__global__ void bounded_wait_selftest_kernel(int* status, unsigned long long timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    const uint32_t b = smem_u32(&bar);
    mbar_init(b, 1);
    fence_barrier_init();
    mbar_wait(b, 0, status, timeout_ns, B200_DEV_TIMEOUT_SELFTEST);
    mbar_inval(b);
}

}  // namespace b200

extern "C" int b200_selftest_bounded_wait(unsigned long long timeout_ns, int* status, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (status == nullptr) {
        b200::set_error("status must be a device pointer");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (timeout_ns == 0 || timeout_ns > 10ull * 1000 * 1000 * 1000) {
        b200::set_error("timeout_ns must be in (0, 10 s]");
        return B200_ERR_INVALID_ARGUMENT;
    }
    b200::bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, timeout_ns);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
    B200_ABI_GUARD_END
}
