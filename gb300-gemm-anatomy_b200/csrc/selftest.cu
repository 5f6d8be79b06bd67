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

// Holds one SM per CTA (the dynamic shared memory keeps a second CTA off it)
// for hold_ns of %globaltimer time, then returns: a stand-in for another
// tenant's kernel, so that tests can launch a GEMM while only part of the GPU
// is free. The loop is bounded by the timer; nothing here waits on anyone.
__global__ void occupy_sms_kernel(unsigned long long hold_ns) {
    extern __shared__ uint8_t hold_smem[];
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < hold_ns) {
        __nanosleep(10000);
    }
    hold_smem[0] = 0;
}

}  // namespace b200

extern "C" int b200_selftest_occupy(int ctas, int smem_bytes, unsigned long long hold_ns, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (ctas < 1 || ctas > 4096 || smem_bytes < 0 || smem_bytes > 232448) {
        b200::set_error("occupy: ctas in [1, 4096] and smem_bytes in [0, 232448] required");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (hold_ns == 0 || hold_ns > 5ull * 1000 * 1000 * 1000) {
        b200::set_error("occupy: hold_ns must be in (0, 5 s]");
        return B200_ERR_INVALID_ARGUMENT;
    }
    B200_CUDA_TRY(cudaFuncSetAttribute(b200::occupy_sms_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes));
    b200::occupy_sms_kernel<<<ctas, 32, smem_bytes, static_cast<cudaStream_t>(stream)>>>(hold_ns);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
    B200_ABI_GUARD_END
}

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
