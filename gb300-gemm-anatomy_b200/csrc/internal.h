// Host-side helpers shared by the C-ABI translation units: the thread-local
// last-error buffer, CUDA error mapping and the cuTensorMapEncodeTiled entry
// point (fetched through the runtime so the library needs no -lcuda).
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include <cuda.h>
#include <cuda_runtime.h>

#include "b200gemm.h"

namespace b200 {

void set_error(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
void clear_error();
int cuda_fail(const char* what, cudaError_t err);

// 2D tensor map over a row-major matrix of `rows` x `cols` elements with a
// row pitch of `ld` elements; box = box_cols x box_rows. Returns B200_OK or
// an error (message in the last-error buffer).
int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                   uint32_t box_cols, CUtensorMapSwizzle swizzle);

struct DeviceProps {
    int sm_count = 0;
    int smem_optin = 0;
    int smem_per_sm = 0;
    int l2_bytes = 0;
    int cc_major = 0;
    int cc_minor = 0;
};
// Cached per device; returns B200_OK or an error.
int device_props(int device, DeviceProps* out);

// Wait budget of every bounded device wait (ns). Overridable with the
// environment variable B200_WAIT_TIMEOUT_MS (read once).
uint64_t wait_timeout_ns();

}  // namespace b200

#define B200_CUDA_TRY(call)                                           \
    do {                                                              \
        cudaError_t err__ = (call);                                   \
        if (err__ != cudaSuccess) return ::b200::cuda_fail(#call, err__); \
    } while (0)

#define B200_ABI_GUARD_BEGIN try {
#define B200_ABI_GUARD_END                                                     \
    }                                                                          \
    catch (...) {                                                              \
        ::b200::set_error("internal error: C++ exception at the C ABI boundary"); \
        return B200_ERR_INTERNAL;                                              \
    }
