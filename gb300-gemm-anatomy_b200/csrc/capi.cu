// Library-level C ABI: version/size handshake, thread-local last error,
// device probe, tensor-map encoding and the N-shard arithmetic.
//
// Mirrors the reference bridge's conventions (src/gemm/cublaslt_bridge.cu:106-126
// last error, :128-191 size handshake; src/gemm/cublaslt_bridge_p35.cu:525-560
// exported metadata) and its device query (src/memory/ldgsts.cu:397-445),
// except that the accepted device is compute capability 10.0 (B200), not 10.3.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include <cudaTypedefs.h>

#include "internal.h"

namespace b200 {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
    va_list args;
    va_start(args, fmt);
    std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
    va_end(args);
}

void clear_error() { g_last_error[0] = '\0'; }

int cuda_fail(const char* what, cudaError_t err) {
    set_error("%s failed: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
    if (err == cudaErrorNoDevice || err == cudaErrorInsufficientDriver) return B200_ERR_NO_DEVICE;
    return B200_ERR_CUDA;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                             cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        } else {
            cudaGetLastError();
        }
    });
    return fn;
}

int encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                   uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
                   uint32_t box_cols, CUtensorMapSwizzle swizzle) {
    auto fn = get_encode_fn();
    if (fn == nullptr) {
        set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
        return B200_ERR_CUDA;
    }
    std::memset(map, 0, sizeof(*map));
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estrides[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estrides,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (CUresult %d) for %llu x %llu (ld %llu) box %u x %u",
                  static_cast<int>(r), static_cast<unsigned long long>(rows),
                  static_cast<unsigned long long>(cols), static_cast<unsigned long long>(ld),
                  box_rows, box_cols);
        return B200_ERR_CUDA;
    }
    return B200_OK;
}

int device_props(int device, DeviceProps* out) {
    constexpr int kMaxDevices = 64;
    static DeviceProps cache[kMaxDevices];
    static bool valid[kMaxDevices] = {};
    static std::mutex mu;
    if (device < 0 || device >= kMaxDevices) {
        set_error("device index %d out of range", device);
        return B200_ERR_INVALID_ARGUMENT;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!valid[device]) {
        DeviceProps p;
        cudaError_t e;
        if ((e = cudaDeviceGetAttribute(&p.sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&p.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&p.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&p.l2_bytes, cudaDevAttrL2CacheSize, device)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&p.cc_major, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&p.cc_minor, cudaDevAttrComputeCapabilityMinor, device)) != cudaSuccess) {
            return cuda_fail("cudaDeviceGetAttribute", e);
        }
        cache[device] = p;
        valid[device] = true;
    }
    *out = cache[device];
    return B200_OK;
}

uint64_t wait_timeout_ns() {
    static uint64_t value = []() {
        uint64_t ms = 2000;
        if (const char* env = std::getenv("B200_WAIT_TIMEOUT_MS")) {
            char* end = nullptr;
            const unsigned long long v = std::strtoull(env, &end, 10);
            if (end != env && *end == '\0' && v >= 1 && v <= 600000) ms = v;
        }
        return ms * 1000000ull;
    }();
    return value;
}

}  // namespace b200

extern "C" {

int b200_abi_version(void) { return B200_ABI_VERSION; }
size_t b200_plan_info_size(void) { return sizeof(B200PlanInfo); }
size_t b200_device_info_size(void) { return sizeof(B200DeviceInfo); }
size_t b200_stream_result_size(void) { return sizeof(B200StreamResult); }
const char* b200_last_error(void) { return b200::g_last_error; }

int b200_device_probe(int device, B200DeviceInfo* out) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (out == nullptr) {
        b200::set_error("out must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    std::memset(out, 0, sizeof(*out));
    int count = 0;
    cudaError_t err = cudaGetDeviceCount(&count);
    if (err != cudaSuccess || count == 0) {
        cudaGetLastError();
        b200::set_error("no CUDA device is visible (%s)",
                        err == cudaSuccess ? "device count 0" : cudaGetErrorName(err));
        return B200_ERR_NO_DEVICE;
    }
    if (device < 0 || device >= count) {
        b200::set_error("device %d out of range [0, %d)", device, count);
        return B200_ERR_INVALID_ARGUMENT;
    }
    cudaDeviceProp prop{};
    B200_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    int optin = 0, drv = 0, rt = 0, clock = 0;
    B200_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    B200_CUDA_TRY(cudaDeviceGetAttribute(&clock, cudaDevAttrClockRate, device));
    B200_CUDA_TRY(cudaDriverGetVersion(&drv));
    B200_CUDA_TRY(cudaRuntimeGetVersion(&rt));
    out->device = device;
    out->cc_major = prop.major;
    out->cc_minor = prop.minor;
    out->sm_count = prop.multiProcessorCount;
    out->l2_bytes = prop.l2CacheSize;
    out->smem_per_sm_bytes = static_cast<int64_t>(prop.sharedMemPerMultiprocessor);
    out->smem_optin_bytes = optin;
    out->global_mem_bytes = static_cast<int64_t>(prop.totalGlobalMem);
    out->driver_version = drv;
    out->runtime_version = rt;
    out->clock_khz = clock;
    out->is_sm100 = (prop.major == 10 && prop.minor == 0) ? 1 : 0;
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_shard_range(int64_t n, int64_t world, int64_t rank, int64_t granule, int64_t* n_begin,
                     int64_t* n_end) {
    b200::clear_error();
    if (n_begin == nullptr || n_end == nullptr) {
        b200::set_error("n_begin and n_end must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (n < 0 || world < 1 || rank < 0 || rank >= world || granule < 1) {
        b200::set_error("invalid shard request n=%lld world=%lld rank=%lld granule=%lld",
                        (long long)n, (long long)world, (long long)rank, (long long)granule);
        return B200_ERR_INVALID_ARGUMENT;
    }
    int64_t width = (n + world - 1) / world;
    width = ((width + granule - 1) / granule) * granule;
    int64_t b = rank * width;
    int64_t e = b + width;
    if (b > n) b = n;
    if (e > n) e = n;
    *n_begin = b;
    *n_end = e;
    return B200_OK;
}

}  // extern "C"
