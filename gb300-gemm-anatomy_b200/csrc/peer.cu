// Peer-visible device buffers for the fused gather of the N-sharded GEMM:
// one process per GPU allocates its full-matrix output here, exports a CUDA
// IPC handle, opens the other ranks' handles and hands the peer pointers to
// b200_gemm_plan_set_peers. No counterpart in the reference (it has no
// multi-GPU path). Buffers come from cudaMalloc directly, so an IPC mapping
// starts exactly at the buffer (no allocator offset to correct).
#include <cstring>

#include "internal.h"

extern "C" {

size_t b200_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int b200_peer_buffer_alloc(int64_t bytes, void** out_ptr, void* out_handle) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (bytes <= 0 || out_ptr == nullptr || out_handle == nullptr) {
        b200::set_error("peer_buffer_alloc: bytes > 0 and non-NULL outputs required");
        return B200_ERR_INVALID_ARGUMENT;
    }
    *out_ptr = nullptr;
    void* p = nullptr;
    B200_CUDA_TRY(cudaMalloc(&p, static_cast<size_t>(bytes)));
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, p);
    if (err != cudaSuccess) {
        cudaFree(p);
        return b200::cuda_fail("cudaIpcGetMemHandle", err);
    }
    std::memcpy(out_handle, &h, sizeof(h));
    *out_ptr = p;
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_peer_buffer_free(void* ptr) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (ptr == nullptr) return B200_OK;
    B200_CUDA_TRY(cudaFree(ptr));
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_peer_open(const void* handle, void** out_ptr) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (handle == nullptr || out_ptr == nullptr) {
        b200::set_error("peer_open: handle and out_ptr must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    B200_CUDA_TRY(cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_peer_close(void* ptr) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (ptr == nullptr) return B200_OK;
    B200_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_peer_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                      int64_t width_bytes, int64_t rows, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (dst == nullptr || src == nullptr || width_bytes < 0 || rows < 0 || dst_pitch < width_bytes ||
        src_pitch < width_bytes) {
        b200::set_error("peer_copy_2d: non-NULL pointers and pitches >= width required");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (width_bytes == 0 || rows == 0) return B200_OK;
    // A device-to-device 2D copy: with `dst` in another GPU's memory (an IPC
    // mapping) the copy engines move it over NVLink, with no SM involved.
    B200_CUDA_TRY(cudaMemcpy2DAsync(dst, static_cast<size_t>(dst_pitch), src, static_cast<size_t>(src_pitch),
                                    static_cast<size_t>(width_bytes), static_cast<size_t>(rows),
                                    cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)));
    return B200_OK;
    B200_ABI_GUARD_END
}

}  // extern "C"
