// UMMA throughput probe: tcgen05.mma kind::f16 (BF16 x BF16 -> FP32) with
// both operands resident in shared memory and D in Tensor Memory. Replaces the
// reference's 24 fixed kernels umma_1sm_m128n{N}k16_d{DEPTH}
// (src/compute/umma_1sm.cu:365-538) and umma_2sm_m256n{N}k16_d{DEPTH}
// (src/compute/umma_2sm.cu:460-737) with one template per (cta_group, N) and
// a runtime depth.
//
// Operand layout: the GEMM's own 128-byte-swizzled K-major layout (one 64-
// element swizzle atom row per matrix row), so the probe exercises exactly
// the descriptors the GEMM uses. The K = 16 operand is replicated into the
// four 16-element K sub-blocks of the atom and MMA i reads sub-block i % 4;
// every MMA therefore adds the same A*B^T and D = depth * A * B^T, the
// reference's known answer (umma_1sm.cu:577-586).
//
// 2-CTA mode (cluster of 2): the even CTA issues M = 256 MMAs over both
// CTAs' operands; it commits to its own barrier only and, once the last
// commit has landed, releases the odd CTA with a cluster-scope arrive on the
// odd CTA's barrier (no per-iteration cluster barrier inside the timed loop,
// unlike umma_2sm.cu:637-672).
#include <algorithm>

#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int kProbeThreads = 128;
constexpr int kProbeK = 16;

template <int kCtaGroup, int N>
struct ProbeCfg {
    static constexpr int kNLocal = N / kCtaGroup;     // B rows held by each CTA
    static constexpr int kABytes = 128 * 128;         // 128 rows x 128-byte atom rows
    static constexpr int kBBytes = kNLocal * 128;
    static constexpr int kSmem = kABytes + kBBytes + 1024 + 64;
};

// Byte offset of element (row, k) of a 128B-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_offset(int row, int k) {
    const int chunk = k >> 3;
    return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4) + (k & 7) * 2);
}

__device__ __forceinline__ float probe_a_value(const __nv_bfloat16* a, int grow, int k) {
    if (a != nullptr) return __bfloat162float(a[grow * kProbeK + k]);
    return static_cast<float>(((grow + 3 * k) % 7) - 3);
}

__device__ __forceinline__ float probe_b_value(const __nv_bfloat16* b, int gcol, int k) {
    if (b != nullptr) return __bfloat162float(b[gcol * kProbeK + k]);
    return static_cast<float>(((2 * k + gcol) % 5) - 2);
}

template <int kCtaGroup, int N>
__global__ void __launch_bounds__(kProbeThreads, 1)
umma_probe_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
                  int depth, long long iterations, int timed, float* __restrict__ d_out,
                  unsigned long long* __restrict__ cycles, int* status,
                  unsigned long long timeout_ns) {
    using C = ProbeCfg<kCtaGroup, N>;
    constexpr bool kPair = kCtaGroup == 2;
    if (blockDim.x != kProbeThreads || (kPair && cluster_nctarank() != 2)) {
        if (threadIdx.x == 0) report_status(status, B200_DEV_BAD_LAUNCH);
        return;
    }
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sa = smem_u32(smem);
    const uint32_t sb = sa + C::kABytes;
    const uint32_t bar = sb + C::kBBytes;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kABytes + C::kBBytes + 16);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = kPair ? cluster_ctarank() : 0;
    const int group_id = blockIdx.x / kCtaGroup;

    // Operands: replicate the K = 16 slice into all four K sub-blocks of the atom.
    __nv_bfloat16* As = reinterpret_cast<__nv_bfloat16*>(smem);
    __nv_bfloat16* Bs = reinterpret_cast<__nv_bfloat16*>(smem + C::kABytes);
    for (int idx = tid; idx < 128 * 64; idx += kProbeThreads) {
        const int r = idx >> 6, k = idx & 63;
        const int grow = static_cast<int>(rank) * 128 + r;
        As[sw128_offset(r, k) / 2] = __float2bfloat16(probe_a_value(a, grow, k & 15));
    }
    for (int idx = tid; idx < C::kNLocal * 64; idx += kProbeThreads) {
        const int r = idx >> 6, k = idx & 63;
        const int gcol = static_cast<int>(rank) * C::kNLocal + r;
        Bs[sw128_offset(r, k) / 2] = __float2bfloat16(probe_b_value(b, gcol, k & 15));
    }
    fence_proxy_async_smem();
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc<kCtaGroup>(smem_u32(tmem_slot), N);
        tmem_relinquish<kCtaGroup>();
    }
    tc_fence_before();
    if constexpr (kPair) cluster_sync(); else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    if (warp == 0 && rank == 0) {
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_bf16_f32(128 * kCtaGroup, N);
            uint64_t adesc[4], bdesc[4];
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                adesc[s] = smem_desc_sw128(sa + 32 * s);
                bdesc[s] = smem_desc_sw128(sb + 32 * s);
            }
            uint32_t parity = 0;
            unsigned long long t0 = 0, t1 = 0;
            if (timed) asm volatile("mov.u64 %0, %%clock64;" : "=l"(t0)::"memory");
            for (long long it = 0; it < iterations; ++it) {
                // depth is a multiple of 4: one pass over the four K sub-blocks per step.
                for (int i = 0; i < depth; i += 4) {
#pragma unroll
                    for (int s = 0; s < 4; ++s)
                        umma_bf16<kCtaGroup>(tmem_d, adesc[s], bdesc[s], idesc, (i | s) != 0 ? 1u : 0u);
                }
                umma_commit<kCtaGroup>(bar);
                if (!mbar_wait(bar, parity, status, timeout_ns, B200_DEV_TIMEOUT_UMMA)) break;
                parity ^= 1;
            }
            if (timed) asm volatile("mov.u64 %0, %%clock64;" : "=l"(t1)::"memory");
            if (cycles != nullptr) cycles[blockIdx.x] = timed ? (t1 - t0) : 0ull;
            if constexpr (kPair) mbar_arrive_cluster(mapa_shared(bar, 1));
        }
        __syncwarp();
    } else if (kPair && warp == 0 && rank == 1) {
        if (elect_one()) {
            mbar_wait<true>(bar, 0, status, timeout_ns, B200_DEV_TIMEOUT_UMMA);
            if (cycles != nullptr) cycles[blockIdx.x] = 0ull;
        }
        __syncwarp();
    }
    __syncthreads();
    tc_fence_after();

    // Readback of D by the first CTA (pair): warp w owns TMEM lanes 32w..32w+31.
    if (group_id == 0 && !status_failed(status)) {
        const int row = static_cast<int>(rank) * 128 + warp * 32 + lane;
        for (int c = 0; c < N; c += 32) {
            uint32_t r[32];
            tmem_ld_32x32b_x32(tmem_addr(tmem_d, warp * 32, c), r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) d_out[static_cast<int64_t>(row) * N + c + i] = __uint_as_float(r[i]);
        }
    }
    tc_fence_before();
    if constexpr (kPair) cluster_sync(); else __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc<kCtaGroup>(tmem_d, N);
    }
}

template <int G, int N>
static int launch_probe(const B200UmmaConfig* cfg, const void* a, const void* b, float* d,
                        unsigned long long* cycles, int* status, cudaStream_t stream) {
    const int smem = ProbeCfg<G, N>::kSmem;
    auto kern = &umma_probe_kernel<G, N>;
    B200_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int groups = cfg->num_ctas > 0 ? static_cast<int>(cfg->num_ctas) : 1;
    cudaLaunchConfig_t lc = {};
    cudaLaunchAttribute attr[1];
    lc.gridDim = dim3(groups * G, 1, 1);
    lc.blockDim = dim3(kProbeThreads, 1, 1);
    lc.dynamicSmemBytes = smem;
    lc.stream = stream;
    if (G == 2) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
    }
    const auto* A = static_cast<const __nv_bfloat16*>(a);
    const auto* B = static_cast<const __nv_bfloat16*>(b);
    B200_CUDA_TRY(cudaLaunchKernelEx(&lc, kern, A, B, static_cast<int>(cfg->depth),
                                     static_cast<long long>(cfg->iterations),
                                     static_cast<int>(cfg->timed), d, cycles, status,
                                     static_cast<unsigned long long>(wait_timeout_ns())));
    return B200_OK;
}

}  // namespace b200

extern "C" int b200_umma_probe(const B200UmmaConfig* cfg, const void* a, const void* b, float* d_out,
                               unsigned long long* cycles, int* status, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (cfg == nullptr || d_out == nullptr || status == nullptr) {
        b200::set_error("cfg, d_out and status must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if ((a == nullptr) != (b == nullptr)) {
        b200::set_error("a and b must both be device pointers or both NULL (integer pattern)");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (cfg->cta_group != 1 && cfg->cta_group != 2) {
        b200::set_error("cta_group=%lld must be 1 or 2", (long long)cfg->cta_group);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (cfg->n != 64 && cfg->n != 128 && cfg->n != 256) {
        b200::set_error("n=%lld must be 64, 128 or 256", (long long)cfg->n);
        return B200_ERR_INVALID_ARGUMENT;
    }
    const int64_t d = cfg->depth;
    if (d != 4 && d != 16 && d != 32 && d != 64 && d != 128 && d != 256) {
        b200::set_error("depth=%lld must be one of 4, 16, 32, 64, 128, 256", (long long)d);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (cfg->iterations < 1 || cfg->iterations > (int64_t(1) << 40)) {
        b200::set_error("iterations=%lld must be >= 1", (long long)cfg->iterations);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (cfg->num_ctas < 0 || cfg->num_ctas > 4096) {
        b200::set_error("num_ctas=%lld out of range [0, 4096]", (long long)cfg->num_ctas);
        return B200_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int g = static_cast<int>(cfg->cta_group), n = static_cast<int>(cfg->n);
    if (g == 1) {
        if (n == 64) return b200::launch_probe<1, 64>(cfg, a, b, d_out, cycles, status, s);
        if (n == 128) return b200::launch_probe<1, 128>(cfg, a, b, d_out, cycles, status, s);
        return b200::launch_probe<1, 256>(cfg, a, b, d_out, cycles, status, s);
    }
    if (n == 64) return b200::launch_probe<2, 64>(cfg, a, b, d_out, cycles, status, s);
    if (n == 128) return b200::launch_probe<2, 128>(cfg, a, b, d_out, cycles, status, s);
    return b200::launch_probe<2, 256>(cfg, a, b, d_out, cycles, status, s);
    B200_ABI_GUARD_END
}
