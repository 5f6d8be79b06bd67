// Memory-path layer: global -> shared-memory streaming with 16-byte cp.async
// (LDGSTS) or 2D TMA tiles, replacing the reference study's two benchmark
// binaries (src/memory/ldgsts.cu:273-380 and src/memory/tma.cu:452-607).
//
// What is kept from the reference: 128 threads per CTA, a ring of `stages`
// slots of `stage_bytes`, one tile = one slot's worth of contiguous bytes,
// `passes` over the working set with a rotated tile order per pass, the
// SplitMix64 index pattern for validation (ldgsts.cu:226-246) and the sink
// word per thread in the timed mode (ldgsts.cu:333-380).
//
// What is B200-first here:
//  * LDGSTS: every thread only ever reads back the 16-byte vectors it copied
//    itself, so the ring needs no __syncthreads at all (the reference pays two
//    per tile); cp.async.wait_group alone orders copy and use.
//  * TMA: four independent per-warp pipelines (each warp loads and reads its
//    own quarter of every stage), and a second geometry uses the GEMM's
//    128-byte-swizzled 64-element rows.
//  * CTAs/SM in {1, 2, 4} with an occupancy-checked shared-memory reservation,
//    tile ranges balanced across the grid so any multiple of stage_bytes works
//    (4 GiB included), and a full-buffer XOR/sum checksum mode that is
//    bit-exact against a host checksum of the same bytes.
//  * Every mbarrier wait is bounded (status word instead of a hang).
#include <algorithm>
#include <cstring>
#include <new>

#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int kStreamThreads = 128;
constexpr uint64_t kPatternSalt = 0xD1B54A32D192ED03ULL;

// SplitMix64 finaliser (Steele, Lea, Flood 2014), the reference's pattern
// generator (src/memory/ldgsts.cu:226-238).
__host__ __device__ __forceinline__ uint64_t splitmix64_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

// The 16-byte vector at index i of the pattern (ldgsts.cu:231-238).
__device__ __forceinline__ uint4 pattern_vector(uint64_t i) {
    const uint64_t lo = splitmix64_mix(i);
    const uint64_t hi = splitmix64_mix(i ^ kPatternSalt);
    return make_uint4(static_cast<uint32_t>(lo), static_cast<uint32_t>(lo >> 32),
                      static_cast<uint32_t>(hi), static_cast<uint32_t>(hi >> 32));
}

__global__ void fill_pattern_kernel(uint4* __restrict__ dst, int64_t vectors) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < vectors; i += stride)
        dst[i] = pattern_vector(static_cast<uint64_t>(i));
}

struct StreamCounters {
    unsigned long long mismatches;
    unsigned long long xor_acc;
    unsigned long long sum_acc;
    unsigned long long sink_xor;
    int status;
    int pad;
};

struct StreamParams {
    const uint8_t* src;
    int64_t total_tiles;
    int64_t stage_bytes;
    int64_t passes;
    int64_t rotation;
    int mode;
    int box_rows;        // TMA: rows per box
    int boxes_per_stage; // TMA: boxes per slot
    int row_bytes;       // TMA: bytes per tensor row (256 reference geometry, 128 swizzled)
    int swizzled;        // TMA: 128-byte swizzle applied in SMEM
    StreamCounters* counters;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ void tile_range(const StreamParams& p, int64_t& begin, int64_t& count) {
    const int64_t g = gridDim.x, b = blockIdx.x;
    begin = (p.total_tiles * b) / g;
    const int64_t end = (p.total_tiles * (b + 1)) / g;
    count = end - begin;
}

// Walks a CTA's tiles pass after pass, each pass rotated by one more tile
// (the reference's rotation, ldgsts.cu:351-356), with one modulo per pass
// instead of 64-bit divisions per step.
struct TileWalk {
    int64_t begin, count, rotation;
    int64_t i = 0, pass = 0, j = 0;
    __device__ TileWalk(int64_t b, int64_t c, int64_t rot) : begin(b), count(c), rotation(rot) {
        j = count > 0 ? rot % count : 0;
    }
    __device__ __forceinline__ int64_t tile() const { return begin + j; }
    __device__ __forceinline__ void next() {
        ++i;
        if (++j == count) j = 0;
        if (i == count) {
            i = 0;
            ++pass;
            j = (rotation + pass) % count;
        }
    }
};

// Per-thread consumption state.
struct Consumer {
    unsigned long long mismatches = 0;
    uint32_t xor_acc = 0;
    unsigned long long sum_acc = 0;
    uint32_t sink = 0;

    __device__ __forceinline__ void vector(int mode, const uint4& v, uint64_t global_vec) {
        if (mode == B200_STREAM_VALIDATE) {
            const uint4 w = pattern_vector(global_vec);
            mismatches += (v.x != w.x || v.y != w.y || v.z != w.z || v.w != w.w) ? 1 : 0;
        } else {
            xor_acc ^= v.x ^ v.y ^ v.z ^ v.w;
            sum_acc += static_cast<unsigned long long>(v.x) + v.y + v.z + v.w;
        }
    }

    __device__ void flush(const StreamParams& p) {
        const int lane = threadIdx.x & 31;
        if (p.mode == B200_STREAM_SINK) {
            unsigned int s = sink;
            for (int o = 16; o > 0; o >>= 1) s ^= __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) atomicXor(&p.counters->sink_xor, static_cast<unsigned long long>(s));
            return;
        }
        unsigned long long mm = mismatches, sm = sum_acc;
        unsigned int xr = xor_acc;
        for (int o = 16; o > 0; o >>= 1) {
            mm += __shfl_xor_sync(0xffffffffu, mm, o);
            sm += __shfl_xor_sync(0xffffffffu, sm, o);
            xr ^= __shfl_xor_sync(0xffffffffu, xr, o);
        }
        if (lane == 0) {
            if (p.mode == B200_STREAM_VALIDATE) {
                if (mm) atomicAdd(&p.counters->mismatches, mm);
            } else {
                atomicXor(&p.counters->xor_acc, static_cast<unsigned long long>(xr));
                atomicAdd(&p.counters->sum_acc, sm);
            }
        }
    }
};

// ---------------------------------------------------------------------------
// LDGSTS ring. Thread t copies vectors t, t+128, ... of each tile and is the
// only reader of those vectors, so no CTA barrier is needed.
// ---------------------------------------------------------------------------
template <int STAGES>
__global__ void __launch_bounds__(kStreamThreads)
ldgsts_stream_kernel(const StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x;
    const int copies = static_cast<int>(p.stage_bytes / (16 * kStreamThreads));
    int64_t tile0, ntiles;
    tile_range(p, tile0, ntiles);
    Consumer cons;
    const uint32_t sbase = smem_u32(smem);
    const int64_t total_steps = ntiles * p.passes;

    TileWalk issue_walk(tile0, ntiles, p.rotation), use_walk(tile0, ntiles, p.rotation);
    const uint32_t stage_bytes = static_cast<uint32_t>(p.stage_bytes);
    auto issue = [&](int64_t step) {
        if (step < total_steps) {
            const uint8_t* src = p.src + issue_walk.tile() * p.stage_bytes + tid * 16;
            const uint32_t slot = sbase + static_cast<uint32_t>(step % STAGES) * stage_bytes + tid * 16;
            for (int c = 0; c < copies; ++c)
                cp_async_16(slot + c * (kStreamThreads * 16), src + c * (kStreamThreads * 16));
            issue_walk.next();
        }
        cp_async_commit();  // possibly empty group: keeps the group count uniform
    };

    if (ntiles > 0) {
        for (int s = 0; s < STAGES - 1; ++s) issue(s);
        for (int64_t step = 0; step < total_steps; ++step) {
            issue(step + STAGES - 1);
            cp_async_wait<STAGES - 1>();
            const int64_t tile = use_walk.tile();
            use_walk.next();
            const uint8_t* slot = smem + (step % STAGES) * p.stage_bytes;
            if (p.mode == B200_STREAM_SINK) {
                cons.sink ^= *reinterpret_cast<const uint32_t*>(slot + tid * 16);
            } else {
                const uint64_t vec0 = static_cast<uint64_t>(tile * (p.stage_bytes / 16));
                for (int c = 0; c < copies; ++c) {
                    const int v = tid + c * kStreamThreads;
                    const uint4 x = *reinterpret_cast<const uint4*>(slot + v * 16);
                    cons.vector(p.mode, x, vec0 + v);
                }
            }
        }
        cp_async_wait<0>();
    }
    cons.flush(p);
}

// ---------------------------------------------------------------------------
// TMA ring, one independent pipeline per warp: warp w owns the w-th quarter of
// every stage, its lane 0 issues that quarter's boxes on the warp's own full
// barrier and refills it as soon as the warp has read it, so no warp ever
// waits for another (the refill in a CTA-wide ring waits for the slowest warp
// every step, which halved the throughput at small stages).
// ---------------------------------------------------------------------------
template <int STAGES>
__global__ void __launch_bounds__(kStreamThreads)
tma_stream_kernel(const __grid_constant__ CUtensorMap tmap, const StreamParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    constexpr int kWarps = kStreamThreads / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + static_cast<uint32_t>(STAGES * p.stage_bytes);
    const uint32_t full_w = bar0 + 8 * STAGES * warp;  // this warp's STAGES barriers
    int64_t tile0, ntiles;
    tile_range(p, tile0, ntiles);
    const int64_t total_steps = ntiles * p.passes;
    const int qbytes = static_cast<int>(p.stage_bytes / kWarps);
    const int qvecs = qbytes / 16;
    const int rows_per_tile = static_cast<int>(p.stage_bytes / p.row_bytes);
    const int qrows = rows_per_tile / kWarps;

    if (tid == 0) {
        for (int i = 0; i < kWarps * STAGES; ++i) mbar_init(bar0 + 8 * i, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmap);
    }
    __syncthreads();

    TileWalk issue_walk(tile0, ntiles, p.rotation), use_walk(tile0, ntiles, p.rotation);
    auto issue = [&](int64_t step) {  // lane 0 only
        const int s = static_cast<int>(step % STAGES);
        const uint32_t slot = sbase + static_cast<uint32_t>(s * p.stage_bytes + warp * qbytes);
        const int64_t row = issue_walk.tile() * rows_per_tile + warp * qrows;
        issue_walk.next();
        mbar_arrive_expect_tx(full_w + 8 * s, static_cast<uint32_t>(qbytes));
        for (int b = 0; b < p.boxes_per_stage; ++b)
            tma_load_2d(slot + b * p.box_rows * p.row_bytes, &tmap, full_w + 8 * s, 0,
                        static_cast<int32_t>(row + b * p.box_rows));
    };

    Consumer cons;
    if (lane == 0) {
        for (int64_t s = 0; s < STAGES && s < total_steps; ++s) issue(s);
    }
    for (int64_t step = 0; step < total_steps; ++step) {
        const int s = static_cast<int>(step % STAGES);
        const uint32_t parity = static_cast<uint32_t>((step / STAGES) & 1);
        if (!mbar_wait(full_w + 8 * s, parity, &p.counters->status, p.timeout_ns,
                       B200_DEV_TIMEOUT_STREAM)) {
            // Abandoning: wait (bounded) for this warp's loads still in flight.
            if (lane == 0) {
                const unsigned long long drain_ns = min(p.timeout_ns, 100000000ull);
                for (int64_t q = step; q < step + STAGES && q < total_steps; ++q)
                    mbar_wait(full_w + 8 * static_cast<int>(q % STAGES),
                              static_cast<uint32_t>((q / STAGES) & 1), nullptr, drain_ns, 0);
            }
            break;
        }
        const uint8_t* slot = smem + s * p.stage_bytes + warp * qbytes;
        const int64_t tile = use_walk.tile();
        use_walk.next();
        if (p.mode == B200_STREAM_SINK) {
            cons.sink ^= *reinterpret_cast<const uint32_t*>(slot + lane * 16);
        } else {
            const uint64_t vec0 = static_cast<uint64_t>(tile * (p.stage_bytes / 16) + warp * qvecs);
            for (int v = lane; v < qvecs; v += 32) {
                const uint4 x = *reinterpret_cast<const uint4*>(slot + v * 16);
                uint64_t logical = static_cast<uint64_t>(v);
                if (p.swizzled) {
                    // 128-byte rows from a 1024-byte aligned quarter; the 16-byte
                    // chunk c of row r sits at c ^ (r % 8).
                    const int r = v >> 3, c = v & 7;
                    logical = static_cast<uint64_t>(r * 8 + (c ^ (r & 7)));
                }
                cons.vector(p.mode, x, vec0 + logical);
            }
        }
        __syncwarp();  // the whole warp has read its quarter
        if (lane == 0 && step + STAGES < total_steps) issue(step + STAGES);
    }
    cons.flush(p);
    __syncthreads();
}

template <int STAGES>
static const void* ldgsts_sym() { return reinterpret_cast<const void*>(&ldgsts_stream_kernel<STAGES>); }
template <int STAGES>
static const void* tma_sym() { return reinterpret_cast<const void*>(&tma_stream_kernel<STAGES>); }

static const void* stream_sym(int method, int stages) {
    if (method == B200_STREAM_LDGSTS) {
        if (stages == 2) return ldgsts_sym<2>();
        if (stages == 4) return ldgsts_sym<4>();
        return ldgsts_sym<8>();
    }
    if (stages == 2) return tma_sym<2>();
    if (stages == 4) return tma_sym<4>();
    return tma_sym<8>();
}

static int check_stream_config(const B200StreamConfig* c) {
    if (c == nullptr) {
        set_error("config must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->method != B200_STREAM_LDGSTS && c->method != B200_STREAM_TMA &&
        c->method != B200_STREAM_TMA_SW128) {
        set_error("method=%lld is not LDGSTS(0), TMA(1) or TMA_SW128(2)", (long long)c->method);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->stages != 2 && c->stages != 4 && c->stages != 8) {
        set_error("stages=%lld must be one of 2, 4, 8", (long long)c->stages);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->stage_bytes < 2048 || c->stage_bytes > 65536 || c->stage_bytes % 2048 != 0) {
        set_error("stage_bytes=%lld must be a multiple of 2048 in [2048, 65536]",
                  (long long)c->stage_bytes);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->method == B200_STREAM_TMA_SW128 && c->stage_bytes % 4096 != 0) {
        set_error("TMA_SW128 needs stage_bytes %% 4096 == 0 (each warp's quarter of a stage "
                  "must hold whole 1024-byte swizzle atoms), got %lld", (long long)c->stage_bytes);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->ctas_per_sm != 1 && c->ctas_per_sm != 2 && c->ctas_per_sm != 4) {
        set_error("ctas_per_sm=%lld must be one of 1, 2, 4", (long long)c->ctas_per_sm);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->passes < 1 || c->passes > 1000000) {
        set_error("passes=%lld must be in [1, 1000000]", (long long)c->passes);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (c->rotation < 0) {
        set_error("rotation must be non-negative");
        return B200_ERR_INVALID_ARGUMENT;
    }
    return B200_OK;
}

}  // namespace b200

struct B200StreamPlan {
    int device = 0;
    B200StreamConfig cfg{};
    b200::StreamParams params{};
    CUtensorMap tmap{};
    const void* sym = nullptr;
    int grid = 0;
    int smem = 0;
    b200::StreamCounters* counters = nullptr;
    B200StreamResult info{};
};

extern "C" {

int b200_fill_pattern(void* buf, int64_t bytes, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (buf == nullptr || bytes < 0 || bytes % 16 != 0) {
        b200::set_error("fill_pattern: buf must be non-NULL and bytes a non-negative multiple of 16");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (bytes == 0) return B200_OK;
    int device = 0;
    B200_CUDA_TRY(cudaGetDevice(&device));
    b200::DeviceProps props;
    int rc = b200::device_props(device, &props);
    if (rc != B200_OK) return rc;
    const int64_t vectors = bytes / 16;
    const int64_t blocks = std::min<int64_t>((vectors + 255) / 256, int64_t(props.sm_count) * 8);
    b200::fill_pattern_kernel<<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 256, 0,
                                static_cast<cudaStream_t>(stream)>>>(static_cast<uint4*>(buf), vectors);
    B200_CUDA_TRY(cudaGetLastError());
    return B200_OK;
    B200_ABI_GUARD_END
}

int64_t b200_stream_plan_granule(const B200StreamConfig* cfg, int device) {
    if (b200::check_stream_config(cfg) != B200_OK) return -1;
    return cfg->stage_bytes;
}

int b200_stream_plan_create(const B200StreamConfig* cfg, const void* buf, int64_t bytes, int device,
                            B200StreamPlan** out_plan, B200StreamResult* out_info) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (out_plan == nullptr) {
        b200::set_error("out_plan must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    *out_plan = nullptr;
    int rc = b200::check_stream_config(cfg);
    if (rc != B200_OK) return rc;
    if (buf == nullptr || reinterpret_cast<uintptr_t>(buf) % 128 != 0) {
        b200::set_error("buf must be a 128-byte aligned device pointer");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (bytes <= 0 || bytes % cfg->stage_bytes != 0) {
        b200::set_error("bytes=%lld must be a positive multiple of stage_bytes=%lld",
                        (long long)bytes, (long long)cfg->stage_bytes);
        return B200_ERR_INVALID_ARGUMENT;
    }
    b200::DeviceProps props;
    B200_CUDA_TRY(cudaSetDevice(device));
    rc = b200::device_props(device, &props);
    if (rc != B200_OK) return rc;

    const bool tma = cfg->method != B200_STREAM_LDGSTS;
    const int64_t payload = cfg->stages * cfg->stage_bytes;
    const int64_t need = payload + (tma ? 1024 + 8 * 4 * cfg->stages : 0);
    // Reserve enough that no more than ctas_per_sm CTAs fit on one SM (the
    // reference forces exactly one with the same device, ldgsts.cu:806-843).
    const int64_t per_sm = props.smem_per_sm;
    int64_t reserve = per_sm / (cfg->ctas_per_sm + 1) + 1;
    reserve = ((reserve + 127) / 128) * 128;
    reserve = std::max<int64_t>(reserve, ((need + 127) / 128) * 128);
    if (reserve > props.smem_optin) {
        b200::set_error("stages x stage_bytes = %lld bytes does not fit %lld CTA(s)/SM",
                        (long long)payload, (long long)cfg->ctas_per_sm);
        return B200_ERR_UNSUPPORTED;
    }
    const void* sym = b200::stream_sym(static_cast<int>(cfg->method), static_cast<int>(cfg->stages));
    B200_CUDA_TRY(cudaFuncSetAttribute(sym, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(reserve)));
    int occ = 0;
    B200_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, sym, b200::kStreamThreads,
                                                                static_cast<size_t>(reserve)));
    if (occ != cfg->ctas_per_sm) {
        b200::set_error("occupancy check: %d CTA(s)/SM resident with %lld bytes of shared memory, "
                        "wanted %lld", occ, (long long)reserve, (long long)cfg->ctas_per_sm);
        return B200_ERR_UNSUPPORTED;
    }

    B200StreamPlan* plan = new (std::nothrow) B200StreamPlan();
    if (plan == nullptr) {
        b200::set_error("out of host memory");
        return B200_ERR_INTERNAL;
    }
    plan->device = device;
    plan->cfg = *cfg;
    plan->sym = sym;
    plan->grid = props.sm_count * static_cast<int>(cfg->ctas_per_sm);
    plan->smem = static_cast<int>(reserve);
    b200::StreamParams& p = plan->params;
    p.src = static_cast<const uint8_t*>(buf);
    p.total_tiles = bytes / cfg->stage_bytes;
    p.stage_bytes = cfg->stage_bytes;
    p.passes = cfg->passes;
    p.rotation = cfg->rotation;
    p.timeout_ns = b200::wait_timeout_ns();
    if (tma) {
        const bool sw = cfg->method == B200_STREAM_TMA_SW128;
        p.row_bytes = sw ? 128 : 256;
        p.swizzled = sw ? 1 : 0;
        // Each of the 4 warps loads a quarter of a stage (see tma_stream_kernel).
        const int qrows = static_cast<int>(cfg->stage_bytes / p.row_bytes) / 4;
        p.box_rows = std::min(qrows, 256);
        p.boxes_per_stage = qrows / p.box_rows;
        const uint64_t total_rows = static_cast<uint64_t>(bytes / p.row_bytes);
        rc = b200::encode_tmap_2d(&plan->tmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, buf, total_rows,
                                  p.row_bytes / 2, p.row_bytes / 2, p.box_rows, p.row_bytes / 2,
                                  sw ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc != B200_OK) {
            delete plan;
            return rc;
        }
    }
    cudaError_t err = cudaMalloc(&plan->counters, sizeof(b200::StreamCounters));
    if (err != cudaSuccess) {
        delete plan;
        return b200::cuda_fail("cudaMalloc(stream counters)", err);
    }
    p.counters = plan->counters;

    B200StreamResult& info = plan->info;
    info.grid_ctas = plan->grid;
    info.threads_per_cta = b200::kStreamThreads;
    info.smem_bytes = plan->smem;
    info.occupancy_ctas_per_sm = occ;
    info.tiles_per_cta = p.total_tiles / plan->grid;
    info.bytes_streamed = bytes * cfg->passes;
    if (out_info != nullptr) *out_info = info;
    *out_plan = plan;
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_stream_plan_execute(B200StreamPlan* plan, int mode, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr) {
        b200::set_error("plan is NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (mode != B200_STREAM_VALIDATE && mode != B200_STREAM_CHECKSUM && mode != B200_STREAM_SINK) {
        b200::set_error("mode=%d is not VALIDATE(0), CHECKSUM(1) or SINK(2)", mode);
        return B200_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    B200_CUDA_TRY(cudaMemsetAsync(plan->counters, 0, sizeof(b200::StreamCounters), s));
    b200::StreamParams p = plan->params;
    p.mode = mode;
    void* args_ldgsts[] = {&p};
    void* args_tma[] = {&plan->tmap, &p};
    void** args = plan->cfg.method == B200_STREAM_LDGSTS ? args_ldgsts : args_tma;
    B200_CUDA_TRY(cudaLaunchKernel(plan->sym, dim3(plan->grid), dim3(b200::kStreamThreads), args,
                                   static_cast<size_t>(plan->smem), s));
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_stream_plan_result(B200StreamPlan* plan, void* stream, B200StreamResult* out) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr || out == nullptr) {
        b200::set_error("plan and out must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    B200_CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    b200::StreamCounters c{};
    B200_CUDA_TRY(cudaMemcpy(&c, plan->counters, sizeof(c), cudaMemcpyDeviceToHost));
    *out = plan->info;
    out->mismatches = static_cast<int64_t>(c.mismatches);
    out->checksum_xor = static_cast<int64_t>(c.xor_acc);
    out->checksum_sum = static_cast<int64_t>(c.sum_acc);
    out->sink_xor = static_cast<int64_t>(c.sink_xor);
    out->status = c.status;
    if (c.status != 0) {
        b200::set_error("stream kernel reported device status 0x%x (bounded wait timed out)", c.status);
        return B200_ERR_DEVICE_TIMEOUT;
    }
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_stream_plan_destroy(B200StreamPlan* plan) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr) return B200_OK;
    cudaError_t err = cudaSuccess;
    if (plan->counters != nullptr) err = cudaFree(plan->counters);
    delete plan;
    if (err != cudaSuccess) return b200::cuda_fail("cudaFree(stream counters)", err);
    return B200_OK;
    B200_ABI_GUARD_END
}

}  // extern "C"
