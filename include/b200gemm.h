/*
 * b200gemm.h — C ABI of the B200 (sm_100a) BF16 GEMM stack.
 *
 * Plain C: every function returns int (0 = B200_OK) or a plain size/pointer,
 * never lets a C++ exception cross, writes nothing to stdout/stderr, and keeps
 * the last error message in thread-local storage (b200_last_error). Pointers
 * are device pointers unless a comment says otherwise; `stream` is a
 * cudaStream_t passed as void* (0 = legacy default stream).
 *
 * Conventions follow the reference study's cuBLASLt bridge, which this library
 * replaces as the GEMM candidate behind the same driver:
 *   src/gemm/cublaslt_bridge.cu:106-126   thread-local last error
 *   src/gemm/cublaslt_bridge.cu:128-191   all-8-byte metadata struct + size handshake
 *   src/gemm/cublaslt_bridge_p35.cu:563-1018  plan create / execute / sync / destroy
 * Layout contract (src/gemm/gemm_comparison.py:2670-2691, cublaslt_bridge_p35.cu:96-111):
 *   A is M x K row-major (K contiguous), B is N x K row-major (K contiguous,
 *   "TN"), D is M x N row-major with leading dimension ldd (elements).
 *   D = A * B^T, bf16 inputs, fp32 accumulation, beta = 0.
 */
#ifndef B200GEMM_H_
#define B200GEMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200_ABI_VERSION 1

/* Host-side return codes. */
enum {
    B200_OK = 0,
    B200_ERR_INVALID_ARGUMENT = 1,
    B200_ERR_UNSUPPORTED = 2,
    B200_ERR_CUDA = 3,
    B200_ERR_DEVICE_TIMEOUT = 4, /* a kernel gave up a bounded wait; see b200_last_error */
    B200_ERR_MISMATCH = 5,       /* a self-validating kernel found wrong data */
    B200_ERR_NO_DEVICE = 6,
    B200_ERR_INTERNAL = 7
};

/* Codes a kernel writes into its device status word (first failure wins). */
enum {
    B200_DEV_OK = 0,
    B200_DEV_TIMEOUT_PRODUCER = 0x101, /* TMA producer waited too long for a free ring slot */
    B200_DEV_TIMEOUT_MMA_FULL = 0x102, /* MMA issuer waited too long for operands */
    B200_DEV_TIMEOUT_MMA_TMEM = 0x103, /* MMA issuer waited too long for a free accumulator */
    B200_DEV_TIMEOUT_EPILOGUE = 0x104, /* epilogue waited too long for an accumulator */
    B200_DEV_TIMEOUT_STREAM = 0x105,   /* memory-path streamer waited too long for a stage */
    B200_DEV_TIMEOUT_UMMA = 0x106,     /* UMMA probe waited too long for its commit */
    B200_DEV_TIMEOUT_SELFTEST = 0x107, /* b200_selftest_bounded_wait ran out, as designed */
    B200_DEV_TIMEOUT_PARTIAL = 0x108,  /* stream-K epilogue waited too long for a partial tile */
    B200_DEV_BAD_LAUNCH = 0x1FF        /* launch geometry differs from the kernel's contract */
};

/* Output element types. */
enum { B200_OUT_BF16 = 0, B200_OUT_F32 = 1 };

/* GEMM modes (tile of D per CTA pair or CTA):
 *   1CTA       128 x 256 per CTA, accumulators double-buffered across tiles
 *   2CTA       256 x 256 per CTA pair (cta_group::2), double-buffered
 *   2CTA_M512  512 x 256 per CTA pair: each CTA owns two 128-row accumulators
 *              that fill TMEM; 25 % fewer L2->SM bytes per FLOP than 2CTA
 *   2CTA_N128  256 x 128 per CTA pair, double-buffered, 8-slot ring: twice the
 *              tiles of 2CTA (dynamic schedule only). Never chosen by AUTO:
 *              measured ~0.7x of 2CTA on B200; kept for experiments
 * AUTO picks by shape. */
enum {
    B200_MODE_AUTO = 0,
    B200_MODE_1CTA = 1,
    B200_MODE_2CTA = 2,
    B200_MODE_2CTA_M512 = 3,
    B200_MODE_2CTA_N128 = 4
};

/* ------------------------------------------------------------------------ */
/* Library / device                                                          */
/* ------------------------------------------------------------------------ */

/* Replaces p35_bridge_abi_version (cublaslt_bridge_p35.cu:525). */
int b200_abi_version(void);
/* Replaces p35_plan_info_size (cublaslt_bridge_p35.cu:530). */
size_t b200_plan_info_size(void);
size_t b200_device_info_size(void);
size_t b200_stream_result_size(void);
/* Replaces p35_last_error (cublaslt_bridge_p35.cu:535). Thread-local, never NULL. */
const char* b200_last_error(void);

typedef struct B200DeviceInfo {
    int64_t device;
    int64_t cc_major;
    int64_t cc_minor;
    int64_t sm_count;
    int64_t l2_bytes;
    int64_t smem_per_sm_bytes;
    int64_t smem_optin_bytes;
    int64_t global_mem_bytes;
    int64_t driver_version;
    int64_t runtime_version;
    int64_t clock_khz;
    int64_t is_sm100; /* 1 when the device runs this library's sm_100a code */
} B200DeviceInfo;

/* Replaces the reference's query_gpu_info (src/memory/ldgsts.cu:397-445) and
 * the CUDA smoke binary (smoke/cuda_smoke.cu): fills *out for `device`.
 * Returns B200_ERR_NO_DEVICE when no CUDA device is visible. */
int b200_device_probe(int device, B200DeviceInfo* out);

/* ------------------------------------------------------------------------ */
/* GEMM plans                                                                */
/* ------------------------------------------------------------------------ */

typedef struct B200Plan B200Plan;

typedef struct B200PlanInfo {
    int64_t abi_version;
    int64_t m;
    int64_t n;
    int64_t k;
    int64_t lda;
    int64_t ldb;
    int64_t ldd;
    int64_t out_dtype;      /* B200_OUT_* */
    int64_t mode;           /* resolved B200_MODE_1CTA or B200_MODE_2CTA */
    int64_t cta_group;      /* 1 or 2 */
    int64_t tile_m;         /* rows of D per tile (per CTA pair in 2-CTA mode) */
    int64_t tile_n;
    int64_t tile_k;
    int64_t stages;
    int64_t cluster_m;
    int64_t grid_ctas;
    int64_t threads_per_cta;
    int64_t smem_bytes;
    int64_t tmem_columns;
    int64_t num_tiles;
    int64_t sm_count;
    int64_t device;
    double waves;           /* num_tiles / resident tile slots */
    double flop_count;      /* 2*M*N*K */
} B200PlanInfo;

/* Reference-compatible plan: the exact argument list of p35_plan_create
 * (src/gemm/cublaslt_bridge_p35.cu:563-572). Output D is fp32 M x N
 * row-major, like the reference's CUDA_R_32F D; C is accepted for signature
 * compatibility and ignored (beta = 0). Mode AUTO. */
int b200_gemm_plan_create(int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                          const void* c, void* d, void* stream, B200Plan** out_plan,
                          B200PlanInfo* out_info);

/* Full-control plan: out_dtype B200_OUT_BF16 or B200_OUT_F32, mode B200_MODE_*,
 * ldd >= n (elements; ldd*elem_size must be a multiple of 16 bytes). No
 * counterpart in the reference beyond p35_plan_create; it exposes the bf16
 * output, the mode choice and strided output placement (used to write an
 * N-shard at its column offset inside a larger matrix). */
int b200_gemm_plan_create_ex(int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                             void* d, int64_t ldd, int out_dtype, int mode, void* stream,
                             B200Plan** out_plan, B200PlanInfo* out_info);

/* Replaces p35_plan_execute (cublaslt_bridge_p35.cu:949): one asynchronous
 * launch on the plan's stream. */
int b200_gemm_plan_execute(B200Plan* plan);

/* Same launch on another stream (e.g. inside a CUDA-graph capture). Launches of
 * one plan must not overlap on the GPU: they share its status word and tile
 * counter. */
int b200_gemm_plan_execute_on(B200Plan* plan, void* stream);

/* Replaces p35_stream_synchronize (cublaslt_bridge_p35.cu:987): waits for the
 * plan's stream, then reads and clears the device status word; a kernel that
 * gave up a bounded wait turns into B200_ERR_DEVICE_TIMEOUT here. */
int b200_stream_synchronize(B200Plan* plan);

/* Replaces p35_plan_destroy (cublaslt_bridge_p35.cu:1008). NULL is a no-op. */
int b200_gemm_plan_destroy(B200Plan* plan);

/* Analogue of CuTe's can_implement (src/gemm/cutedsl_variants.py:1296-1324):
 * B200_OK when the shape/dtype/mode is accepted, otherwise an error code with
 * the reason in b200_last_error. Pointer alignment is checked at create. */
int b200_gemm_supported(int64_t m, int64_t n, int64_t k, int64_t ldd, int out_dtype, int mode);

/* One-shot GEMM: create, execute, synchronise, check the status word, destroy. */
int b200_gemm(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d,
              int64_t ldd, int out_dtype, int mode, void* stream);

/* Allocation-free GEMM. No counterpart in the reference. Same arguments,
 * tile shapes, grid and synchronous behaviour as b200_gemm, but it calls no cudaMalloc,
 * cudaFree or other allocating routine: the kernel's only scratch (16 bytes:
 * the status word for bounded-wait timeouts and the tile scheduler's counter)
 * lives in a 256-byte static device
 * array of the library, which every GPU that loads the library holds until
 * exit. For callers that cannot allocate device memory -- programs that give
 * all device memory to their own pool up front, or paths that must avoid the
 * device-wide synchronisation cudaMalloc/cudaFree imply.
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture. Calls
 * share the array: each clears those 16 bytes before its launch, and calls
 * that overlap on the GPU (other streams, other threads) race on it. A launch
 * whose scratch need exceeded the array would be refused with
 * B200_ERR_UNSUPPORTED; this kernel needs 16 bytes whatever M, N and K are.
 * It always runs the dynamic tile schedule: the stream-K schedule's partial
 * buffer (about 19 MB) does not fit the static array, so on shapes where
 * b200_gemm picks stream-K (e.g. 4096^3) the fp32 sums are associated
 * differently and the last bits may differ (B200_GEMM_SCHEDULE is ignored).
 * The cached address belongs to the device's current context; after a
 * cudaDeviceReset the next call looks it up again. */
int b200_gemm_noalloc(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d,
                      int64_t ldd, int out_dtype, int mode, void* stream);

/* Fused gather for the N-sharded multi-GPU GEMM. After set_peers, every launch
 * also writes each staged output chunk into the npeers (<= 7) peer buffers over
 * NVLink -- by default as TMA bulk stores (one per peer per chunk, through
 * tensor maps encoded here), with B200_PEER_STORES=st at set_peers as per-thread
 * 16-byte stores -- at the same rows/columns and row pitch as the
 * plan's own D; peer_d[g] must already point at this shard's first column in
 * peer g's full matrix (see b200_peer_*). The caller orders the ranks after
 * the launch (e.g. one NCCL all-reduce of a scalar) before reading peers'
 * data. npeers = 0 turns it off. No counterpart in the reference (no
 * multi-GPU path there); replaces GEMM-then-all-gather with one kernel. */
int b200_gemm_plan_set_peers(B200Plan* plan, int npeers, void* const* peer_d);

/* Multicast form of the fused gather (NVLink SHARP / NVLS). mc_d is this
 * shard's first column inside an NVLink multicast mapping of the full M x N
 * bf16 output that every rank has bound its own buffer to (for example
 * torch.distributed._symmetric_memory's multicast_ptr plus n0 * 2); row pitch
 * = the plan's ldd. Every launch then writes each output chunk once, with
 * 16-byte multimem stores, and the switch replicates it into every GPU's
 * buffer: each GPU sends its shard once instead of once per peer. The caller
 * orders the ranks after the launch, as for set_peers. NULL turns it off.
 * Plain stores only: no TMA or bulk load ever reads a multicast or peer
 * address. No counterpart in the reference (no multi-GPU path there). */
int b200_gemm_plan_set_multicast(B200Plan* plan, void* mc_d);

/* Peer-visible buffers (CUDA IPC) for the fused gather. alloc: cudaMalloc of
 * `bytes` plus its IPC handle (b200_ipc_handle_size() bytes written to
 * out_handle); open/close map another process's buffer on the current device. */
size_t b200_ipc_handle_size(void);
int b200_peer_buffer_alloc(int64_t bytes, void** out_ptr, void* out_handle);
int b200_peer_buffer_free(void* ptr);
int b200_peer_open(const void* handle, void** out_ptr);
int b200_peer_close(void* ptr);
/* Copy-engine gather step: an asynchronous 2D device copy of `rows` rows of
 * width_bytes from src (row pitch src_pitch bytes) to dst (pitch dst_pitch) on
 * `stream`; dst may be a peer buffer opened with b200_peer_open, so the copy
 * engines carry this shard to that GPU over NVLink while the SMs stay free. No
 * counterpart in the reference (no multi-GPU path there). */
int b200_peer_copy_2d(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                      int64_t width_bytes, int64_t rows, void* stream);

/* Timeline tracing (off by default). trace: device buffer of grid_ctas x 64
 * uint64 (%globaltimer ns) that each later execute fills per CTA: [0] entry,
 * [1] setup done, [2] producer done, [3] MMA issuer done, [4] epilogue done,
 * [5] exit, [6+i] accumulator of the CTA's i-th tile ready; unused slots keep
 * their old contents. NULL turns tracing off. No counterpart in the reference
 * (its UMMA probe times with %clock64 only, src/compute/umma_1sm.cu:449-475). */
int b200_gemm_plan_set_trace(B200Plan* plan, unsigned long long* trace, int64_t slots_per_cta);

/* Number of device kernels one execute launches (for launch accounting). */
int64_t b200_gemm_plan_launches(const B200Plan* plan);

/* Tile schedule a plan runs. DYNAMIC: whole tiles handed out by a global
 * counter. STREAM_K (128x256 and 256x256 tiles only; chosen when the dynamic
 * schedule would run at least three waves with the last one under 90 % busy):
 * the leftover tiles are split along K into one equal run per cluster group
 * and run first, whole tiles follow, and the cut tiles are finished through
 * an fp32 partial buffer the plan allocates (this ties each result's
 * summation split to the device's SM count). The environment variable
 * B200_GEMM_SCHEDULE=dynamic|streamk overrides the choice at plan creation.
 * No counterpart in the reference, whose persistent CuTe kernel
 * (src/gemm/gemm_comparison.py candidate table) runs whole tiles.
 * Returns -1 for a NULL plan. */
enum { B200_SCHEDULE_DYNAMIC = 0, B200_SCHEDULE_STREAM_K = 1 };
int b200_gemm_plan_schedule(const B200Plan* plan);

/* Host-side policy of a GEMM plan, computed without a device: the mode that
 * B200_MODE_AUTO resolves to, the tile grid, the raster of the tile walk and
 * the tile schedule, for a GPU with `sm_count` SMs on which one cluster per
 * SM (1-CTA) or per SM pair (2-CTA) is resident. Plans on such a GPU make the
 * same choices; the environment overrides B200_GEMM_SCHEDULE, B200_GEMM_RASTER
 * and B200_GEMM_GROUP apply here as well. No counterpart in the reference. */
typedef struct B200PolicyInfo {
    int64_t mode;            /* resolved B200_MODE_1CTA, _2CTA or _2CTA_M512 */
    int64_t tile_m;          /* rows of D per tile (per CTA pair in 2-CTA modes) */
    int64_t tile_n;
    int64_t num_m_blocks;
    int64_t num_n_blocks;
    int64_t num_k_blocks;    /* 64-wide k-slices */
    int64_t num_tiles;
    int64_t clusters;        /* resident clusters assumed */
    int64_t raster_n;        /* 0: groups of m-blocks walk every n-block; 1: the reverse */
    int64_t group;           /* blocks per raster group */
    int64_t schedule;        /* B200_SCHEDULE_* */
    int64_t sk_groups;       /* stream-K: cluster groups, lanes per group, lane axis */
    int64_t sk_lanes;
    int64_t sk_lane_n;
    int64_t sk_rounds;       /* whole-tile rounds after the split block */
    int64_t sk_split_tiles;  /* super-tiles in the split block */
    int64_t grid_ctas;
    int64_t kserp_wave;      /* dynamic schedule: tiles of odd waves of this many tiles walk K
                                backwards (0 = off, and always 0 under stream-K) */
    double waves;            /* num_tiles / clusters */
} B200PolicyInfo;

size_t b200_policy_info_size(void);
int b200_gemm_policy(int64_t m, int64_t n, int64_t k, int mode, int sm_count, B200PolicyInfo* out);

/* ------------------------------------------------------------------------ */
/* Memory path: global -> shared streaming (LDGSTS / TMA)                     */
/* Replaces the ldgsts and tma benchmark binaries                             */
/* (src/memory/ldgsts.cu:273-380, src/memory/tma.cu:452-607).                 */
/* ------------------------------------------------------------------------ */

enum {
    B200_STREAM_LDGSTS = 0,  /* 16-byte cp.async.cg, 128 threads, ring of `stages` slots */
    B200_STREAM_TMA = 1,     /* reference geometry: box 128 x tile_h of 2-byte elements, no swizzle */
    B200_STREAM_TMA_SW128 = 2 /* GEMM geometry: box 64 x rows bf16 (128-byte rows), 128B swizzle */
};

enum {
    B200_STREAM_VALIDATE = 0, /* compare every 16-byte vector with the SplitMix64 pattern */
    B200_STREAM_CHECKSUM = 1, /* XOR and wrapping sum of every 32-bit word read */
    B200_STREAM_SINK = 2      /* timed mode of the reference: XOR one word per thread per stage */
};

typedef struct B200StreamConfig {
    int64_t method;       /* B200_STREAM_* */
    int64_t stages;       /* 2, 4 or 8 */
    int64_t stage_bytes;  /* bytes per ring slot: multiple of 2048, <= 65536 */
    int64_t ctas_per_sm;  /* 1, 2 or 4 (reference: 1) */
    int64_t passes;       /* >= 1 */
    int64_t rotation;     /* tile-order rotation of the first pass (reference rotation_base) */
} B200StreamConfig;

typedef struct B200StreamResult {
    int64_t grid_ctas;
    int64_t threads_per_cta;
    int64_t smem_bytes;
    int64_t occupancy_ctas_per_sm;
    int64_t tiles_per_cta;
    int64_t bytes_streamed;      /* working set bytes x passes */
    int64_t mismatches;          /* VALIDATE */
    int64_t checksum_xor;        /* CHECKSUM: XOR of all 32-bit words (zero-extended) */
    int64_t checksum_sum;        /* CHECKSUM: sum of all 32-bit words mod 2^64, as int64 */
    int64_t sink_xor;            /* SINK: XOR over the per-thread sink words */
    int64_t status;              /* device status word */
} B200StreamResult;

typedef struct B200StreamPlan B200StreamPlan;

/* Fills `bytes` (multiple of 16) of device memory with the reference's
 * SplitMix64 index pattern (src/memory/ldgsts.cu:226-246). */
int b200_fill_pattern(void* buf, int64_t bytes, void* stream);

/* Creates a streaming plan over `bytes` of device memory at `buf`. The
 * working set must split into whole stages per CTA: bytes must be a multiple
 * of grid_ctas * stage_bytes (b200_stream_plan_granule gives that unit). */
int b200_stream_plan_create(const B200StreamConfig* cfg, const void* buf, int64_t bytes,
                            int device, B200StreamPlan** out_plan, B200StreamResult* out_info);
int64_t b200_stream_plan_granule(const B200StreamConfig* cfg, int device);
/* One asynchronous launch in mode B200_STREAM_*; clears the plan's counters first. */
int b200_stream_plan_execute(B200StreamPlan* plan, int mode, void* stream);
/* Synchronises `stream` and fills *out with the last launch's results. */
int b200_stream_plan_result(B200StreamPlan* plan, void* stream, B200StreamResult* out);
int b200_stream_plan_destroy(B200StreamPlan* plan);

/* ------------------------------------------------------------------------ */
/* UMMA throughput probe (tcgen05.mma kind::f16, operands resident in SMEM)  */
/* Replaces umma_1sm_m128n{N}k16_d{DEPTH} (src/compute/umma_1sm.cu:520-538)  */
/* and umma_2sm_m256n{N}k16_d{DEPTH} (src/compute/umma_2sm.cu:733-737).      */
/* ------------------------------------------------------------------------ */

typedef struct B200UmmaConfig {
    int64_t cta_group;   /* 1 (M = 128, one CTA) or 2 (M = 256, one CTA pair) */
    int64_t n;           /* 64, 128 or 256 */
    int64_t depth;       /* MMAs of K = 16 per commit: 4, 16, 32, 64, 128 or 256 */
    int64_t iterations;  /* commit+wait rounds, >= 1 */
    int64_t timed;       /* 1: leader thread reads %clock64 around the loop */
    int64_t num_ctas;    /* 0: one CTA (pair); else that many CTAs (pairs x2) in parallel */
} B200UmmaConfig;

/* Runs the probe. a (M x 16 bf16, row-major) and b (N x 16 bf16, row-major)
 * may be NULL, which selects the reference's integer pattern
 * A[r,k] = ((r+3k) mod 7) - 3, B[k,c] = ((2k+c) mod 5) - 2 on global rows/cols.
 * d_out receives D of the first CTA (pair): M x N fp32 row-major, which equals
 * depth * A * B^T. cycles (device, one uint64 per CTA) receives the leader's
 * %clock64 delta when timed. status (device int) receives B200_DEV_* codes. */
int b200_umma_probe(const B200UmmaConfig* cfg, const void* a, const void* b, float* d_out,
                    unsigned long long* cycles, int* status, void* stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU N-sharding (host arithmetic; the collective runs in the caller) */
/* ------------------------------------------------------------------------ */

/* Column range [*n_begin, *n_end) of output shard `rank` of `world` for an
 * N-column GEMM: shards are ceil(N/world) rounded up to `granule` columns,
 * the last one takes the remainder (possibly empty). No counterpart in the
 * reference (it has no multi-GPU path). */
int b200_shard_range(int64_t n, int64_t world, int64_t rank, int64_t granule, int64_t* n_begin,
                     int64_t* n_end);

/* ------------------------------------------------------------------------ */
/* Failure detection                                                         */
/* ------------------------------------------------------------------------ */

/* Launches one kernel that waits on an mbarrier nothing arrives on, with a
 * budget of timeout_ns; the wait gives up, writes B200_DEV_TIMEOUT_SELFTEST to
 * *status (device int, caller-zeroed) and the kernel returns normally. Tests
 * the bounded-wait machinery every kernel here relies on instead of the
 * reference's unbounded spins (src/memory/tma.cu:404-408). */
int b200_selftest_bounded_wait(unsigned long long timeout_ns, int* status, void* stream);

/* Launches `ctas` CTAs of 32 threads with smem_bytes of dynamic shared memory
 * each (large enough to keep one CTA per SM) that hold their SMs for hold_ns
 * (at most 5 s) of timer time and return. Stands in for another kernel sharing
 * the GPU, so tests can check that a GEMM launched meanwhile on another stream
 * completes correctly with only part of the SMs free. No counterpart in the
 * reference. */
int b200_selftest_occupy(int ctas, int smem_bytes, unsigned long long hold_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200GEMM_H_ */
