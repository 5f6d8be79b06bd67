// Persistent, warp-specialised BF16 GEMM for B200 (sm_100a): D = A * B^T.
//
// This is the GEMM candidate that replaces, behind the reference driver's
// plan API, the CuTe DSL PersistentDenseGemmKernel / DenseGemmKernel and the
// cuBLASLt call the reference study measures (driven by
// src/gemm/gemm_comparison.py:2813-2876 and src/gemm/cublaslt_bridge_p35.cu:949-985;
// candidate table gemm_comparison.py:214-265). Layout contract "TN":
// A M x K row-major, B N x K row-major, D M x N row-major (gemm_comparison.py:2670-2691).
//
// One CTA per SM (1-CTA mode) or one CTA pair per two SMs (tcgen05
// cta_group::2), 192 threads:
//   warp 0      TMA producer: one elected lane streams 128*sub_m x 64 A and
//               (256/cta_group) x 64 B K-slices into a ring of `kStages`
//               128B-swizzled SMEM slots, guarded by full/empty mbarriers. The
//               leader's producer also takes tile ids from a global counter and
//               publishes them through a shared-memory queue (dynamic schedule).
//   warp 1      allocates all 512 TMEM columns; one elected lane (leader CTA
//               only in pair mode) issues tcgen05.mma kind::f16 into 128 x 256
//               fp32 accumulators ("units") rotating through two TMEM slots,
//               and frees ring slots with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld 32 rows each -> bf16/fp32 -> swizzled
//               SMEM staging -> TMA store (and, for the fused multi-GPU gather,
//               the same chunk to every peer's D); a unit's TMEM slot is handed
//               back as soon as it is in registers, so the epilogue overlaps the
//               next MMAs.
// Tile shapes: 128 x 256 (1-CTA), 256 x 256 per pair (sub_m = 1, successive
// tiles double-buffer TMEM) and 512 x 256 per pair (sub_m = 2, a tile's two
// row halves fill TMEM; 25 % fewer L2->SM bytes per FLOP).
//
// Pair mode: M = 256 MMAs issued by the even CTA. Each CTA loads its own A
// rows and its half of B (unicast TMA) and signals the leader's full barrier;
// the leader's commits are sent to each CTA's barrier separately (two unicast
// commits, no multicast anywhere).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "internal.h"
#include "ptx.cuh"

namespace b200 {

constexpr int kBK = 64;            // K elements per ring slot (128 bytes: one swizzle atom row)
constexpr int kBN = 256;           // MMA N: columns of D per tile (the 2CTA_N128 tile: 128)
constexpr int kRowsPerCta = 128;   // D rows per CTA per tile (TMEM lanes)
constexpr int kThreads = 192;
constexpr int kEpiWarps = 4;
constexpr int kEpiBufBytes = 32 * 128;  // one warp's staging tile: 32 rows x 128 bytes
constexpr int kTmemCols = 2 * kBN;      // double-buffered accumulator
constexpr int kQueue = 4;
constexpr int kMaxPeers = 7;            // fused gather: up to 8 GPUs               // tile-id queue slots (producer -> MMA, epilogue, peer)

// kSubM = 128-row accumulators each CTA owns per tile. 1: tile = 128 x 256 per
// CTA and the two 256-column TMEM slots double-buffer successive tiles.
// 2 (pair mode only): tile = 256 x 256 per CTA (512 x 256 per pair), the two
// slots hold the tile's two row halves; each is handed back to the MMA warp as
// soon as the epilogue has drained it. Per k-slice a CTA then loads 48 KiB for
// 2 x 4.2 MFLOP instead of 32 KiB for 4.2 MFLOP: 25 % fewer L2->SM bytes.
// kTileN = 128 (pair mode, one accumulator per tile): 256 x 128 pair tiles,
// twice as many tiles as 256 x 256, for shapes whose 256-wide tiles leave the
// last wave half empty; the smaller stages give the ring eight slots.
template <int kCtaGroup, int kSubM, int kTileN = kBN>
struct GemmCfg {
    static_assert(kSubM == 1 || (kSubM == 2 && kCtaGroup == 2), "unsupported tile shape");
    static_assert(kTileN == kBN || (kTileN == 128 && kCtaGroup == 2 && kSubM == 1), "unsupported tile N");
    static constexpr int kStages = kTileN == 128 ? 8 : ((kCtaGroup == 1 || kSubM == 2) ? 4 : 6);
    static constexpr int kARows = kRowsPerCta * kSubM;
    static constexpr int kABytes = kARows * kBK * 2;
    static constexpr int kBRows = kTileN / kCtaGroup;
    static constexpr int kBBytes = kBRows * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kTileM = kARows * kCtaGroup;
    static constexpr int kEpiOffset = kStages * kStageBytes;
    static constexpr int kEpiBytes = kEpiWarps * 2 * kEpiBufBytes;
    static constexpr int kBarOffset = kEpiOffset + kEpiBytes;
    // full[S], empty[S], tfull[2], tempty[2], qfull[Q], qempty[Q], TMEM address, tile-id ring[Q]
    static constexpr int kBarCount = 2 * kStages + 4 + 2 * kQueue;
    static constexpr int kBarBytes = kBarCount * 8 + 16 + 4 * kQueue;
    static constexpr int kSmemBytes = kBarOffset + kBarBytes + 1024;  // + alignment slack
    static_assert(kStageBytes % 1024 == 0, "ring slots must keep 1024-byte alignment");
    static_assert(kSmemBytes <= 232448, "exceeds the 227 KB opt-in shared memory");
};

struct GemmParams {
    int m, n, k;
    int num_m_blocks, num_n_blocks, num_k_blocks;
    int num_tiles;
    int group_m;     // blocks per raster group along the grouped dimension
    int raster_n;    // 0: groups of m-blocks walk all n-blocks; 1: groups of n-blocks walk all m-blocks
    int* status;
    // Dynamic tile scheduler: [0] next tile id, [1] fetchers that found the end.
    // Zero before a launch; the last fetcher of every launch zeroes it again.
    int* tile_counter;
    unsigned long long timeout_ns;
    // Optional timeline (nullptr = off): per CTA kTraceSlots %globaltimer stamps.
    unsigned long long* trace;
    // Fused gather (N-sharded multi-GPU): every staged output chunk is also
    // written with 16-byte stores into each peer GPU's copy of the full D, at
    // the same row/column (peer_d already points at this shard's columns;
    // the same row pitch as the local D). npeers = 0: off.
    int npeers;
    int peer_tma;    // 1: peer chunks go out as TMA bulk stores (PeerMaps), 0: 16-byte stores
    long long ldd;
    void* peer_d[kMaxPeers];
    // Multicast gather (NVLS): every staged chunk is also written once, with
    // 16-byte multimem stores, at the same row/column of this multicast
    // address (already at this shard's first column, row pitch ldd); the switch
    // replicates it into every GPU's full D. nullptr: off.
    void* mc_d;
    // Stream-K schedule (sk_iters > 0; otherwise the dynamic schedule above).
    // The clusters form sk_groups groups of sk_lanes; group g, lane l is
    // cluster g * sk_lanes + l (clusters past the last group get no work). A
    // group works on "super-tiles": with one lane a super-tile is a tile of
    // the raster walk; with several it is one m-block (sk_lane_n = 1, lane l
    // takes n-block l) or one n-block (lane l takes m-block l), so the tiles
    // that share an A (or B) panel run the same k-slices at the same time.
    // The first sk_iters / num_k_blocks super-tiles (the "split block") are
    // cut into sk_groups equal runs of k-slices, one per group, run first;
    // then `sk_rounds` rounds of whole super-tiles follow (split + j *
    // sk_groups + g in round j), so every group ends at the same time on whole
    // tiles and the reductions of the cut tiles overlap the later MMAs. A cut
    // super-tile is finished by the group that runs its last k-slices (that
    // group's last split-block run) after every earlier group holding a run of
    // it (their first run) has left its fp32 partial in its own slot of
    // sk_partial and set its sk_flags word; the finisher adds the partials in
    // k order, writes D and clears the flags.
    int sk_rounds;
    int sk_groups;
    int sk_lanes;
    int sk_lane_n;
    long long sk_iters;   // k-slices in the split block (per lane)
    float* sk_partial;    // [cluster][cta rank][sub_m][warp] x 32 x 256 fp32
    int* sk_flags;        // same indexing, one int each; zero between launches
    // Failure-path test hook (B200_TEST_DROP_PARTIAL_FLAGS at plan creation):
    // partial writers skip their flag, so finishers' bounded waits run out and
    // report B200_DEV_TIMEOUT_PARTIAL. Nothing faults or hangs.
    int sk_test_drop_flags;
    // K walk direction of the dynamic schedule ("K serpentine"): with
    // kserp_wave > 0, the tiles of odd waves (tile id / kserp_wave odd) run
    // their k-slices from the last to the first, so each wave starts on the
    // k-slices the previous wave left most recently in L2 instead of on the
    // ones it evicted first. The direction is a function of the tile id alone,
    // so results stay bit-identical from launch to launch.
    int kserp_wave;
};

// Tensor maps of the peers' D slices for the TMA form of the fused gather.
struct PeerMaps {
    CUtensorMap map[kMaxPeers];
};

// Trace slots per CTA: 0 entry, 1 setup done, 2 producer done, 3 MMA done,
// 4 epilogue done, 5 exit, 6.. the epilogue's "accumulator ready" time of each
// tile this CTA processed (up to kTraceSlots - 6 tiles).
constexpr int kTraceSlots = 64;

__device__ __forceinline__ void trace_stamp(const GemmParams& p, int slot) {
    if (p.trace != nullptr && slot < kTraceSlots)
        p.trace[static_cast<size_t>(blockIdx.x) * kTraceSlots + slot] = globaltimer_ns();
}

// One unit of a cluster's work: super-tile t over k-slices [kb0, kb1).
// role 0: the whole K range; 1: a run that stops short of K (its fp32 partial
// goes to this cluster's slot); 2: a run that ends at K but does not start at
// k-slice 0 (finished with the partials of the earlier groups).
struct WorkItem {
    int t, kb0, kb1, role;
};

struct SkCursor {
    int group, lane, round;
    long long lo, hi;  // the group's split-block k-slices not yet walked: [lo, hi)
};

__device__ __forceinline__ long long sk_group_start(const GemmParams& p, int g) {
    return static_cast<long long>(g) * p.sk_iters / p.sk_groups;
}

__device__ __forceinline__ void sk_begin(const GemmParams& p, int cluster, SkCursor& cur) {
    cur.group = cluster / p.sk_lanes;
    cur.lane = cluster - cur.group * p.sk_lanes;
    cur.round = 0;
    if (cur.group >= p.sk_groups) {  // spare cluster: no work
        cur.round = p.sk_rounds;
        cur.lo = cur.hi = 0;
        return;
    }
    cur.lo = sk_group_start(p, cur.group);
    cur.hi = sk_group_start(p, cur.group + 1);
}

// Next item of the cluster's static stream-K walk; false at the end. Every
// role of a CTA walks the same sequence. The split block is walked from the
// group's last super-tile down to its first: the run that stops short of K
// (a partial for a LATER group to finish) comes first, the run that finishes a
// super-tile begun by EARLIER groups comes last. A finisher therefore only
// ever waits for lower-numbered clusters; the hardware dispatches clusters in
// index order, so whenever a finisher is resident its writers are resident or
// done, even when other work holds some SMs.
__device__ __forceinline__ bool sk_next(const GemmParams& p, SkCursor& cur, WorkItem& w) {
    const int nk = p.num_k_blocks;
    if (cur.lo < cur.hi) {
        const long long tl = (cur.hi - 1) / nk;
        const long long lo = max(cur.lo, tl * nk);
        const int kb0 = static_cast<int>(lo - tl * nk);
        const int kb1 = static_cast<int>(cur.hi - tl * nk);
        w = {static_cast<int>(tl), kb0, kb1, kb1 < nk ? 1 : (kb0 > 0 ? 2 : 0)};
        cur.hi = lo;
        return true;
    }
    if (cur.round >= p.sk_rounds) return false;
    w = {static_cast<int>(p.sk_iters / nk) + cur.round * p.sk_groups + cur.group, 0, nk, 0};
    ++cur.round;
    return true;
}

// Linear tile id -> (m block, n block): M-grouped raster so that the tiles in
// flight at one time share A rows and B rows in L2.
__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& mb, int& nb) {
    const int major = p.raster_n ? p.num_n_blocks : p.num_m_blocks;  // grouped dimension
    const int minor = p.raster_n ? p.num_m_blocks : p.num_n_blocks;
    const int per_group = p.group_m * minor;
    const int g = t / per_group;
    const int first = g * p.group_m;
    const int gsize = min(p.group_m, major - first);
    const int r = t - g * per_group;
    const int a = first + r % gsize;
    const int b = r / gsize;
    mb = p.raster_n ? b : a;
    nb = p.raster_n ? a : b;
}

// (m block, n block) of lane `lane`'s tile in super-tile t (stream-K).
__device__ __forceinline__ void sk_tile_coords(int t, int lane, const GemmParams& p, int& mb, int& nb) {
    if (p.sk_lanes == 1) {
        tile_coords(t, p, mb, nb);
    } else if (p.sk_lane_n) {
        mb = t;
        nb = lane;
    } else {
        mb = lane;
        nb = t;
    }
}

// kStreamK selects the stream-K schedule at compile time, so the dynamic
// schedule's kernels carry none of its code (it measured 0.4-1 % on them).
template <int kCtaGroup, int kSubM, bool kOutF32, bool kStreamK, int kTileN = kBN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tn_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmD, const GemmParams p,
                     const __grid_constant__ PeerMaps peers) {
    using C = GemmCfg<kCtaGroup, kSubM, kTileN>;
    // This instantiation's tile width (shadows the namespace-wide 256).
    constexpr int kBN = kTileN;
    constexpr int kTmemCols = 2 * kBN;
    static_assert(!kStreamK || kTileN == b200::kBN, "stream-K runs 256-wide tiles only");
    constexpr int kStages = C::kStages;
    constexpr int kColsPerChunk = kOutF32 ? 32 : 64;  // output columns per 128-byte staging row
    constexpr int kChunks = kBN / kColsPerChunk;
    constexpr bool kPair = kCtaGroup == 2;

    // Launch contract: uniform across the grid, checked before any barrier.
    if (blockDim.x != kThreads || blockDim.y != 1 || blockDim.z != 1 ||
        (kPair && cluster_nctarank() != 2) || (gridDim.x % kCtaGroup) != 0) {
        if (threadIdx.x == 0) report_status(p.status, B200_DEV_BAD_LAUNCH);
        return;
    }

    if (threadIdx.x == 0) trace_stamp(p, 0);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t full0 = sbase + C::kBarOffset;
    const uint32_t empty0 = full0 + 8 * kStages;
    const uint32_t tfull0 = empty0 + 8 * kStages;
    const uint32_t tempty0 = tfull0 + 16;
    const uint32_t qfull0 = tempty0 + 16;
    const uint32_t qempty0 = qfull0 + 8 * kQueue;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOffset + C::kBarCount * 8);
    volatile int* ring = reinterpret_cast<volatile int*>(smem + C::kBarOffset + C::kBarCount * 8 + 16);
    const uint32_t ring_addr = smem_u32(const_cast<int*>(ring));

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = kPair ? cluster_ctarank() : 0;
    const int num_clusters = gridDim.x / kCtaGroup;
    const int cluster = blockIdx.x / kCtaGroup;
    // Stream-K runs only with one accumulator per tile (see the epilogue's finisher).
    static_assert(!kStreamK || kSubM == 1, "stream-K needs one accumulator per tile");
    constexpr bool sk = kStreamK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull0 + 8 * a, 1);
            mbar_init(tempty0 + 8 * a, kEpiWarps * kCtaGroup);
        }
        // A queued tile id is read by the MMA issuer and 4 epilogue warps of the
        // leader, and in pair mode also by the peer's producer and 4 epilogue warps.
        for (int q = 0; q < kQueue; ++q) {
            mbar_init(qfull0 + 8 * q, 1);
            mbar_init(qempty0 + 8 * q, kPair ? 10 : 5);
        }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmD);
    }
    if (warp == 1) {
        tmem_alloc<kCtaGroup>(smem_u32(tmem_slot), kTmemCols);
        tmem_relinquish<kCtaGroup>();
    }
    tc_fence_before();
    if constexpr (kPair) cluster_sync(); else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
    // Everything above touched only shared memory, TMEM and the kernel
    // parameters, so with programmatic dependent launch it overlaps the tail of
    // the previous kernel in the stream; no global memory (operands, D, the tile
    // counter, the status word) is touched before this wait.
    griddep_wait();
    if (threadIdx.x == 0) trace_stamp(p, 1);

    // Tile-id queue. The leader's producer fetches ids from the global counter
    // in launch-wide order (so tiles sharing A/B panels run at the same time
    // whatever the drift between pairs) and publishes them to every consumer;
    // -1 ends the walk. Consumers read a slot and release it at once.
    auto queue_wait = [&](uint32_t qs, uint32_t qph, int code) -> bool {
        return mbar_wait<kPair>(qfull0 + 8 * qs, qph, p.status, p.timeout_ns, code);
    };
    auto queue_release = [&](uint32_t qs) {
        if constexpr (kPair) mbar_arrive_cluster(mapa_shared(qempty0 + 8 * qs, 0));
        else mbar_arrive(qempty0 + 8 * qs);
    };

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (elect_one()) {
            uint32_t stage = 0, phase = 0, qs = 0, qph = 0;
            long long issued = 0;  // ring slots armed so far (failure-path drain)
            bool ok = true;
            // The leader fetches the first tile id now and each later one while the
            // current tile is still loading (see fetch_kb).
            int next = (rank == 0 && !sk) ? atomicAdd(&p.tile_counter[0], 1) : -1;
            SkCursor cur;
            if (sk) sk_begin(p, cluster, cur);
            while (ok) {
                int t, kb0 = 0, kb1 = p.num_k_blocks;
                if (sk) {
                    WorkItem w;
                    t = sk_next(p, cur, w) ? w.t : -1;
                    if (t >= 0) { kb0 = w.kb0; kb1 = w.kb1; }
                } else if (rank == 0) {
                    // Publish the prefetched tile id.
                    if (!mbar_wait(qempty0 + 8 * qs, qph ^ 1, p.status, p.timeout_ns,
                                   B200_DEV_TIMEOUT_PRODUCER)) {
                        break;
                    }
                    t = next;
                    if (t >= p.num_tiles) {
                        t = -1;
                        __threadfence();
                        if (atomicAdd(&p.tile_counter[1], 1) == num_clusters - 1) {
                            // Every fetcher has made its last increment: re-arm the counter.
                            atomicExch(&p.tile_counter[0], 0);
                            atomicExch(&p.tile_counter[1], 0);
                        }
                    }
                    ring[qs] = t;
                    if constexpr (kPair) {
                        st_shared_cluster_u32(mapa_shared(ring_addr + 4 * qs, 1), static_cast<uint32_t>(t));
                        mbar_arrive_cluster(mapa_shared(qfull0 + 8 * qs, 1));
                    }
                    mbar_arrive(qfull0 + 8 * qs);
                } else {
                    if (!queue_wait(qs, qph, B200_DEV_TIMEOUT_PRODUCER)) break;
                    t = ring[qs];
                    queue_release(qs);
                }
                if (++qs == kQueue) { qs = 0; qph ^= 1; }
                if (t < 0) {
                    // No more tiles for this CTA: the next launch may start its setup.
                    griddep_launch_dependents();
                    break;
                }
                int mb, nb;
                if (sk) sk_tile_coords(t, cur.lane, p, mb, nb);
                else tile_coords(t, p, mb, nb);
                const int a_row = mb * C::kTileM + static_cast<int>(rank) * C::kARows;
                const int b_row = nb * kBN + static_cast<int>(rank) * C::kBRows;
                // The next tile id is fetched late in this tile (two ring depths
                // before its last k-slice): early enough to hide the atomic's round
                // trip, late enough that a fast pair cannot take two tiles while a
                // slow one has none.
                const int fetch_kb = max(0, p.num_k_blocks - 2 * kStages);
                const bool rev = !sk && p.kserp_wave > 0 && ((t / p.kserp_wave) & 1);
                for (int i = kb0; i < kb1; ++i) {
                    const int kb = rev ? kb0 + kb1 - 1 - i : i;
                    if (!sk && rank == 0 && i == fetch_kb) next = atomicAdd(&p.tile_counter[0], 1);
                    if (!mbar_wait(empty0 + 8 * stage, phase ^ 1, p.status, p.timeout_ns,
                                   B200_DEV_TIMEOUT_PRODUCER)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = sbase + stage * C::kStageBytes;
                    const uint32_t sb = sa + C::kABytes;
                    const uint32_t fb = full0 + 8 * stage;
                    if constexpr (!kPair) {
                        mbar_arrive_expect_tx(fb, C::kStageBytes);
                        tma_load_2d(sa, &tmA, fb, kb * kBK, a_row);
                        tma_load_2d(sb, &tmB, fb, kb * kBK, b_row);
                    } else {
                        const uint32_t leader_fb = mapa_shared(fb, 0);
                        if (rank == 0) mbar_arrive_expect_tx(fb, 2 * C::kStageBytes);
                        tma_load_2d_pair(sa, &tmA, leader_fb, kb * kBK, a_row);
                        tma_load_2d_pair(sb, &tmB, leader_fb, kb * kBK, b_row);
                    }
                    ++issued;
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
            }
            if (status_failed(p.status) && rank == 0) {
                // The launch is being abandoned: before this CTA (pair) exits, wait
                // (bounded) for the TMA loads it still has in flight into its ring.
                const unsigned long long drain_ns = min(p.timeout_ns, 100000000ull);
                for (int s = 0; s < kStages; ++s) {
                    if (issued <= s) continue;
                    const long long last = ((issued - 1 - s) / kStages) * kStages + s;
                    mbar_wait(full0 + 8 * s, static_cast<uint32_t>((last / kStages) & 1), nullptr,
                              drain_ns, 0);
                }
            }
            trace_stamp(p, 2);
        }
        __syncwarp();
    } else if (warp == 1) {
        // --------------------------------------------------------- MMA issuer
        if (rank == 0 && elect_one()) {
            constexpr uint32_t idesc = idesc_bf16_f32(kRowsPerCta * kCtaGroup, kBN);
            // Accumulator unit u (kSubM per tile) lives in TMEM slot u & 1; its
            // barriers' phase flips every second unit.
            uint32_t stage = 0, phase = 0, unit = 0, qs = 0, qph = 0;
            bool ok = true;
            SkCursor cur;
            if (sk) sk_begin(p, cluster, cur);
            while (ok) {
                int kb0 = 0, kb1 = p.num_k_blocks;
                if (sk) {
                    WorkItem w;
                    if (!sk_next(p, cur, w)) break;
                    kb0 = w.kb0;
                    kb1 = w.kb1;
                } else {
                    if (!queue_wait(qs, qph, B200_DEV_TIMEOUT_MMA_FULL)) break;
                    const int t = ring[qs];
                    queue_release(qs);
                    if (++qs == kQueue) { qs = 0; qph ^= 1; }
                    if (t < 0) break;
                }
                // MMAs of row half `sm` for k-slice `kb` held in ring slot `st`; the
                // item's first k-slice of a half waits for its TMEM slot (and
                // overwrites the accumulator), the last one signals the epilogue.
                auto issue_sub = [&](int sm, uint32_t st, int kb) -> bool {
                    const uint32_t u = unit + sm;
                    const uint32_t slot = u & 1;
                    if (kb == kb0) {
                        if (!mbar_wait<kPair>(tempty0 + 8 * slot, ((u >> 1) & 1) ^ 1, p.status,
                                              p.timeout_ns, B200_DEV_TIMEOUT_MMA_TMEM)) {
                            return false;
                        }
                        tc_fence_after();
                    }
                    const uint32_t sa = sbase + st * C::kStageBytes;
                    const uint32_t sb = sa + C::kABytes;
                    const uint32_t d_tmem = tmem_base + slot * kBN;
                    const uint32_t a_sub = sa + sm * (kRowsPerCta * kBK * 2);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        umma_bf16<kCtaGroup>(d_tmem, smem_desc_sw128(a_sub + 32 * k),
                                             smem_desc_sw128(sb + 32 * k), idesc,
                                             (kb != kb0 || k != 0) ? 1u : 0u);
                    }
                    if (kb == kb1 - 1) {
                        const uint32_t tb = tfull0 + 8 * slot;
                        if constexpr (!kPair) {
                            umma_commit<1>(tb);
                        } else {
                            umma_commit<2>(mapa_shared(tb, 0));
                            umma_commit<2>(mapa_shared(tb, 1));
                        }
                    }
                    return true;
                };
                auto wait_full = [&](uint32_t st, uint32_t ph) -> bool {
                    if (!mbar_wait(full0 + 8 * st, ph, p.status, p.timeout_ns,
                                   B200_DEV_TIMEOUT_MMA_FULL)) {
                        return false;
                    }
                    tc_fence_after();
                    return true;
                };
                auto release_stage = [&](uint32_t st) {
                    const uint32_t eb = empty0 + 8 * st;
                    if constexpr (!kPair) {
                        umma_commit<1>(eb);
                    } else {
                        umma_commit<2>(mapa_shared(eb, 0));
                        umma_commit<2>(mapa_shared(eb, 1));
                    }
                };
                // Head start (two row halves): the first half runs over the first
                // `head` k-slices while the epilogue is still draining the second
                // half's slot; those ring slots are held until the second half has
                // used them too.
                const int head = kSubM == 2 ? min(kStages, kb1 - kb0) : 0;
                if (head > 0) {
                    uint32_t st = stage, ph = phase;
                    for (int kb = kb0; ok && kb < kb0 + head; ++kb) {
                        ok = wait_full(st, ph) && issue_sub(0, st, kb);
                        if (++st == kStages) { st = 0; ph ^= 1; }
                    }
                    for (int kb = kb0; ok && kb < kb0 + head; ++kb) {
                        ok = issue_sub(1, stage, kb);
                        if (!ok) break;
                        release_stage(stage);
                        if (++stage == kStages) { stage = 0; phase ^= 1; }
                    }
                }
                for (int kb = kb0 + head; ok && kb < kb1; ++kb) {
                    ok = wait_full(stage, phase);
#pragma unroll
                    for (int sm = 0; ok && sm < kSubM; ++sm) ok = issue_sub(sm, stage, kb);
                    if (!ok) break;
                    release_stage(stage);
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
                unit += kSubM;
            }
            trace_stamp(p, 3);
        }
        __syncwarp();
    } else {
        // ----------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const uint32_t stage_buf0 = sbase + C::kEpiOffset + q * 2 * kEpiBufBytes;
        uint32_t unit = 0, buf = 0, qs = 0, qph = 0;
        int local_tile = 0;
        bool ok = true;
        SkCursor cur;
        if (sk) sk_begin(p, cluster, cur);
        for (; ok; ++local_tile) {
            int t, role = 0;
            if (sk) {
                WorkItem w;
                t = sk_next(p, cur, w) ? w.t : -1;
                if (t >= 0) role = w.role;
            } else {
                if (!queue_wait(qs, qph, B200_DEV_TIMEOUT_EPILOGUE)) break;
                t = ring[qs];
                __syncwarp();
                if (lane == 0) queue_release(qs);
                if (++qs == kQueue) { qs = 0; qph ^= 1; }
            }
            if (t < 0) break;
            int mb, nb;
            if (sk) sk_tile_coords(t, cur.lane, p, mb, nb);
            else tile_coords(t, p, mb, nb);
            const int col0 = nb * kBN;
            // A finisher (role 2) adds the partials of the earlier groups whose runs
            // lie inside this super-tile, in k order: groups group-nwriters .. group-1.
            int nwriters = 0;
            if (role == 2) {
                const long long tile_start = static_cast<long long>(t) * p.num_k_blocks;
                while (cur.group - 1 - nwriters >= 0 &&
                       sk_group_start(p, cur.group - nwriters) > tile_start) {
                    ++nwriters;
                }
            }
            for (int sm = 0; sm < kSubM; ++sm, ++unit) {
                const uint32_t slot = unit & 1;
                const int row0 = mb * C::kTileM + static_cast<int>(rank) * C::kARows +
                                 sm * kRowsPerCta + q * 32;
                const uint32_t t_row = tmem_base + slot * kBN + (static_cast<uint32_t>(q * 32) << 16);
                // Stream-K partial of this warp's 32 x 256 accumulator block, kept in
                // the slot of the cluster that computed it, laid out [32-column
                // chunk][float4 column group][lane] so that every warp access is 512
                // contiguous bytes.
                auto slot_of = [&](int cl) -> long long {
                    return ((static_cast<long long>(cl) * kCtaGroup + rank) * kSubM + sm) * kEpiWarps + q;
                };
                auto writer_cluster = [&](int w) { return (cur.group - nwriters + w) * p.sk_lanes + cur.lane; };
                auto partial_src = [&](int w) {
                    return reinterpret_cast<const float4*>(p.sk_partial) +
                           slot_of(writer_cluster(w)) * (32 * kBN / 4) + lane;
                };
                // Without whole-tile rounds after the split block a finisher's item is
                // the CTA's last, so the other TMEM slot is free: the partials are
                // summed into it while the item's MMAs still run, and only TMEM reads
                // remain at the end. With rounds to follow, the partials are added
                // from L2 while the next whole tile's MMAs run.
                const bool stage_in_tmem = p.sk_rounds == 0;
                const uint32_t t_stage = tmem_base + (slot ^ 1) * kBN + (static_cast<uint32_t>(q * 32) << 16);
                if (role == 2) {
                    // Wait (bounded) for every earlier run's partial.
                    bool got = true;
#pragma unroll 1
                    for (int w = 0; w < nwriters && got; ++w) {
                        const int* flag = p.sk_flags + slot_of(writer_cluster(w));
                        got = ld_acquire_gpu(flag) != 0;
                        const uint64_t t0 = globaltimer_ns();
                        while (!got) {
#pragma unroll 1
                            for (int i = 0; i < 32 && !got; ++i) got = ld_acquire_gpu(flag) != 0;
                            if (got || status_failed(p.status)) break;
                            if (globaltimer_ns() - t0 > p.timeout_ns) {
                                report_status(p.status, B200_DEV_TIMEOUT_PARTIAL);
                                break;
                            }
                        }
                    }
                    if (!__all_sync(0xffffffffu, got)) {
                        ok = false;
                        break;
                    }
                    // Consumed in this launch; the next launch's writers set them again.
                    for (int w = lane; w < nwriters; w += 32) p.sk_flags[slot_of(writer_cluster(w))] = 0;
                    if (stage_in_tmem) {
                        // One 32-column chunk per batch: this path only runs when no whole
                        // tiles follow the split block (never under the auto policy, which
                        // needs three waves), so it is kept small in registers.
                        constexpr int kBatch = 1;
#pragma unroll 1
                        for (int c0 = 0; c0 < kBN / 32; c0 += kBatch) {
                            uint32_t r[kBatch][32];
#pragma unroll
                            for (int j = 0; j < kBatch; ++j) {
#pragma unroll
                                for (int i = 0; i < 8; ++i) {
                                    const float4 v = __ldcg(partial_src(0) + ((c0 + j) * 8 + i) * 32);
                                    r[j][4 * i] = __float_as_uint(v.x);
                                    r[j][4 * i + 1] = __float_as_uint(v.y);
                                    r[j][4 * i + 2] = __float_as_uint(v.z);
                                    r[j][4 * i + 3] = __float_as_uint(v.w);
                                }
                            }
#pragma unroll 1
                            for (int w = 1; w < nwriters; ++w) {
#pragma unroll
                                for (int j = 0; j < kBatch; ++j) {
#pragma unroll
                                    for (int i = 0; i < 8; ++i) {
                                        const float4 v = __ldcg(partial_src(w) + ((c0 + j) * 8 + i) * 32);
                                        r[j][4 * i] = __float_as_uint(__uint_as_float(r[j][4 * i]) + v.x);
                                        r[j][4 * i + 1] = __float_as_uint(__uint_as_float(r[j][4 * i + 1]) + v.y);
                                        r[j][4 * i + 2] = __float_as_uint(__uint_as_float(r[j][4 * i + 2]) + v.z);
                                        r[j][4 * i + 3] = __float_as_uint(__uint_as_float(r[j][4 * i + 3]) + v.w);
                                    }
                                }
                            }
#pragma unroll
                            for (int j = 0; j < kBatch; ++j) tmem_st_32x32b_x32(t_stage + (c0 + j) * 32, r[j]);
                        }
                        tmem_st_wait();
                    }
                }
                if (!mbar_wait<kPair, true>(tfull0 + 8 * slot, (unit >> 1) & 1, p.status,
                                            p.timeout_ns, B200_DEV_TIMEOUT_EPILOGUE)) {
                    ok = false;
                    break;
                }
                if (sm == 0 && warp == 2 && lane == 0) trace_stamp(p, 6 + local_tile);
                tc_fence_after();
                // Finisher: accumulator + partials (summed in k order of the runs).
                auto add_partial = [&](int c32, uint32_t (&r)[32]) {
                    if (stage_in_tmem) {
                        uint32_t t[32];
                        tmem_ld_32x32b_x32(t_stage + c32 * 32, t);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(t[i]));
                        return;
                    }
                    // Sum of the partials in k order first, then onto the accumulator:
                    // the same association as the TMEM-staged path.
                    float4 acc[8];
#pragma unroll 1
                    for (int w = 0; w < nwriters; ++w) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float4 v = __ldcg(partial_src(w) + (c32 * 8 + i) * 32);
                            if (w == 0) {
                                acc[i] = v;
                            } else {
                                acc[i].x += v.x;
                                acc[i].y += v.y;
                                acc[i].z += v.z;
                                acc[i].w += v.w;
                            }
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        r[4 * i] = __float_as_uint(__uint_as_float(r[4 * i]) + acc[i].x);
                        r[4 * i + 1] = __float_as_uint(__uint_as_float(r[4 * i + 1]) + acc[i].y);
                        r[4 * i + 2] = __float_as_uint(__uint_as_float(r[4 * i + 2]) + acc[i].z);
                        r[4 * i + 3] = __float_as_uint(__uint_as_float(r[4 * i + 3]) + acc[i].w);
                    }
                };
                // Stage one 32-row x 128-byte chunk of this warp's rows and TMA-store it.
                auto store_chunk = [&](int c, const uint32_t* packed) {
                    // Chunks wholly outside D are skipped before touching the staging
                    // buffers: every staged chunk must commit one bulk group, or the
                    // wait_group.read accounting below would let a later chunk overwrite
                    // a buffer whose store is still reading it.
                    const int col = col0 + c * kColsPerChunk;
                    if (row0 >= p.m || col >= p.n) return;
                    const uint32_t sbuf = stage_buf0 + buf * kEpiBufBytes;
                    if (lane == 0) bulk_wait_group_read<1>();
                    __syncwarp();
                    const uint32_t row_addr = sbuf + lane * 128;
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), packed[4 * j], packed[4 * j + 1],
                                     packed[4 * j + 2], packed[4 * j + 3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmD, sbuf, col, row0);
                        if (p.peer_tma) {
                            // Same staged box to every peer's D: one bulk group per chunk.
                            // Rotate the peer order by CTA and chunk so the SMs spread their
                            // traffic over all destinations instead of all hitting one peer.
                            const int g0 = static_cast<int>(blockIdx.x + c + q) % p.npeers;
                            for (int i = 0; i < p.npeers; ++i) {
                                const int g = g0 + i < p.npeers ? g0 + i : g0 + i - p.npeers;
                                tma_store_2d(&peers.map[g], sbuf, col, row0);
                            }
                        }
                        bulk_commit_group();
                    }
                    if (p.mc_d != nullptr) {
                        // Multicast gather: 8 lanes cover one 128-byte staged row, one
                        // 16-byte multimem store each; the switch fans it out to all GPUs.
                        constexpr int kElem = 128 / kColsPerChunk;
                        const int piece = lane & 7;
                        const int pcol = col + piece * (16 / kElem);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = (lane >> 3) + 4 * i;
                            if (row0 + r >= p.m || pcol >= p.n) continue;
                            const uint4 v = ld_shared_v4(sbuf + r * 128 + ((piece ^ (r & 7)) << 4));
                            const long long off = (static_cast<long long>(row0 + r) * p.ldd + pcol) * kElem;
                            multimem_st_v4(static_cast<uint8_t*>(p.mc_d) + off, v);
                        }
                    }
                    if (p.npeers > 0 && !p.peer_tma) {
                        // Fused gather: 8 lanes cover one 128-byte staged row, so each
                        // warp store writes four contiguous 128-byte row segments.
                        constexpr int kElem = 128 / kColsPerChunk;
                        const int piece = lane & 7;
                        const int pcol = col + piece * (16 / kElem);
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int r = (lane >> 3) + 4 * i;
                            if (row0 + r >= p.m || pcol >= p.n) continue;
                            const uint4 v = ld_shared_v4(sbuf + r * 128 + ((piece ^ (r & 7)) << 4));
                            const long long off = (static_cast<long long>(row0 + r) * p.ldd + pcol) * kElem;
                            const int g0 = static_cast<int>(blockIdx.x + c + q) % p.npeers;
                            for (int i = 0; i < p.npeers; ++i) {
                                const int g = g0 + i < p.npeers ? g0 + i : g0 + i - p.npeers;
                                *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.peer_d[g]) + off) = v;
                            }
                        }
                    }
                    buf ^= 1;
                };
                auto release_tmem = [&]() {
                    // Accumulator fully read: hand it back to the MMA issuer.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (!kPair) mbar_arrive(tempty0 + 8 * slot);
                        else mbar_arrive_cluster(mapa_shared(tempty0 + 8 * slot, 0));
                    }
                };
                if (role == 1) {
                    // A run that stops short of K: leave the fp32 partial in this
                    // cluster's slot for the finisher; D is not written.
                    float4* part = reinterpret_cast<float4*>(p.sk_partial) +
                                   slot_of(cluster) * (32 * kBN / 4) + lane;
                    int* flag = p.sk_flags + slot_of(cluster);
#pragma unroll 1
                    for (int c = 0; c < kBN / 32; ++c) {
                        uint32_t r[32];
                        tmem_ld_32x32b_x32(t_row + c * 32, r);
                        tmem_ld_wait();
                        if (c == kBN / 32 - 1) release_tmem();
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            __stcg(part + (c * 8 + i) * 32,
                                   make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                               __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])));
                        }
                    }
                    __threadfence();
                    __syncwarp();
                    if (lane == 0 && !p.sk_test_drop_flags) st_release_gpu(flag, 1);
                    continue;
                }
                if constexpr (kOutF32) {
#pragma unroll 1
                    for (int c = 0; c < kChunks; ++c) {
                        uint32_t packed[32];
                        tmem_ld_32x32b_x32(t_row + c * 32, packed);
                        tmem_ld_wait();
                        if (c == kChunks - 1) release_tmem();
                        if (role == 2) add_partial(c, packed);
                        store_chunk(c, packed);
                    }
                } else if (kStreamK) {
                    // bf16 under stream-K: one 64-column chunk at a time (the partial
                    // sums need the registers the drain-all path below keeps packed
                    // rows in).
#pragma unroll 1
                    for (int c = 0; c < kChunks; ++c) {
                        uint32_t r0[32], r1[32], pk[32];
                        tmem_ld_32x32b_x32(t_row + c * 64, r0);
                        tmem_ld_32x32b_x32(t_row + c * 64 + 32, r1);
                        tmem_ld_wait();
                        if (c == kChunks - 1) release_tmem();
                        if (role == 2) {
                            add_partial(2 * c, r0);
                            add_partial(2 * c + 1, r1);
                        }
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            pk[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
                            pk[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
                        }
                        store_chunk(c, pk);
                    }
                } else {
                    // bf16: the whole 256-column row fits in 128 registers once
                    // packed, so drain TMEM completely first and release it before
                    // any store; the next tile's MMAs into this slot start sooner.
                    uint32_t packed[kChunks][32];
#pragma unroll
                    for (int c = 0; c < kChunks; ++c) {
                        uint32_t r0[32], r1[32];
                        tmem_ld_32x32b_x32(t_row + c * 64, r0);
                        tmem_ld_32x32b_x32(t_row + c * 64 + 32, r1);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            packed[c][i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
                            packed[c][16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
                        }
                    }
                    release_tmem();
#pragma unroll
                    for (int c = 0; c < kChunks; ++c) store_chunk(c, packed[c]);
                }
            }
        }
        if (lane == 0) bulk_wait_group<0>();
        if (p.npeers > 0 || p.mc_d != nullptr) __threadfence_system();  // peer writes visible before exit
        __syncwarp();
        if (warp == 2 && lane == 0) trace_stamp(p, 4);
    }

    // Teardown: every role is done with TMEM and with the peer's barriers.
    tc_fence_before();
    if constexpr (kPair) cluster_sync(); else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc<kCtaGroup>(tmem_base, kTmemCols);
    }
    if (threadIdx.x == 0) trace_stamp(p, 5);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, GemmParams, PeerMaps);

// Kernel variants: (cta_group, sub_m) in {(1,1), (2,1), (2,2)} x {bf16, fp32} D.
template <int G, int S, bool K>
static const void* kernel_sym_t(bool f32) {
    return f32 ? reinterpret_cast<const void*>(&gemm_tn_sm100_kernel<G, S, true, K>)
               : reinterpret_cast<const void*>(&gemm_tn_sm100_kernel<G, S, false, K>);
}

static const void* kernel_sym(int cta_group, int sub_m, bool f32, bool stream_k, int tile_n) {
    if (tile_n == 128)
        return f32 ? reinterpret_cast<const void*>(&gemm_tn_sm100_kernel<2, 1, true, false, 128>)
                   : reinterpret_cast<const void*>(&gemm_tn_sm100_kernel<2, 1, false, false, 128>);
    if (cta_group == 1) return stream_k ? kernel_sym_t<1, 1, true>(f32) : kernel_sym_t<1, 1, false>(f32);
    if (sub_m == 2) return kernel_sym_t<2, 2, false>(f32);
    return stream_k ? kernel_sym_t<2, 1, true>(f32) : kernel_sym_t<2, 1, false>(f32);
}

static int smem_bytes_for(int cta_group, int sub_m, int tile_n) {
    if (tile_n == 128) return GemmCfg<2, 1, 128>::kSmemBytes;
    if (cta_group == 1) return GemmCfg<1, 1>::kSmemBytes;
    return sub_m == 2 ? GemmCfg<2, 2>::kSmemBytes : GemmCfg<2, 1>::kSmemBytes;
}

static int stages_for(int cta_group, int sub_m, int tile_n) {
    if (tile_n == 128) return GemmCfg<2, 1, 128>::kStages;
    if (cta_group == 1) return GemmCfg<1, 1>::kStages;
    return sub_m == 2 ? GemmCfg<2, 2>::kStages : GemmCfg<2, 1>::kStages;
}

// Columns of D per tile for a resolved mode.
static int tile_n_for(int resolved_mode) { return resolved_mode == B200_MODE_2CTA_N128 ? 128 : kBN; }

}  // namespace b200

struct B200Plan {
    int device = 0;
    cudaStream_t stream = nullptr;
    int cta_group = 1;
    int sub_m = 1;  // 128-row accumulators per CTA per tile
    int tile_n = 256;  // columns of D per tile
    bool pdl = false;  // launch with programmatic stream serialization
    bool out_f32 = false;
    CUtensorMap tmA{}, tmB{}, tmD{};
    b200::PeerMaps peer_maps{};
    b200::GemmParams params{};
    int grid = 0;
    int smem = 0;
    int* d_status = nullptr;
    size_t words_bytes = 0;  // device words reset after a failed launch (status, counter, stream-K flags)
    bool empty_problem = false;
    B200PlanInfo info{};
};

namespace b200 {

constexpr size_t kPlanWordsBytes = 16;  // status word, pad, 2-int tile counter

// Stream-K layout for a plan with `slots` resident clusters; returns false
// (p untouched) for the dynamic schedule. Lanes: when one side of the tile
// grid is at most 4 blocks wide, each group holds one lane per block of that
// side, so the tiles sharing an A (or B) panel stream the same k-slices at the
// same time and the panel crosses HBM once. A super-tile is cut into at most
// four runs (each group's run is at least a third of K). Only tiles with one
// accumulator per CTA (1-CTA 128 x 256, pair 256 x 256) qualify: the finisher
// adds the partials while later MMAs run. Auto: used when the dynamic
// schedule's last wave would leave more than 10 % of the clusters idle on
// average (busy = waves / ceil(waves) < 0.9) and it runs at least three waves:
// a cut tile costs its CTAs an extra 128 KB out and back through L2 in the
// epilogue (measured on B200 with per-CTA timer stamps: 7-9 us for the run
// that writes a partial, 11-17 us for the finisher, against ~4 us for a whole
// tile with fp32 D), which whole-tile rounds after the split block absorb.
// Measured: 4096^3 and 32768 x 512 x 4096 (3.46 waves) gain 1-3 %; the
// 1.73-wave shapes 16384 x 512 x 4096 and 512 x 16384 x 4096 lose ~3 %.
// B200_GEMM_SCHEDULE=dynamic or =streamk overrides the choice (still subject
// to the tile-shape and run-length rules).
static bool stream_k_layout(GemmParams& p, int slots, int sub_m) {
    if (sub_m != 1) return false;
    bool forced = false;
    if (const char* e = std::getenv("B200_GEMM_SCHEDULE")) {
        if (e[0] == 'd') return false;
        forced = e[0] == 's';
    }
    if (slots < 2 || p.num_tiles < 2) return false;
    if (!forced) {
        const double w = static_cast<double>(p.num_tiles) / slots;
        if (w < 3.0 || w / std::ceil(w) >= 0.9) return false;
    }
    int lanes = 1, lane_n = 0;
    if (p.num_n_blocks <= 4 && p.num_n_blocks <= p.num_m_blocks) {
        lanes = p.num_n_blocks;
        lane_n = 1;
    } else if (p.num_m_blocks <= 4) {
        lanes = p.num_m_blocks;
    }
    const int groups = slots / lanes;
    const long long supers = lanes == 1 ? p.num_tiles : (lane_n ? p.num_m_blocks : p.num_n_blocks);
    if (groups < 2) return false;
    // Split block: the super-tiles left over after whole rounds, or one round
    // more when they are too few for runs of a third of K.
    const long long rounds = supers / groups;
    const long long rest = supers - rounds * groups;
    long long split;
    if (rest == 0) return false;  // whole rounds fill every group already
    if (rest * 3 >= groups) split = rest;
    else if (rounds >= 1) split = rest + groups;
    else return false;
    p.sk_lanes = lanes;
    p.sk_lane_n = lane_n;
    p.sk_groups = groups;
    p.sk_rounds = static_cast<int>((supers - split) / groups);
    p.sk_iters = split * p.num_k_blocks;
    return true;
}

// Bytes of the stream-K partial buffer: one 32 x 256 fp32 block per
// (cluster slot, CTA of the pair, row half, epilogue warp).
static size_t stream_k_partial_bytes(int clusters, int cta_group, int sub_m) {
    return static_cast<size_t>(clusters) * cta_group * sub_m * kEpiWarps * 32 * kBN * sizeof(float);
}

static int check_shape(int64_t m, int64_t n, int64_t k, int64_t ldd, int out_dtype, int mode) {
    if (out_dtype != B200_OUT_BF16 && out_dtype != B200_OUT_F32) {
        set_error("out_dtype=%d is neither B200_OUT_BF16 nor B200_OUT_F32", out_dtype);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (mode != B200_MODE_AUTO && mode != B200_MODE_1CTA && mode != B200_MODE_2CTA &&
        mode != B200_MODE_2CTA_M512 && mode != B200_MODE_2CTA_N128) {
        set_error("mode=%d is not one of AUTO(0), 1CTA(1), 2CTA(2), 2CTA_M512(3), 2CTA_N128(4)", mode);
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (m < 0 || n < 0 || k < 0) {
        set_error("(M,N,K)=(%lld,%lld,%lld): extents must be non-negative", (long long)m,
                  (long long)n, (long long)k);
        return B200_ERR_INVALID_ARGUMENT;
    }
    const int64_t kMax = (int64_t(1) << 31) - 1;
    if (m > kMax || n > kMax || k > kMax) {
        set_error("(M,N,K)=(%lld,%lld,%lld): every extent must be below 2^31", (long long)m,
                  (long long)n, (long long)k);
        return B200_ERR_UNSUPPORTED;
    }
    if (k % 8 != 0) {
        set_error("K=%lld: rows of A and B must be whole 16-byte units for TMA (K %% 8 == 0)",
                  (long long)k);
        return B200_ERR_UNSUPPORTED;
    }
    if (ldd < n) {
        set_error("ldd=%lld is smaller than N=%lld", (long long)ldd, (long long)n);
        return B200_ERR_INVALID_ARGUMENT;
    }
    const int64_t elem = out_dtype == B200_OUT_F32 ? 4 : 2;
    if ((ldd * elem) % 16 != 0) {
        set_error("ldd=%lld: the row pitch of D (%lld bytes) must be a multiple of 16 bytes",
                  (long long)ldd, (long long)(ldd * elem));
        return B200_ERR_UNSUPPORTED;
    }
    return B200_OK;
}

// Raster of the tile walk: tile ids are handed out in launch-wide order, in
// groups of `group` m-blocks that each walk every n-block. Measured on B200
// with ncu DRAM counters (8192^3, 16384^3, 8192 x {14336, 128256} x 4096):
// the least traffic came when a group spans ~4096 rows of A, capped so the
// group's A panel stays within 64 MiB (2048 rows at K = 16384). Overridable
// for tuning with B200_GEMM_GROUP (>= 1) and B200_GEMM_RASTER ("m" or "n").
static void raster_for(const GemmParams& p, int tile_m, int sub_m, int* group, int* raster_n) {
    (void)sub_m;
    const double rows = std::min(4096.0, 64.0 * 1024 * 1024 / (2.0 * std::max(p.k, 64)));
    int g = static_cast<int>(rows / tile_m + 0.5);
    g = std::max(2, std::min(16, g));
    *group = std::min(g, std::max(p.num_m_blocks, 1));
    *raster_n = 0;
    // A B that stays in L2 (<= 64 MiB) and is the narrower side: walk every
    // n-block of one m-block before the next, so A and B each cross HBM once.
    // Measured on B200 (bf16 D): 8192 x {1792, 2048, 4096} x 4096 and
    // 8192 x 3072 x 8192 run 2.7-4 % faster than with m-groups.
    const double b_bytes = 2.0 * static_cast<double>(p.n) * static_cast<double>(p.k);
    if (p.num_n_blocks < p.num_m_blocks && b_bytes <= 64.0 * 1024 * 1024) {
        *raster_n = 1;
        *group = std::max(p.num_n_blocks, 1);
    }
    if (const char* e = std::getenv("B200_GEMM_GROUP")) {
        const int v = std::atoi(e);
        if (v >= 1 && v <= 4096) *group = v;
    }
    if (const char* r = std::getenv("B200_GEMM_RASTER")) *raster_n = (r[0] == 'n' || r[0] == 'N');
}

// K serpentine for the dynamic schedule: on unless B200_GEMM_KSERP=0.
// Measured on B200 (ncu, 8192^3 512 x 256 tiles): DRAM reads 818 -> 661 MB per
// launch and 673 -> 667 us; an L2 evict_last / evict_first policy on the
// operand loads was tried beside it and read more (878 MB) and ran slower.
static int kserp_wave_for(int clusters) {
    if (const char* e = std::getenv("B200_GEMM_KSERP")) {
        if (e[0] == '0') return 0;
    }
    return clusters;
}

// AUTO: small problems that cannot fill the pairs run 1-CTA tiles. Otherwise
// the pair-tile shape with the better score wins, score = waves / ceil(waves)
// (the fraction of the last wave that is busy) x 1.03 for 512 x 256 tiles,
// whose smaller L2->SM traffic measured ~3 % more work per joule; 512 x 256
// needs at least four waves. Measured on B200: 8192^3, 16384^3 and
// 8192 x 128256 x 4096 pick 512 x 256; 4096^3 and 8192 x {4096, 14336} x 4096
// pick 256 x 256.
static int resolve_mode(int mode, int64_t m, int64_t n, int sm_count) {
    if (mode != B200_MODE_AUTO) return mode;
    const double pairs = std::max(sm_count / 2, 1);
    const int64_t nb = (n + kBN - 1) / kBN;
    const int64_t tiles_2cta = ((m + 255) / 256) * nb;
    if (m < 256 || tiles_2cta < pairs / 2) return B200_MODE_1CTA;
    const int64_t tiles_m512 = ((m + 511) / 512) * nb;
    auto busy = [&](int64_t tiles) {
        const double w = static_cast<double>(tiles) / pairs;
        return w / std::ceil(w);
    };
    if (tiles_m512 >= 4 * pairs && 1.03 * busy(tiles_m512) > busy(tiles_2cta))
        return B200_MODE_2CTA_M512;
    return B200_MODE_2CTA;
}

// Clusters (CTA pairs, or single CTAs in 1-CTA mode) of this kernel that fit
// on the GPU at once: the persistent grid. Pairs use the occupancy query
// (co-scheduling rules can leave fewer pairs than SMs / 2), falling back to
// SMs / 2. Allocates nothing.
static int resident_slots(const void* sym, int cta_group, int smem, int sm_count) {
    if (cta_group == 1) return sm_count;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(sm_count, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    const cudaError_t err = cudaOccupancyMaxActiveClusters(&clusters, sym, &cfg);
    if (err != cudaSuccess || clusters <= 0) {
        cudaGetLastError();
        clusters = sm_count / 2;
    }
    return std::max(clusters, 1);
}

static int plan_create(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d,
                       int64_t ldd, int out_dtype, int mode, void* stream, B200Plan** out_plan,
                       B200PlanInfo* out_info) {
    if (out_plan == nullptr) {
        set_error("out_plan must not be NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    *out_plan = nullptr;
    if (out_info != nullptr) std::memset(out_info, 0, sizeof(*out_info));
    int rc = check_shape(m, n, k, ldd, out_dtype, mode);
    if (rc != B200_OK) return rc;
    const bool empty = (m == 0 || n == 0);
    if (!empty && (a == nullptr && k > 0)) {
        set_error("A must be a device pointer");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (!empty && ((b == nullptr && k > 0) || d == nullptr)) {
        set_error("B and D must be device pointers");
        return B200_ERR_INVALID_ARGUMENT;
    }
    for (const void* ptr : {a, b, static_cast<const void*>(d)}) {
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
            set_error("operand pointer %p is not 16-byte aligned (TMA requirement)", ptr);
            return B200_ERR_UNSUPPORTED;
        }
    }
    if (!empty && k == 0) {
        set_error("K=0 with a non-empty output is not supported (D would be all zeros)");
        return B200_ERR_UNSUPPORTED;
    }

    int device = 0;
    B200_CUDA_TRY(cudaGetDevice(&device));
    DeviceProps props;
    rc = device_props(device, &props);
    if (rc != B200_OK) return rc;
    if (props.cc_major != 10 || props.cc_minor != 0) {
        set_error("device %d has compute capability %d.%d; this library is built for sm_100a (10.0)",
                  device, props.cc_major, props.cc_minor);
        return B200_ERR_UNSUPPORTED;
    }

    B200Plan* plan = new (std::nothrow) B200Plan();
    if (plan == nullptr) {
        set_error("out of host memory");
        return B200_ERR_INTERNAL;
    }
    plan->device = device;
    plan->stream = static_cast<cudaStream_t>(stream);
    plan->out_f32 = out_dtype == B200_OUT_F32;
    const int resolved = resolve_mode(mode, m, n, props.sm_count);
    plan->cta_group = resolved == B200_MODE_1CTA ? 1 : 2;
    plan->sub_m = resolved == B200_MODE_2CTA_M512 ? 2 : 1;
    plan->tile_n = tile_n_for(resolved);
    plan->empty_problem = empty;
    // Programmatic dependent launch: on unless B200_PDL=0.
    plan->pdl = true;
    if (const char* e = std::getenv("B200_PDL")) plan->pdl = e[0] != '0';

    const int tile_m = kRowsPerCta * plan->sub_m * plan->cta_group;
    GemmParams& p = plan->params;
    p.m = static_cast<int>(m);
    p.n = static_cast<int>(n);
    p.k = static_cast<int>(k);
    p.num_m_blocks = static_cast<int>((m + tile_m - 1) / tile_m);
    p.num_n_blocks = static_cast<int>((n + plan->tile_n - 1) / plan->tile_n);
    p.num_k_blocks = static_cast<int>((k + kBK - 1) / kBK);
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    raster_for(p, tile_m, plan->sub_m, &p.group_m, &p.raster_n);
    p.timeout_ns = wait_timeout_ns();

    cudaError_t err = cudaSuccess;
    int slots = 0;
    if (!empty) {
        rc = encode_tmap_2d(&plan->tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, m, k, k,
                            kRowsPerCta * plan->sub_m, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc == B200_OK)
            rc = encode_tmap_2d(&plan->tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, n, k, k,
                                plan->tile_n / plan->cta_group, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc == B200_OK) {
            if (plan->out_f32)
                rc = encode_tmap_2d(&plan->tmD, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d, m, n, ldd, 32,
                                    32, CU_TENSOR_MAP_SWIZZLE_128B);
            else
                rc = encode_tmap_2d(&plan->tmD, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, m, n, ldd, 32,
                                    64, CU_TENSOR_MAP_SWIZZLE_128B);
        }
        if (rc != B200_OK) {
            delete plan;
            return rc;
        }
        plan->smem = smem_bytes_for(plan->cta_group, plan->sub_m, plan->tile_n);
        const void* sym = kernel_sym(plan->cta_group, plan->sub_m, plan->out_f32, false, plan->tile_n);
        err = cudaFuncSetAttribute(sym, cudaFuncAttributeMaxDynamicSharedMemorySize, plan->smem);
        if (err == cudaSuccess && plan->cta_group == 2)
            err = cudaFuncSetAttribute(sym, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
        if (err != cudaSuccess) {
            delete plan;
            return cuda_fail("cudaFuncSetAttribute", err);
        }
        slots = resident_slots(sym, plan->cta_group, plan->smem, props.sm_count);
        const int clusters = std::min(p.num_tiles, slots);
        plan->grid = clusters * plan->cta_group;
        p.kserp_wave = kserp_wave_for(clusters);
        if (plan->tile_n == kBN && stream_k_layout(p, slots, plan->sub_m)) {
            plan->grid = p.sk_groups * p.sk_lanes * plan->cta_group;
            const void* sk_sym = kernel_sym(plan->cta_group, plan->sub_m, plan->out_f32, true, kBN);
            err = cudaFuncSetAttribute(sk_sym, cudaFuncAttributeMaxDynamicSharedMemorySize, plan->smem);
            if (err == cudaSuccess && plan->cta_group == 2)
                err = cudaFuncSetAttribute(sk_sym, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
            if (err != cudaSuccess) {
                delete plan;
                return cuda_fail("cudaFuncSetAttribute", err);
            }
            if (const char* e = std::getenv("B200_TEST_DROP_PARTIAL_FLAGS")) p.sk_test_drop_flags = e[0] == '1';
        }
    }

    // Device words of the plan: [0] status, [2..3] tile scheduler counter; with
    // stream-K also the flags (from byte 256) and the partial buffer (after them).
    const int sk_clusters = plan->grid / plan->cta_group;
    const size_t flags_off = 256;
    const size_t flags_bytes =
        p.sk_iters > 0 ? static_cast<size_t>(sk_clusters) * plan->cta_group * plan->sub_m * kEpiWarps * sizeof(int)
                       : 0;
    const size_t part_off = (flags_off + flags_bytes + 255) / 256 * 256;
    plan->words_bytes = p.sk_iters > 0 ? flags_off + flags_bytes : kPlanWordsBytes;
    const size_t alloc_bytes =
        p.sk_iters > 0 ? part_off + stream_k_partial_bytes(sk_clusters, plan->cta_group, plan->sub_m)
                       : kPlanWordsBytes;
    err = cudaMalloc(&plan->d_status, alloc_bytes);
    if (err != cudaSuccess) {
        delete plan;
        return cuda_fail("cudaMalloc(plan device words)", err);
    }
    err = cudaMemset(plan->d_status, 0, plan->words_bytes);
    if (err != cudaSuccess) {
        cudaFree(plan->d_status);
        delete plan;
        return cuda_fail("cudaMemset(plan device words)", err);
    }
    p.status = plan->d_status;
    p.tile_counter = plan->d_status + 2;
    if (p.sk_iters > 0) {
        uint8_t* base = reinterpret_cast<uint8_t*>(plan->d_status);
        p.sk_flags = reinterpret_cast<int*>(base + flags_off);
        p.sk_partial = reinterpret_cast<float*>(base + part_off);
    }

    B200PlanInfo& info = plan->info;
    info.abi_version = B200_ABI_VERSION;
    info.m = m;
    info.n = n;
    info.k = k;
    info.lda = k;
    info.ldb = k;
    info.ldd = ldd;
    info.out_dtype = out_dtype;
    info.mode = resolved;
    info.cta_group = plan->cta_group;
    info.tile_m = tile_m;
    info.tile_n = plan->tile_n;
    info.tile_k = kBK;
    info.stages = stages_for(plan->cta_group, plan->sub_m, plan->tile_n);
    info.cluster_m = plan->cta_group;
    info.grid_ctas = plan->grid;
    info.threads_per_cta = kThreads;
    info.smem_bytes = plan->smem;
    info.tmem_columns = 2 * plan->tile_n;
    info.num_tiles = empty ? 0 : p.num_tiles;
    info.sm_count = props.sm_count;
    info.device = device;
    info.waves = (slots > 0) ? static_cast<double>(p.num_tiles) / slots : 0.0;
    info.flop_count = 2.0 * static_cast<double>(m) * static_cast<double>(n) * static_cast<double>(k);
    if (out_info != nullptr) *out_info = info;
    *out_plan = plan;
    return B200_OK;
}

static int plan_launch(B200Plan* plan, cudaStream_t stream) {
    if (plan->empty_problem) return B200_OK;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    cfg.gridDim = dim3(plan->grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = plan->smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 0;
    if (plan->cta_group == 2) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = 2;
        attr[cfg.numAttrs].val.clusterDim.y = 1;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        ++cfg.numAttrs;
    }
    if (plan->pdl) {
        attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
        ++cfg.numAttrs;
    }
    cudaError_t err;
#define B200_LAUNCH(G, S, F, K) \
    cudaLaunchKernelEx(&cfg, gemm_tn_sm100_kernel<G, S, F, K>, plan->tmA, plan->tmB, plan->tmD, plan->params, \
                       plan->peer_maps)
    const bool sk = plan->params.sk_iters > 0;
    if (plan->tile_n == 128)
        err = plan->out_f32 ? cudaLaunchKernelEx(&cfg, gemm_tn_sm100_kernel<2, 1, true, false, 128>, plan->tmA,
                                                 plan->tmB, plan->tmD, plan->params, plan->peer_maps)
                            : cudaLaunchKernelEx(&cfg, gemm_tn_sm100_kernel<2, 1, false, false, 128>, plan->tmA,
                                                 plan->tmB, plan->tmD, plan->params, plan->peer_maps);
    else if (plan->cta_group == 1 && sk)
        err = plan->out_f32 ? B200_LAUNCH(1, 1, true, true) : B200_LAUNCH(1, 1, false, true);
    else if (plan->cta_group == 1)
        err = plan->out_f32 ? B200_LAUNCH(1, 1, true, false) : B200_LAUNCH(1, 1, false, false);
    else if (plan->sub_m == 2)
        err = plan->out_f32 ? B200_LAUNCH(2, 2, true, false) : B200_LAUNCH(2, 2, false, false);
    else if (sk)
        err = plan->out_f32 ? B200_LAUNCH(2, 1, true, true) : B200_LAUNCH(2, 1, false, true);
    else
        err = plan->out_f32 ? B200_LAUNCH(2, 1, true, false) : B200_LAUNCH(2, 1, false, false);
#undef B200_LAUNCH
    if (err != cudaSuccess) return cuda_fail("cudaLaunchKernelEx(gemm_tn_sm100_kernel)", err);
    return B200_OK;
}

}  // namespace b200

extern "C" {

int b200_gemm_supported(int64_t m, int64_t n, int64_t k, int64_t ldd, int out_dtype, int mode) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    return b200::check_shape(m, n, k, ldd, out_dtype, mode);
    B200_ABI_GUARD_END
}

int b200_gemm_plan_create(int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                          const void* c, void* d, void* stream, B200Plan** out_plan,
                          B200PlanInfo* out_info) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    (void)c;
    return b200::plan_create(m, n, k, a, b, d, n, B200_OUT_F32, B200_MODE_AUTO, stream, out_plan,
                             out_info);
    B200_ABI_GUARD_END
}

int b200_gemm_plan_create_ex(int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                             void* d, int64_t ldd, int out_dtype, int mode, void* stream,
                             B200Plan** out_plan, B200PlanInfo* out_info) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    return b200::plan_create(m, n, k, a, b, d, ldd, out_dtype, mode, stream, out_plan, out_info);
    B200_ABI_GUARD_END
}

int b200_gemm_plan_execute(B200Plan* plan) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr) {
        b200::set_error("plan is NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    return b200::plan_launch(plan, plan->stream);
    B200_ABI_GUARD_END
}

int b200_gemm_plan_execute_on(B200Plan* plan, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr) {
        b200::set_error("plan is NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    return b200::plan_launch(plan, static_cast<cudaStream_t>(stream));
    B200_ABI_GUARD_END
}

int b200_stream_synchronize(B200Plan* plan) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr) {
        b200::set_error("plan is NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    B200_CUDA_TRY(cudaStreamSynchronize(plan->stream));
    int status = 0;
    B200_CUDA_TRY(cudaMemcpy(&status, plan->d_status, sizeof(int), cudaMemcpyDeviceToHost));
    if (status != 0) {
        // An aborted launch may leave the tile counter mid-walk: re-arm it too.
        B200_CUDA_TRY(cudaMemset(plan->d_status, 0, plan->words_bytes));
        b200::set_error("GEMM kernel reported device status 0x%x (%s)", status,
                        status == B200_DEV_BAD_LAUNCH ? "launch contract violated"
                                                      : "bounded wait timed out");
        return status == B200_DEV_BAD_LAUNCH ? B200_ERR_INTERNAL : B200_ERR_DEVICE_TIMEOUT;
    }
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_gemm_plan_destroy(B200Plan* plan) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (plan == nullptr) return B200_OK;
    cudaError_t err = cudaSuccess;
    if (plan->d_status != nullptr) err = cudaFree(plan->d_status);
    delete plan;
    if (err != cudaSuccess) return b200::cuda_fail("cudaFree(status word)", err);
    return B200_OK;
    B200_ABI_GUARD_END
}

int b200_gemm_plan_set_peers(B200Plan* plan, int npeers, void* const* peer_d) {
    b200::clear_error();
    if (plan == nullptr || npeers < 0 || npeers > b200::kMaxPeers || (npeers > 0 && peer_d == nullptr)) {
        b200::set_error("set_peers: plan must be valid and npeers in [0, %d]", b200::kMaxPeers);
        return B200_ERR_INVALID_ARGUMENT;
    }
    for (int g = 0; g < npeers; ++g) {
        if (peer_d[g] == nullptr || reinterpret_cast<uintptr_t>(peer_d[g]) % 16 != 0) {
            b200::set_error("set_peers: peer pointer %d is NULL or not 16-byte aligned", g);
            return B200_ERR_INVALID_ARGUMENT;
        }
    }
    // Peer chunks go out as TMA bulk stores by default (one per peer per staged
    // chunk); B200_PEER_STORES=st selects per-thread 16-byte stores instead.
    int use_tma = 1;
    if (const char* e = std::getenv("B200_PEER_STORES")) use_tma = !(e[0] == 's' && e[1] == 't');
    const b200::GemmParams& q = plan->params;
    for (int g = 0; g < npeers && use_tma; ++g) {
        const int rc = plan->out_f32
            ? b200::encode_tmap_2d(&plan->peer_maps.map[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, peer_d[g],
                                   q.m, q.n, plan->info.ldd, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B)
            : b200::encode_tmap_2d(&plan->peer_maps.map[g], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, peer_d[g],
                                   q.m, q.n, plan->info.ldd, 32, 64, CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc != B200_OK) return rc;
    }
    plan->params.npeers = npeers;
    plan->params.peer_tma = use_tma;
    plan->params.ldd = plan->info.ldd;
    for (int g = 0; g < b200::kMaxPeers; ++g) plan->params.peer_d[g] = g < npeers ? peer_d[g] : nullptr;
    return B200_OK;
}

int b200_gemm_plan_set_multicast(B200Plan* plan, void* mc_d) {
    b200::clear_error();
    if (plan == nullptr || reinterpret_cast<uintptr_t>(mc_d) % 16 != 0) {
        b200::set_error("set_multicast: plan must be valid and mc_d 16-byte aligned (or NULL)");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (mc_d != nullptr && (plan->out_f32 || (plan->info.ldd * 2) % 16 != 0)) {
        b200::set_error("set_multicast: the multicast gather needs bf16 D with 16-byte rows");
        return B200_ERR_UNSUPPORTED;
    }
    plan->params.mc_d = mc_d;
    plan->params.ldd = plan->info.ldd;
    return B200_OK;
}

int b200_gemm_plan_set_trace(B200Plan* plan, unsigned long long* trace, int64_t slots_per_cta) {
    b200::clear_error();
    if (plan == nullptr) {
        b200::set_error("plan is NULL");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (trace != nullptr && slots_per_cta != b200::kTraceSlots) {
        b200::set_error("the trace buffer must hold %d slots per CTA (grid_ctas x %d uint64)",
                        b200::kTraceSlots, b200::kTraceSlots);
        return B200_ERR_INVALID_ARGUMENT;
    }
    plan->params.trace = trace;
    return B200_OK;
}

int b200_gemm_plan_schedule(const B200Plan* plan) {
    if (plan == nullptr) return -1;
    return plan->params.sk_iters > 0 ? B200_SCHEDULE_STREAM_K : B200_SCHEDULE_DYNAMIC;
}

size_t b200_policy_info_size(void) { return sizeof(B200PolicyInfo); }

int b200_gemm_policy(int64_t m, int64_t n, int64_t k, int mode, int sm_count, B200PolicyInfo* out) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    if (out == nullptr || sm_count < 2) {
        b200::set_error("policy: out must not be NULL and sm_count must be at least 2");
        return B200_ERR_INVALID_ARGUMENT;
    }
    if (m < 1 || n < 1 || k < 1) {
        b200::set_error("policy: (M,N,K)=(%lld,%lld,%lld) must be positive", (long long)m, (long long)n,
                        (long long)k);
        return B200_ERR_INVALID_ARGUMENT;
    }
    const int rc = b200::check_shape(m, n, k, n + (8 - n % 8) % 8, B200_OUT_BF16, mode);
    if (rc != B200_OK) return rc;
    // The same steps as plan creation, with the resident clusters a full GPU holds.
    const int resolved = b200::resolve_mode(mode, m, n, sm_count);
    const int cta_group = resolved == B200_MODE_1CTA ? 1 : 2;
    const int sub_m = resolved == B200_MODE_2CTA_M512 ? 2 : 1;
    const int tile_m = b200::kRowsPerCta * sub_m * cta_group;
    const int tile_n = b200::tile_n_for(resolved);
    b200::GemmParams p{};
    p.m = static_cast<int>(m);
    p.n = static_cast<int>(n);
    p.k = static_cast<int>(k);
    p.num_m_blocks = static_cast<int>((m + tile_m - 1) / tile_m);
    p.num_n_blocks = static_cast<int>((n + tile_n - 1) / tile_n);
    p.num_k_blocks = static_cast<int>((k + b200::kBK - 1) / b200::kBK);
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    b200::raster_for(p, tile_m, sub_m, &p.group_m, &p.raster_n);
    const int slots = cta_group == 1 ? sm_count : sm_count / 2;
    const int clusters = std::min(p.num_tiles, slots);
    int grid = clusters * cta_group;
    const bool sk = tile_n == b200::kBN && b200::stream_k_layout(p, slots, sub_m);
    if (sk) grid = p.sk_groups * p.sk_lanes * cta_group;
    B200PolicyInfo& o = *out;
    std::memset(&o, 0, sizeof(o));
    o.mode = resolved;
    o.tile_m = tile_m;
    o.tile_n = tile_n;
    o.num_m_blocks = p.num_m_blocks;
    o.num_n_blocks = p.num_n_blocks;
    o.num_k_blocks = p.num_k_blocks;
    o.num_tiles = p.num_tiles;
    o.clusters = sk ? p.sk_groups * p.sk_lanes : clusters;
    o.raster_n = p.raster_n;
    o.group = p.group_m;
    o.schedule = sk ? B200_SCHEDULE_STREAM_K : B200_SCHEDULE_DYNAMIC;
    o.sk_groups = p.sk_groups;
    o.sk_lanes = p.sk_lanes;
    o.sk_lane_n = p.sk_lane_n;
    o.sk_rounds = p.sk_rounds;
    o.sk_split_tiles = sk ? p.sk_iters / p.num_k_blocks : 0;
    o.grid_ctas = grid;
    o.kserp_wave = sk ? 0 : b200::kserp_wave_for(clusters);
    o.waves = static_cast<double>(p.num_tiles) / slots;
    return B200_OK;
    B200_ABI_GUARD_END
}

int64_t b200_gemm_plan_launches(const B200Plan* plan) {
    if (plan == nullptr || plan->empty_problem) return 0;
    return 1;
}

int b200_gemm(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d, int64_t ldd,
              int out_dtype, int mode, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    B200Plan* plan = nullptr;
    int rc = b200::plan_create(m, n, k, a, b, d, ldd, out_dtype, mode, stream, &plan, nullptr);
    if (rc != B200_OK) return rc;
    rc = b200::plan_launch(plan, plan->stream);
    // The status word is freed with the plan; synchronise so the launch no
    // longer references it.
    cudaError_t err = cudaStreamSynchronize(plan->stream);
    int status = 0;
    if (err == cudaSuccess) err = cudaMemcpy(&status, plan->d_status, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(plan->d_status);
    delete plan;
    if (rc != B200_OK) return rc;
    if (err != cudaSuccess) return b200::cuda_fail("b200_gemm synchronize", err);
    if (status != 0) {
        b200::set_error("GEMM kernel reported device status 0x%x", status);
        return B200_ERR_DEVICE_TIMEOUT;
    }
    return B200_OK;
    B200_ABI_GUARD_END
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// b200_gemm_noalloc runs the same kernel as b200_gemm (always with the dynamic
// tile schedule: stream-K's partial buffer does not fit), but the device scratch
// the kernel needs -- its status word, where bounded waits record a timeout,
// and the tile scheduler's counter -- lives in the file-scope array below
// instead of a cudaMalloc'd buffer. Callers that cannot allocate device memory use it:
// applications that hand all device memory to their own pool at start-up and
// forbid later driver allocations, and latency-critical paths that must not
// take the implicit device-wide synchronisation cudaMalloc/cudaFree imply.
// ---------------------------------------------------------------------------
namespace b200 {

constexpr size_t kNoAllocScratchBytes = 256;  // stated maximum of the static scratch
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The current CUDA context (driver handle), or nullptr if it cannot be read.
static void* current_context() {
    using CtxGetCurrent = CUresult (*)(CUcontext*);
    static CtxGetCurrent fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &ptr, 12000, cudaEnableDefault, &q) !=
                cudaSuccess || q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return static_cast<CtxGetCurrent>(nullptr);
        }
        return reinterpret_cast<CtxGetCurrent>(ptr);
    }();
    CUcontext ctx = nullptr;
    if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
    return ctx;
}

// Device address of g_noalloc_scratch on `device` (the current device). In
// host code the array's name is only a host-side stand-in, so the address is
// looked up with the device current, checked, and cached per device together
// with the context it belongs to: after a cudaDeviceReset the device gets a new
// context (and the array a new address), so a changed context means a new lookup.
static int noalloc_scratch_address(int device, void** out) {
    constexpr int kMaxDevices = 64;
    static void* addr[kMaxDevices] = {};
    static void* ctx_of[kMaxDevices] = {};
    static std::mutex mu;
    if (device < 0 || device >= kMaxDevices) {
        set_error("device index %d out of range", device);
        return B200_ERR_INVALID_ARGUMENT;
    }
    std::lock_guard<std::mutex> lock(mu);
    void* ctx = current_context();
    if (addr[device] == nullptr || ctx == nullptr || ctx != ctx_of[device]) {
        void* p = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) return cuda_fail("cudaGetSymbolAddress(g_noalloc_scratch)", err);
        addr[device] = p;
        ctx_of[device] = ctx;
    }
    *out = addr[device];
    return B200_OK;
}

// Fills `plan` like plan_create, without any allocation; the status word is
// `status` (a pointer into the static scratch).
static int noalloc_prepare(B200Plan* plan, int64_t m, int64_t n, int64_t k, const void* a,
                           const void* b, void* d, int64_t ldd, int out_dtype, int mode,
                           int device, const DeviceProps& props, int* status) {
    plan->device = device;
    plan->out_f32 = out_dtype == B200_OUT_F32;
    const int resolved = resolve_mode(mode, m, n, props.sm_count);
    plan->cta_group = resolved == B200_MODE_1CTA ? 1 : 2;
    plan->sub_m = resolved == B200_MODE_2CTA_M512 ? 2 : 1;
    plan->tile_n = tile_n_for(resolved);
    plan->empty_problem = (m == 0 || n == 0);
    plan->d_status = status;
    const int tile_m = kRowsPerCta * plan->sub_m * plan->cta_group;
    GemmParams& p = plan->params;
    p.m = static_cast<int>(m);
    p.n = static_cast<int>(n);
    p.k = static_cast<int>(k);
    p.num_m_blocks = static_cast<int>((m + tile_m - 1) / tile_m);
    p.num_n_blocks = static_cast<int>((n + plan->tile_n - 1) / plan->tile_n);
    p.num_k_blocks = static_cast<int>((k + kBK - 1) / kBK);
    p.num_tiles = p.num_m_blocks * p.num_n_blocks;
    raster_for(p, tile_m, plan->sub_m, &p.group_m, &p.raster_n);
    p.timeout_ns = wait_timeout_ns();
    p.status = status;
    p.tile_counter = status + 2;
    if (plan->empty_problem) return B200_OK;
    int rc = encode_tmap_2d(&plan->tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, m, k, k,
                            kRowsPerCta * plan->sub_m, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == B200_OK)
        rc = encode_tmap_2d(&plan->tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, n, k, k,
                            plan->tile_n / plan->cta_group, kBK, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == B200_OK)
        rc = plan->out_f32
                 ? encode_tmap_2d(&plan->tmD, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d, m, n, ldd, 32, 32,
                                  CU_TENSOR_MAP_SWIZZLE_128B)
                 : encode_tmap_2d(&plan->tmD, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, m, n, ldd, 32, 64,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != B200_OK) return rc;
    plan->smem = smem_bytes_for(plan->cta_group, plan->sub_m, plan->tile_n);
    const void* sym = kernel_sym(plan->cta_group, plan->sub_m, plan->out_f32, false, plan->tile_n);
    B200_CUDA_TRY(cudaFuncSetAttribute(sym, cudaFuncAttributeMaxDynamicSharedMemorySize, plan->smem));
    if (plan->cta_group == 2)
        B200_CUDA_TRY(cudaFuncSetAttribute(sym, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
    // The same persistent grid as plan_create's dynamic schedule.
    const int slots = resident_slots(sym, plan->cta_group, plan->smem, props.sm_count);
    plan->grid = std::min(p.num_tiles, slots) * plan->cta_group;
    p.kserp_wave = kserp_wave_for(plan->grid / plan->cta_group);
    return B200_OK;
}

}  // namespace b200

extern "C" int b200_gemm_noalloc(int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                                 void* d, int64_t ldd, int out_dtype, int mode, void* stream) {
    B200_ABI_GUARD_BEGIN
    b200::clear_error();
    int rc = b200::check_shape(m, n, k, ldd, out_dtype, mode);
    if (rc != B200_OK) return rc;
    const bool empty = (m == 0 || n == 0);
    if (!empty && (a == nullptr || b == nullptr || d == nullptr)) {
        b200::set_error("A, B and D must be device pointers");
        return B200_ERR_INVALID_ARGUMENT;
    }
    for (const void* ptr : {a, b, static_cast<const void*>(d)}) {
        if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
            b200::set_error("operand pointer %p is not 16-byte aligned (TMA requirement)", ptr);
            return B200_ERR_UNSUPPORTED;
        }
    }
    if (!empty && k == 0) {
        b200::set_error("K=0 with a non-empty output is not supported (D would be all zeros)");
        return B200_ERR_UNSUPPORTED;
    }
    // This launch needs 16 bytes of scratch (status word and the tile
    // scheduler's counter); refuse anything that would not fit the static array.
    constexpr size_t kNeeded = b200::kPlanWordsBytes;
    if (kNeeded > b200::kNoAllocScratchBytes) {
        b200::set_error("b200_gemm_noalloc needs %zu bytes of scratch, the static array holds %zu",
                        kNeeded, b200::kNoAllocScratchBytes);
        return B200_ERR_UNSUPPORTED;
    }
    int device = 0;
    B200_CUDA_TRY(cudaGetDevice(&device));
    b200::DeviceProps props;
    rc = b200::device_props(device, &props);
    if (rc != B200_OK) return rc;
    if (props.cc_major != 10 || props.cc_minor != 0) {
        b200::set_error("device %d has compute capability %d.%d; this library is built for sm_100a (10.0)",
                        device, props.cc_major, props.cc_minor);
        return B200_ERR_UNSUPPORTED;
    }
    void* scratch = nullptr;
    rc = b200::noalloc_scratch_address(device, &scratch);
    if (rc != B200_OK) return rc;
    int* status = static_cast<int*>(scratch);

    B200Plan plan;  // on the stack: no host or device allocation
    plan.stream = static_cast<cudaStream_t>(stream);
    rc = b200::noalloc_prepare(&plan, m, n, k, a, b, d, ldd, out_dtype, mode, device, props, status);
    if (rc != B200_OK) return rc;
    if (plan.empty_problem) return B200_OK;

    // The array keeps the previous call's contents: status word and tile
    // counter must start at zero.
    B200_CUDA_TRY(cudaMemsetAsync(status, 0, b200::kPlanWordsBytes, plan.stream));
    rc = b200::plan_launch(&plan, plan.stream);
    if (rc != B200_OK) return rc;
    int host_status = 0;
    B200_CUDA_TRY(cudaMemcpyAsync(&host_status, status, sizeof(int), cudaMemcpyDeviceToHost, plan.stream));
    B200_CUDA_TRY(cudaStreamSynchronize(plan.stream));
    if (host_status != 0) {
        b200::set_error("GEMM kernel reported device status 0x%x", host_status);
        return host_status == B200_DEV_BAD_LAUNCH ? B200_ERR_INTERNAL : B200_ERR_DEVICE_TIMEOUT;
    }
    return B200_OK;
    B200_ABI_GUARD_END
}
