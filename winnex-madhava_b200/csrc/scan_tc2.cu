// Tensor-core u8 L2 scan on SM pairs (tcgen05 cta_group::2), sm_100a.
//
// Same contract as the other filter kernels (scan_simt.cu): pairs with
// (key, id) <= (thr_key[q], thr_id[q]), key = |q|^2 + |v|^2 - 2 q.v, are
// appended to q's candidate list as {key, row}; dense levels write row r at
// slot r.
//
// A cluster of two CTAs on two SMs shares every MMA: M = 256 queries (128 in
// each CTA's tensor memory), N = 128 corpus rows (each CTA stages 64 of them),
// K = 128 bytes (four kind::i8 steps of 32).  Each CTA keeps two query tiles
// resident, so one pair holds 512 queries and every corpus tile fetched from
// L2 feeds 512 x 128 dot products -- a quarter of the L2 traffic per product
// of one 128-query CTA -- while each SM reads only 6 KB of shared-memory
// operands per 64-cycle MMA step.
//
// Per CTA (576 threads, one CTA per SM, persistent):
//   warps 0-15 epilogue: warp w reads TMEM lanes 32*(w%4).. of query tile
//              (w/4)%2, columns [64*(w/8), +64): both 32-column chunks are
//              copied to registers and the accumulator released (a remote
//              arrive on the even CTA's barrier) before the Cauchy-Schwarz
//              chunk filter runs.  The filter needs only the first (smallest)
//              norm of each chunk, read from L2 one tile ahead; the rare
//              chunks that pass are expanded by a bit-mask loop;
//   warp 16    TMA producer: its own two query tiles per work unit and its
//              half of each corpus tile;
//   warp 17    TMEM allocator (both CTAs) and, in the even CTA only, the
//              single-thread MMA issuer.
// Barriers with cross-CTA producers live in the even CTA (FULL, A_FULL,
// ACC_EMPTY); the MMA commits arrive on both CTAs' EMPTY / ACC_FULL / A_EMPTY
// through tcgen05.commit's cluster multicast.  No TMA load uses multicast.
//
// Every wait is bounded (see tc_ptx.cuh); both CTAs leave through a cluster
// barrier so neither exits while the other's copies or MMAs can still touch
// its shared or tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "internal.h"
#include "tc_ptx.cuh"

namespace mdh {

namespace {

using namespace tc;

constexpr int QT = 2;                 // query tiles per CTA
constexpr int BM = 128;               // query rows per CTA per query tile (TMEM lanes)
constexpr int PAIR_M = 2 * BM;        // MMA M of the pair
constexpr int QGROUP = QT * PAIR_M;   // queries per work unit (512)
constexpr int BN = 128;               // corpus rows per pair tile (MMA N)
constexpr int BN_HALF = BN / 2;       // corpus rows each CTA stages
constexpr int BK = 128;               // bytes per row (K)
constexpr int STAGES = 12;            // corpus ring depth
constexpr int ACC_STAGES = 2;
constexpr int TMEM_COLS = 512;        // ACC_STAGES * QT * BN
static_assert(ACC_STAGES * QT * BN == TMEM_COLS, "tensor memory split");
constexpr int EPI_WARPS = 16;
constexpr int COLS_PER_WARP = 64;     // two 32-column chunks
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int PRODUCER_WARP = EPI_WARPS;
constexpr int MMA_WARP = EPI_WARPS + 1;
constexpr int NUM_THREADS = 32 * (EPI_WARPS + 2);
constexpr int BUFN = 4;
constexpr uint32_t A_TILE_BYTES = BM * BK;
constexpr uint32_t A_BYTES = QT * A_TILE_BYTES;
constexpr uint32_t B_BYTES = BN_HALF * BK;
constexpr uint32_t IDESC = idesc_u8(PAIR_M, BN);

constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_B = OFF_A + A_BYTES;
constexpr uint32_t OFF_BUF = OFF_B + STAGES * B_BYTES;
constexpr uint32_t OFF_BAR = OFF_BUF + BUFN * EPI_THREADS * 8;
constexpr uint32_t BAR_FULL = 0, BAR_EMPTY = STAGES, BAR_ACC_FULL = 2 * STAGES,
                   BAR_ACC_EMPTY = 2 * STAGES + ACC_STAGES,
                   BAR_A_FULL = 2 * STAGES + 2 * ACC_STAGES, BAR_A_EMPTY = BAR_A_FULL + 1, BAR_DRAIN = BAR_A_FULL + 2,
                   NUM_BARS = BAR_A_FULL + 3;
constexpr uint32_t OFF_TMEM_SLOT = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t OFF_ABORT = OFF_TMEM_SLOT + 4;
constexpr uint32_t SMEM_USED = OFF_ABORT + 4;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(OFF_B % 1024 == 0 && B_BYTES % 1024 == 0 && A_TILE_BYTES % 1024 == 0, "swizzle alignment");

struct Sched2 {
    int n_groups;     // query groups of QGROUP
    int n_tiles;      // corpus tiles of BN rows
    int n_chunks;     // corpus chunks per query group
    long long n_units;
};

__device__ __forceinline__ void unit_coords(const Sched2& s, long long u, int& g, int& t0, int& t1) {
    const int c = (int)(u / s.n_groups);
    g = (int)(u - (long long)c * s.n_groups);
    t0 = (int)((long long)c * s.n_tiles / s.n_chunks);
    t1 = (int)((long long)(c + 1) * s.n_tiles / s.n_chunks);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_filter_tc2_u8_l2(const __grid_constant__ CUtensorMap tmap_rows, const __grid_constant__ CUtensorMap tmap_q,
                       const int32_t* __restrict__ norms, const int32_t* __restrict__ ids, int32_t n_rows,
                       const int32_t* __restrict__ qn, int nq, const uint32_t* __restrict__ thr_key,
                       const int32_t* __restrict__ thr_id, uint32_t* __restrict__ counts, uint2* __restrict__ cand,
                       int cap, int dense, Sched2 sched, int32_t* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + OFF_BAR;
    volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + OFF_ABORT);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM_SLOT);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const long long pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bars + 8 * (BAR_FULL + s), 1);
            mbar_init(bars + 8 * (BAR_EMPTY + s), 1);
        }
        for (int s = 0; s < ACC_STAGES; s++) {
            mbar_init(bars + 8 * (BAR_ACC_FULL + s), 1);
            mbar_init(bars + 8 * (BAR_ACC_EMPTY + s), 2 * EPI_WARPS);
        }
        mbar_init(bars + 8 * BAR_A_FULL, 1);
        mbar_init(bars + 8 * BAR_A_EMPTY, 1);
        mbar_init(bars + 8 * BAR_DRAIN, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == MMA_WARP) tmem_alloc<2>(smem_u32(tmem_slot), TMEM_COLS);
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers initialized and tensor memory allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == PRODUCER_WARP) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_rows) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
            const uint32_t leader_bars = map_to_cta(bars, 0);  // the even CTA's barriers, cluster address
            int stage = 0;
            uint32_t phase = 0, a_iter = 0;
            bool ok = true;
            for (long long u = pair; u < sched.n_units && ok; u += n_pairs) {
                int g, t0, t1;
                unit_coords(sched, u, g, t0, t1);
                ok = mbar_wait<true>(bars + 8 * BAR_A_EMPTY, (a_iter & 1) ^ 1, abort_flag, status);
                if (!ok) break;
                if (rank == 0) mbar_expect_tx(bars + 8 * BAR_A_FULL, 2 * A_BYTES);
                for (int qt = 0; qt < QT; qt++)
                    tma_load_2d_pair(sbase + OFF_A + qt * A_TILE_BYTES, &tmap_q, leader_bars + 8 * BAR_A_FULL, 0,
                                     g * QGROUP + qt * PAIR_M + (int)rank * BM);
                a_iter++;
                for (int t = t0; t < t1; t++) {
                    ok = mbar_wait<true>(bars + 8 * (BAR_EMPTY + stage), phase ^ 1, abort_flag, status);
                    if (!ok) break;
                    if (rank == 0) mbar_expect_tx(bars + 8 * (BAR_FULL + stage), 2 * B_BYTES);
                    tma_load_2d_pair(sbase + OFF_B + stage * B_BYTES, &tmap_rows, leader_bars + 8 * (BAR_FULL + stage), 0,
                                     t * BN + (int)rank * BN_HALF);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Tensor copies complete on the even CTA's barriers, which the
            // cluster barrier at exit keeps alive until both CTAs are done.
        }
    } else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        if (lane == 0 && rank == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0, a_iter = 0;
            bool ok = true, issued = false;
            for (long long u = pair; u < sched.n_units && ok; u += n_pairs) {
                int g, t0, t1;
                unit_coords(sched, u, g, t0, t1);
                ok = mbar_wait<true>(bars + 8 * BAR_A_FULL, a_iter & 1, abort_flag, status);
                if (!ok) break;
                a_iter++;
                tc_fence_after();
                for (int t = t0; t < t1; t++) {
                    ok = mbar_wait<true>(bars + 8 * (BAR_ACC_EMPTY + acc), acc_phase ^ 1, abort_flag, status);
                    if (!ok) break;
                    ok = mbar_wait<true>(bars + 8 * (BAR_FULL + stage), phase, abort_flag, status);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t bdesc = sw128_desc(sbase + OFF_B + stage * B_BYTES);
#pragma unroll
                    for (int qt = 0; qt < QT; qt++) {
                        const uint64_t adesc = sw128_desc(sbase + OFF_A + qt * A_TILE_BYTES);
                        const uint32_t d = tmem_base + (uint32_t)(acc * QT * BN + qt * BN);
#pragma unroll
                        for (int kk = 0; kk < BK / 32; kk++)
                            umma_i8<2>(d, adesc + (uint64_t)((kk * 32) >> 4), bdesc + (uint64_t)((kk * 32) >> 4),
                                       IDESC, kk > 0 ? 1u : 0u);
                    }
                    issued = true;
                    umma_commit_pair(bars + 8 * (BAR_EMPTY + stage), 0x3);
                    umma_commit_pair(bars + 8 * (BAR_ACC_FULL + acc), 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (++acc == ACC_STAGES) {
                        acc = 0;
                        acc_phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit_pair(bars + 8 * BAR_A_EMPTY, 0x3);
            }
            if (!ok && issued) {
                umma_commit_pair(bars + 8 * BAR_DRAIN, 0x1);
                mbar_drain_wait<false>(bars + 8 * BAR_DRAIN, 0);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 0-15, both CTAs)
        const int quarter = warp & 3, qt = (warp >> 2) & 1, part = warp >> 3;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t leader_acc_empty = map_to_cta(bars + 8 * BAR_ACC_EMPTY, 0);
        CandBuf<EPI_THREADS, BUFN> buf;
        buf.base = reinterpret_cast<uint2*>(smem + OFF_BUF) + threadIdx.x;
        buf.n = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (long long u = pair; u < sched.n_units && ok; u += n_pairs) {
            int g, t0, t1;
            unit_coords(sched, u, g, t0, t1);
            const int qi = g * QGROUP + qt * PAIR_M + (int)rank * BM + quarter * 32 + lane;
            const bool qvalid = qi < nq;
            uint32_t tkey = 0;
            int32_t tid = 0, qnv = 0;
            if (qvalid) {
                tkey = thr_key[qi];
                tid = thr_id[qi];
                qnv = qn[qi];
            }
            // A row passes when qn + n - 2v <= tkey; with n >= n_min of its
            // 32-row chunk, 2v >= n_min + bias (bias = qn - tkey) is necessary.
            // Keys of real rows are below 2^30: an infinite threshold maps to a
            // bias that always passes, an invalid query to one that never does.
            int32_t bias;
            if (!qvalid)
                bias = 1 << 29;  // need stays below 2^31 even for pad rows (norm 2^30)
            else if (tkey >= (1u << 30))
                bias = -(1 << 30);
            else
                bias = qnv - (int32_t)tkey;
            // n_min of this warp's two chunks, one tile ahead of their use.
            const int32_t* nrm = norms + part * COLS_PER_WARP;
            int32_t nx0 = 0, nx1 = 0;
            if (t0 < t1) {
                nx0 = __ldg(nrm + (int64_t)t0 * BN);
                nx1 = __ldg(nrm + (int64_t)t0 * BN + 32);
            }
            for (int t = t0; t < t1; t++) {
                const int32_t need0 = nx0 + bias, need1 = nx1 + bias;
                if (t + 1 < t1) {
                    nx0 = __ldg(nrm + (int64_t)(t + 1) * BN);
                    nx1 = __ldg(nrm + (int64_t)(t + 1) * BN + 32);
                }
                ok = mbar_wait_inl<true>(bars + 8 * (BAR_ACC_FULL + acc), acc_phase, abort_flag, status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tcol = tmem_base + lane_base + (uint32_t)(acc * QT * BN + qt * BN + part * COLS_PER_WARP);
                uint32_t v[2][32];
                __syncwarp();
                tmem_ld32_issue(tcol, v[0]);
                tmem_ld32_issue(tcol + 32, v[1]);
                tmem_ld_wait(v[0]);  // waits for both loads
                tmem_ld_wait(v[1]);
                // Both chunks are in registers: release the accumulator to the MMA.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(leader_acc_empty + 8 * acc);
                if (++acc == ACC_STAGES) {
                    acc = 0;
                    acc_phase ^= 1;
                }
                const int32_t m0 = max32(v[0]), m1 = max32(v[1]);
                if (2 * m0 < need0 && 2 * m1 < need1) continue;
                const int32_t row0 = t * BN + part * COLS_PER_WARP;  // rows < 2^31 (ids are int32)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    uint32_t mask = pass_mask32(v[c], c ? need1 : need0);
                    while (mask) {
                        const int j = __ffs(mask) - 1;
                        mask &= mask - 1;
                        const int32_t r = row0 + c * 32 + j;
                        if (r >= n_rows) break;  // pad rows trail the level
                        const uint32_t key = (uint32_t)(qnv + __ldg(norms + r) - 2 * (int32_t)pick32(v[c], j));
                        if (dense)
                            cand[(size_t)qi * cap + r] = make_uint2(key, (uint32_t)r);
                        else if (key < tkey || (key == tkey && __ldg(ids + r) <= tid))
                            buf.push(key, (uint32_t)r, counts, cand, cap, qi);
                    }
                }
            }
            if (qvalid) buf.flush(counts, cand, cap, qi);
        }
    }

    tc_fence_before();
    cluster_sync();  // no copy or MMA of either CTA is still in flight past this point
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc<2>(tmem_base, TMEM_COLS);
    }
}

}  // namespace

bool tc2_supported(const mdh_index* ix, const Level& lv) {
    return ix && !ix->is_f32 && ix->dpad == BK && ix->dim <= BK && lv.rows && lv.norms && lv.n_pad % BN == 0 &&
           lv.n_pad < (int64_t(1) << 31);
}

void make_tmap_rows_pair(Level& lv, int dpad) {
    if (dpad != BK || !lv.rows) return;
    encode_u8_rows_tmap(&lv.tmap_rows_pair, lv.rows, lv.n_pad, dpad, BN_HALF);
    lv.has_tmap_pair = true;
}

void launch_filter_tc2_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                             const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap,
                             int dense, int32_t* status, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    MDH_REQUIRE(dpad == BK && lv.has_tmap_pair, MDH_ERR_INTERNAL, "pair scan needs 128-byte rows and a TMA map");
    MDH_REQUIRE(!dense || cap >= lv.n, MDH_ERR_INTERNAL, "dense scan needs cap >= rows");
    MDH_REQUIRE((reinterpret_cast<uintptr_t>(lv.norms) & 15) == 0, MDH_ERR_INTERNAL, "norms must be 16-byte aligned");
    CUtensorMap tq;
    encode_u8_rows_tmap(&tq, q, nq, dpad, BM);
    // A function attribute belongs to the current device: set it on every launch.
    MDH_CUDA(cudaFuncSetAttribute(k_filter_tc2_u8_l2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int max_pairs_dev[64] = {0};  // per device; a racing double query is harmless
    int max_pairs = (dev >= 0 && dev < 64) ? max_pairs_dev[dev] : 0;
    if (!max_pairs) {
        cfg.gridDim = dim3(2 * device_sm_count(dev) / 2, 1, 1);
        int clusters = 0;
        MDH_CUDA(cudaOccupancyMaxActiveClusters(&clusters, k_filter_tc2_u8_l2, &cfg));
        MDH_REQUIRE(clusters > 0, MDH_ERR_CUDA, "no SM pair can host the pair scan kernel");
        max_pairs = clusters;
        if (dev >= 0 && dev < 64) max_pairs_dev[dev] = clusters;
    }
    Sched2 s;
    s.n_groups = (nq + QGROUP - 1) / QGROUP;
    s.n_tiles = (int)(lv.n_pad / BN);
    int pairs = max_pairs;
    s.n_chunks = choose_scan_chunks(s.n_groups, s.n_tiles, pairs, 64);
    s.n_units = (long long)s.n_groups * s.n_chunks;
    if (s.n_units < pairs) pairs = (int)s.n_units;
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    MDH_CUDA(cudaLaunchKernelEx(&cfg, k_filter_tc2_u8_l2, lv.tmap_rows_pair, tq, (const int32_t*)lv.norms,
                                (const int32_t*)lv.ids, (int32_t)lv.n, qn, nq, thr_key, thr_id, counts, cand, cap,
                                dense, s, status));
}

}  // namespace mdh
