// Streaming CUDA-core scan for small batches (1..63 queries), sm_100a.
//
// Same contract as the other filter kernels (scan_simt.cu).  A small batch
// does 2 * QG int operations per corpus byte, so the scan is bound by
// reading the u8 corpus from HBM; this kernel keeps that stream full.  One
// CTA per SM (17 warps):
//   warp 16  producer: 1-D bulk copies (cp.async.bulk) of 256-row tiles
//            (32 KB of contiguous 128-byte rows, then their 1 KB of norms)
//            into a 6-stage shared-memory ring, completion counted on
//            per-stage mbarriers -- ~198 KB in flight per SM, enough to cover
//            HBM latency at full bandwidth;
//   warps 0-15 consumers: warp w takes rows [16w, 16w + 16) of each tile,
//            four rows per step: 8 lanes read one row (16 bytes each, a warp
//            reads 512 contiguous bytes of shared memory, conflict-free),
//            __dp4a forms the partial dot products with QG queries held in
//            registers and an 8-lane reduce-scatter (scan_common.cuh) leaves
//            one lane per (row, query) with the full dot product.
// Tiles are dealt round-robin to the CTAs of a query group (blockIdx.y).
//
// Every mbarrier wait is bounded; on expiry the kernel records kDevTimeout
// in *status, raises a shared abort flag, drains its issued copies with
// bounded waits and returns.
#include "internal.h"
#include "scan_common.cuh"
#include "tc_ptx.cuh"

namespace mdh {

namespace {

using namespace tc;

constexpr int kRowBytes = 128;     // dpad handled by this kernel
constexpr int kStreamRows = 256;
constexpr uint32_t kStreamTileBytes = kStreamRows * kRowBytes;
constexpr uint32_t kNormBytes = kStreamRows * 4;
constexpr uint32_t kStageBytes = kStreamTileBytes + kNormBytes;  // rows, then their norms
constexpr int kStages = 6;
constexpr int kConsumerWarps = 16;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr uint32_t kOffBar = kStages * kStageBytes;
constexpr uint32_t kBarFull = 0, kBarEmpty = kStages, kNumBars = 2 * kStages;
constexpr uint32_t kOffAbort = kOffBar + kNumBars * 8;
constexpr uint32_t kSmemBytes = kOffAbort + 16 + 128;  // + alignment slack
static_assert(kStreamRows == kConsumerWarps * 16, "16 rows per consumer warp");
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

template <int QG, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    k_scan_stream_u8(const uint8_t* __restrict__ rows, const int32_t* __restrict__ norms,
                     const int32_t* __restrict__ ids, int64_t n, int64_t n_pad, const uint8_t* __restrict__ q,
                     const int32_t* __restrict__ qn, int nq, const uint32_t* __restrict__ thr_key,
                     const int32_t* __restrict__ thr_id, uint32_t* __restrict__ counts, uint2* __restrict__ cand,
                     int cap, int dense, int32_t* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + kOffBar;
    volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + kOffAbort);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t n_tiles = n_pad / kStreamRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(bars + 8 * (kBarFull + s), 1);
            mbar_init(bars + 8 * (kBarEmpty + s), kConsumerWarps);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_parity = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
                ok = mbar_wait<false>(bars + 8 * (kBarEmpty + stage), phase ^ 1, abort_flag, status);
                if (!ok) break;
                mbar_expect_tx(bars + 8 * (kBarFull + stage), kStageBytes);
                bulk_load(sbase + stage * kStageBytes, rows + t * kStreamTileBytes, kStreamTileBytes,
                          bars + 8 * (kBarFull + stage));
                bulk_load(sbase + stage * kStageBytes + kStreamTileBytes, norms + t * kStreamRows, kNormBytes,
                          bars + 8 * (kBarFull + stage));
                issued_mask |= 1u << stage;
                last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            if (!ok)
                for (int s = 0; s < kStages; s++)
                    if (issued_mask & (1u << s))
                        mbar_drain_wait<false>(bars + 8 * (kBarFull + s), (last_parity >> s) & 1);
        }
    } else {
        // ------------------------------------------------------------ consumers
        const int l8 = lane & 7, grp = lane >> 3;
        const int q0 = blockIdx.y * QG;
        uint4 qv[QG];
#pragma unroll
        for (int j = 0; j < QG; j++)
            qv[j] = q0 + j < nq ? *reinterpret_cast<const uint4*>(q + (size_t)(q0 + j) * kRowBytes + l8 * 16)
                                : make_uint4(0, 0, 0, 0);
        int qsel;
        bool active;
        {
            uint32_t dummy[QG];
#pragma unroll
            for (int j = 0; j < QG; j++) dummy[j] = 0;
            reduce_scatter8<QG>(dummy, l8, qsel, active);
        }
        const int qi = q0 + qsel;
        const bool qvalid = active && qi < nq;
        uint32_t tkey = 0;
        int32_t tid = 0, my_qn = 0;
        if (qvalid) {
            tkey = thr_key[qi];
            tid = thr_id[qi];
            my_qn = qn[qi];
        }
        const float qn_f = (float)my_qn;
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int64_t t = blockIdx.x; t < n_tiles && ok; t += gridDim.x) {
            ok = mbar_wait_inl<false>(bars + 8 * (kBarFull + stage), phase, abort_flag, status);
            if (!ok) break;
            const uint8_t* tile = smem + stage * kStageBytes;
            const int32_t* tnorm = reinterpret_cast<const int32_t*>(tile + kStreamTileBytes);
#pragma unroll
            for (int step = 0; step < 4; step++) {
                const int lr = warp * 16 + step * 4 + grp;  // row within the tile
                const uint4 x = *reinterpret_cast<const uint4*>(tile + lr * kRowBytes + l8 * 16);
                uint32_t acc[QG];
#pragma unroll
                for (int j = 0; j < QG; j++) {
                    uint32_t a = __dp4a(x.x, qv[j].x, 0u);
                    a = __dp4a(x.y, qv[j].y, a);
                    a = __dp4a(x.z, qv[j].z, a);
                    acc[j] = __dp4a(x.w, qv[j].w, a);
                }
                int qs2;
                bool act2;
                reduce_scatter8<QG>(acc, l8, qs2, act2);
                const int64_t r = t * kStreamRows + lr;
                if (qvalid && r < n) {
                    const uint32_t dot = acc[0];
                    const int32_t nv = tnorm[lr];
                    uint32_t key;
                    if (MODE == 0) {
                        key = (uint32_t)(my_qn + nv - 2 * (int32_t)dot);
                    } else {
                        const float denom = __fsqrt_rn(__fmul_rn((float)nv, qn_f));
                        const float sc = denom > 1e-10f ? __fdiv_rn((float)dot, denom) : 0.0f;
                        key = ordered_key_desc(sc);
                    }
                    offer_candidate(counts, cand, cap, dense, qi, key, r, ids, tkey, tid);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bars + 8 * (kBarEmpty + stage));
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1;
            }
        }
    }
    __syncthreads();  // no copy into this CTA's shared memory is in flight past here
}

template <int QG, int MODE>
void launch_stream_t(const Level& lv, const uint8_t* q, const int32_t* qn, int nq, const uint32_t* tk,
                     const int32_t* ti, uint32_t* counts, uint2* cand, int cap, int dense, int32_t* status,
                     cudaStream_t st) {
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    const int groups = (nq + QG - 1) / QG;
    MDH_REQUIRE(groups <= 65535, MDH_ERR_INTERNAL, "too many query groups for one launch");
    const int64_t n_tiles = lv.n_pad / kStreamRows;
    int64_t gx = sms / groups;
    if (gx < 1) gx = 1;
    if (gx > n_tiles) gx = n_tiles;
    // A function attribute belongs to the current device: set it on every launch.
    MDH_CUDA(cudaFuncSetAttribute(k_scan_stream_u8<QG, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemBytes));
    dim3 grid((unsigned)gx, (unsigned)groups);
    k_scan_stream_u8<QG, MODE><<<grid, kThreads, kSmemBytes, st>>>(lv.rows, lv.norms, lv.ids, lv.n, lv.n_pad, q, qn,
                                                                    nq, tk, ti, counts, cand, cap, dense, status);
    MDH_CUDA(cudaGetLastError());
}

template <int MODE>
void launch_stream_dispatch(const Level& lv, const uint8_t* q, const int32_t* qn, int nq, const uint32_t* tk,
                            const int32_t* ti, uint32_t* counts, uint2* cand, int cap, int dense, int32_t* status,
                            cudaStream_t st) {
    if (nq >= 8)
        launch_stream_t<8, MODE>(lv, q, qn, nq, tk, ti, counts, cand, cap, dense, status, st);
    else if (nq >= 4)
        launch_stream_t<4, MODE>(lv, q, qn, nq, tk, ti, counts, cand, cap, dense, status, st);
    else if (nq >= 2)
        launch_stream_t<2, MODE>(lv, q, qn, nq, tk, ti, counts, cand, cap, dense, status, st);
    else
        launch_stream_t<1, MODE>(lv, q, qn, nq, tk, ti, counts, cand, cap, dense, status, st);
}

}  // namespace

bool stream_supported(int dpad, const Level& lv) {
    return dpad == kRowBytes && lv.rows && lv.norms && lv.n_pad % kStreamRows == 0 &&
           (reinterpret_cast<uintptr_t>(lv.rows) & 15) == 0 && (reinterpret_cast<uintptr_t>(lv.norms) & 15) == 0;
}

void launch_scan_stream_u8(const Level& lv, int dpad, int mode, const uint8_t* q, const int32_t* qn, int nq,
                           const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap,
                           int dense, int32_t* status, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    MDH_REQUIRE(stream_supported(dpad, lv), MDH_ERR_INTERNAL, "streaming scan needs 128-byte rows");
    MDH_REQUIRE(!dense || cap >= lv.n, MDH_ERR_INTERNAL, "dense scan needs cap >= rows");
    if (mode == 0)
        launch_stream_dispatch<0>(lv, q, qn, nq, thr_key, thr_id, counts, cand, cap, dense, status, st);
    else
        launch_stream_dispatch<1>(lv, q, qn, nq, thr_key, thr_id, counts, cand, cap, dense, status, st);
}

}  // namespace mdh
