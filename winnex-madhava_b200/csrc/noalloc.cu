// mdh_search_u8_device_noalloc: the device-resident exact L2 search of
// mdh_search_u8_device (capi.cu) for small batches, run entirely in a fixed
// scratch area that is a file-scope __device__ array.  It allocates nothing:
// no cudaMalloc / cudaFree, no stream-ordered or library allocation, no
// growth of the index's workspace.  Callers that must not allocate are
// serving loops that run next to a caching allocator holding most of HBM
// (PyTorch's, for one), where a cudaMalloc can fail or fragment the pool, and
// latency-bound loops, where cudaFree synchronises the whole device and
// stalls every other stream.
//
// Limits (rejected with MDH_ERR_UNSUPPORTED): L2 metric, u8 index on one
// device, dim <= 256, nq <= 256, k <= 256.  Candidate lists hold up to 4,096
// entries per query and level; a list that overflows is rerun with a
// strictly tighter threshold, as on the main path, so results stay exact.
//
// Set-up: the first call on a device resolves the scratch array's device
// address with cudaGetSymbolAddress (with that device current) and caches
// it; make that first call before any stream capture.  Everything read from
// the scratch is written by the same call before use: the counts and status
// words are cleared by cudaMemsetAsync and the thresholds filled by a kernel,
// so no part of the scratch has to start at zero.
//
// Every call on a device shares that device's scratch, so overlapping calls
// would race; calls are serialised by a process-wide lock and each returns
// after its work on `stream` has completed.
#include <chrono>
#include <mutex>

#include "internal.h"

namespace mdh {

namespace {

constexpr int kNaMaxQueries = 256;
constexpr int kNaMaxK = 256;
constexpr int kNaMaxDpad = 256;
constexpr int kNaCap = 4096;      // candidate list entries per query and level
constexpr int kNaMaxSteps = 16;

// Scratch map (offsets in bytes, each 256-byte aligned).
constexpr size_t al(size_t x) { return (x + 255) & ~size_t(255); }
constexpr size_t kOffQ = 0;                                                   // u8 [nq][dpad]
constexpr size_t kOffQn = kOffQ + al((size_t)kNaMaxQueries * kNaMaxDpad);    // s32 [nq]
constexpr size_t kOffThrKey = kOffQn + al(kNaMaxQueries * 4);                // u32 [nq]
constexpr size_t kOffThrId = kOffThrKey + al(kNaMaxQueries * 4);             // s32 [nq]
constexpr size_t kOffCounts = kOffThrId + al(kNaMaxQueries * 4);             // u32 [nq]
constexpr size_t kOffFlags = kOffCounts + al(kNaMaxQueries * 4);             // s32 [nq]
constexpr size_t kOffStatus = kOffFlags + al(kNaMaxQueries * 4);             // s32 [2]
constexpr size_t kOffOutKey = kOffStatus + 256;                               // u32 [nq][k]
constexpr size_t kOffOutId = kOffOutKey + al((size_t)kNaMaxQueries * kNaMaxK * 4);  // s32 [nq][k]
constexpr size_t kOffCand = kOffOutId + al((size_t)kNaMaxQueries * kNaMaxK * 4);    // uint2 [nq][cap]
constexpr size_t kNaUsed = kOffCand + (size_t)kNaMaxQueries * kNaCap * 8;
constexpr size_t kNaScratchBytes = size_t(9) << 20;  // 9 MiB per device
static_assert(kNaUsed <= kNaScratchBytes, "scratch map exceeds the scratch array");

__device__ __align__(256) uint8_t g_na_scratch[kNaScratchBytes];

std::mutex g_na_mu;
uint8_t* g_na_ptr[64] = {nullptr};  // device address of g_na_scratch per device ordinal
int32_t g_na_host_status[2];        // pageable: read back with a synchronous copy

uint8_t* scratch_for_device(int dev) {
    MDH_REQUIRE(dev >= 0 && dev < 64, MDH_ERR_UNSUPPORTED, "device ordinal above 63");
    if (!g_na_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_na_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            throw Error(MDH_ERR_CUDA, std::string("cudaGetSymbolAddress of the static scratch failed: ") +
                                          cudaGetErrorString(e));
        }
        g_na_ptr[dev] = static_cast<uint8_t*>(p);
    }
    return g_na_ptr[dev];
}

int pow2_at_least(int64_t x) {
    int64_t p = 1;
    while (p < x) p <<= 1;
    return (int)p;
}

struct NaStep {
    int level;
    int cap;
    bool first;  // infinite threshold
};

// Level plan of the main path with every candidate list capped at kNaCap.
int plan(const Shard& sh, int k, NaStep* steps) {
    const int L = (int)sh.levels.size();
    MDH_REQUIRE(L >= 1 && L <= kNaMaxSteps, MDH_ERR_INTERNAL, "unexpected level count");
    const int cap_floor = pow2_at_least(k + 1 > 64 ? k + 1 : 64);
    auto clampcap = [&](int cap) { return cap < cap_floor ? cap_floor : (cap > kNaCap ? kNaCap : cap); };
    int i0 = L - 1;
    for (int i = 0; i < L; i++)
        if (sh.levels[i].n >= k) {
            i0 = i;
            break;
        }
    int ns = 0;
    steps[ns++] = {i0, clampcap(pow2_at_least(sh.levels[i0].n > k ? sh.levels[i0].n : k)), true};
    const double rmax = 2048.0 / (double)k > 4.0 ? 2048.0 / (double)k : 4.0;
    int cur = i0;
    while (cur != L - 1) {
        int nxt = cur + 1;
        for (int j = cur + 1; j < L; j++)
            if ((double)sh.levels[j].n <= (double)sh.levels[cur].n * rmax) nxt = j;
        steps[ns++] = {nxt, kNaCap, false};
        cur = nxt;
    }
    return ns;
}

// rerun: an overflow rerun (the tensor scan then keeps only rows at or under
// the threshold, so each rerun tightens it).
void filter(mdh_index* ix, const Level& lv, const uint8_t* q, const int32_t* qn, int nq, const uint32_t* tk,
            const int32_t* ti, uint32_t* counts, uint2* cand, int cap, bool dense, int32_t* status, cudaStream_t st,
            int* path, bool rerun = false) {
    const int d = dense ? 1 : 0;
    if (lv.has_tmap && tc_supported(ix, lv)) {
        launch_filter_tc_u8_l2(lv, ix->dpad, q, qn, nq, tk, ti, counts, cand, cap, d, status, nullptr, rerun ? 1 : 0,
                               st);
        *path = 1;
    } else if (stream_supported(ix->dpad, lv)) {
        launch_scan_stream_u8(lv, ix->dpad, 0, q, qn, nq, tk, ti, counts, cand, cap, d, status, st);
        *path = 0;
    } else {
        launch_filter_simt_u8_l2(lv, ix->dpad, q, qn, nq, tk, ti, counts, cand, cap, d, st);
        *path = 0;
    }
    if (dense) launch_fill_u32(counts, nq, (uint32_t)lv.n, st);
}

void read_status(const int32_t* dev_status, cudaStream_t st) {
    MDH_CUDA(cudaMemcpyAsync(g_na_host_status, dev_status, sizeof(g_na_host_status), cudaMemcpyDeviceToHost, st));
    MDH_CUDA(cudaStreamSynchronize(st));
    if (g_na_host_status[0] != kDevOk)
        throw Error(g_na_host_status[0] == kDevTimeout ? MDH_ERR_TIMEOUT : MDH_ERR_INTERNAL,
                    "tensor-core scan reported device status " + std::to_string(g_na_host_status[0]));
}

void search_noalloc(mdh_index* ix, const uint8_t* dev_q, int nq, int k, int32_t* dev_ids, int32_t* dev_dist,
                    cudaStream_t st, mdh_stats* stats) {
    auto t0 = std::chrono::high_resolution_clock::now();
    MDH_REQUIRE(ix && !ix->is_f32, MDH_ERR_INVALID_ARG, "u8 queries need a u8 index");
    MDH_REQUIRE(ix->metric == MDH_METRIC_L2, MDH_ERR_UNSUPPORTED, "the no-alloc search supports the L2 metric only");
    MDH_REQUIRE(ix->shards.size() == 1, MDH_ERR_UNSUPPORTED, "the no-alloc search needs a single-device index");
    MDH_REQUIRE(ix->dpad <= kNaMaxDpad, MDH_ERR_UNSUPPORTED, "the no-alloc search supports dim <= 256");
    MDH_REQUIRE(nq >= 0 && k >= 0, MDH_ERR_INVALID_ARG, "nq and k must be >= 0");
    MDH_REQUIRE(nq <= kNaMaxQueries, MDH_ERR_UNSUPPORTED,
                "the no-alloc search takes at most 256 queries per call (got " + std::to_string(nq) + ")");
    MDH_REQUIRE(k <= kNaMaxK, MDH_ERR_UNSUPPORTED,
                "the no-alloc search supports k <= 256 (got " + std::to_string(k) + ")");
    MDH_REQUIRE(nq == 0 || k == 0 || (dev_q && dev_ids), MDH_ERR_INVALID_ARG, "null device buffer");
    std::lock_guard<std::mutex> glock(g_na_mu);
    std::lock_guard<std::mutex> lock(ix->mu);
    Shard& sh = ix->shards[0];
    MDH_CUDA(cudaSetDevice(sh.device));
    uint8_t* base = scratch_for_device(sh.device);
    mdh_stats s{};
    const int kk = (int)(k < ix->n ? k : ix->n);
    if (nq > 0 && k > 0) {
        uint8_t* q = base + kOffQ;
        int32_t* qn = reinterpret_cast<int32_t*>(base + kOffQn);
        uint32_t* thr_key = reinterpret_cast<uint32_t*>(base + kOffThrKey);
        int32_t* thr_id = reinterpret_cast<int32_t*>(base + kOffThrId);
        uint32_t* counts = reinterpret_cast<uint32_t*>(base + kOffCounts);
        int32_t* flags = reinterpret_cast<int32_t*>(base + kOffFlags);
        int32_t* status = reinterpret_cast<int32_t*>(base + kOffStatus);
        uint32_t* out_key = reinterpret_cast<uint32_t*>(base + kOffOutKey);
        int32_t* out_id = reinterpret_cast<int32_t*>(base + kOffOutId);
        uint2* cand = reinterpret_cast<uint2*>(base + kOffCand);
        const int dpad = ix->dpad, dim = ix->dim;
        if (kk > 0) {
            if (dpad != dim) MDH_CUDA(cudaMemsetAsync(q, 0, (size_t)nq * dpad, st));
            MDH_CUDA(cudaMemcpy2DAsync(q, dpad, dev_q, dim, dim, nq, cudaMemcpyDeviceToDevice, st));
            launch_query_norms_u8(q, nq, dpad, qn, st);
            s.kernel_launches++;
            NaStep steps[kNaMaxSteps];
            const int ns = plan(sh, kk, steps);
            MDH_CUDA(cudaMemsetAsync(status, 0, 2 * sizeof(int32_t), st));
            int path = 0;
            for (int si = 0; si < ns; si++) {
                const NaStep& p = steps[si];
                const Level& lv = sh.levels[p.level];
                if (p.first) {
                    launch_fill_threshold(thr_key, thr_id, nq, kKeyInf, kIdInf, st);
                    s.kernel_launches++;
                }
                MDH_CUDA(cudaMemsetAsync(counts, 0, (size_t)nq * 4, st));
                const bool dense = p.first && p.cap >= lv.n;
                filter(ix, lv, q, qn, nq, thr_key, thr_id, counts, cand, p.cap, dense, status, st, &path);
                s.kernel_launches += dense ? 2 : 1;
                s.pairs_scored += lv.n * (int64_t)nq;
                const bool final_ = si + 1 == ns;
                launch_select(counts, cand, p.cap, lv.ids, nq, kk, final_ ? 1 : 0, thr_key, thr_id, out_key, out_id,
                              flags, status + 1, nullptr, nullptr, st);
                s.kernel_launches++;
                if (final_) {
                    s.full_scan_pairs = lv.n * (int64_t)nq;
                    s.tensor_core_path = path;
                }
            }
            s.levels = ns;
            read_status(status, st);
            // Overflowed lists: every query rescans the full level; queries that
            // did not overflow keep their threshold and get the same result.
            const NaStep& last = steps[ns - 1];
            const Level& lv = sh.levels[last.level];
            int rounds = 0;
            while (g_na_host_status[1] > 0) {
                MDH_REQUIRE(++rounds < 64, MDH_ERR_INTERNAL, "candidate overflow did not converge");
                MDH_CUDA(cudaMemsetAsync(counts, 0, (size_t)nq * 4, st));
                MDH_CUDA(cudaMemsetAsync(status + 1, 0, sizeof(int32_t), st));
                filter(ix, lv, q, qn, nq, thr_key, thr_id, counts, cand, last.cap, false, status, st, &path, true);
                launch_select(counts, cand, last.cap, lv.ids, nq, kk, 1, thr_key, thr_id, out_key, out_id, flags,
                              status + 1, nullptr, nullptr, st);
                s.kernel_launches += 2;
                s.pairs_scored += lv.n * (int64_t)nq;
                read_status(status, st);
            }
        }
        if (kk == k) {
            MDH_CUDA(cudaMemcpyAsync(dev_ids, out_id, (size_t)nq * k * 4, cudaMemcpyDeviceToDevice, st));
            if (dev_dist)
                MDH_CUDA(cudaMemcpyAsync(dev_dist, out_key, (size_t)nq * k * 4, cudaMemcpyDeviceToDevice, st));
        } else {
            MDH_CUDA(cudaMemsetAsync(dev_ids, 0xFF, (size_t)nq * k * 4, st));
            if (dev_dist) MDH_CUDA(cudaMemsetAsync(dev_dist, 0xFF, (size_t)nq * k * 4, st));
            if (kk > 0) {
                MDH_CUDA(cudaMemcpy2DAsync(dev_ids, (size_t)k * 4, out_id, (size_t)kk * 4, (size_t)kk * 4, nq,
                                           cudaMemcpyDeviceToDevice, st));
                if (dev_dist)
                    MDH_CUDA(cudaMemcpy2DAsync(dev_dist, (size_t)k * 4, out_key, (size_t)kk * 4, (size_t)kk * 4, nq,
                                               cudaMemcpyDeviceToDevice, st));
            }
        }
        MDH_CUDA(cudaStreamSynchronize(st));
    }
    s.latency_ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0).count();
    if (stats) *stats = s;
}

}  // namespace

}  // namespace mdh

extern "C" mdh_status mdh_search_u8_device_noalloc(mdh_index* index, const uint8_t* dev_queries, int32_t nq,
                                                   int32_t k, int32_t* dev_ids, int32_t* dev_dist, void* stream,
                                                   mdh_stats* stats) {
    struct Args {
        mdh_index* index;
        const uint8_t* q;
        int32_t nq, k;
        int32_t *ids, *dist;
        void* stream;
        mdh_stats* stats;
    } a{index, dev_queries, nq, k, dev_ids, dev_dist, stream, stats};
    return mdh::run_guarded(
        [](void* p) {
            const Args& x = *static_cast<const Args*>(p);
            mdh::search_noalloc(x.index, x.q, x.nq, x.k, x.ids, x.dist, static_cast<cudaStream_t>(x.stream), x.stats);
        },
        &a);
}
