// C ABI and search orchestration.
//
// Search algorithm (exact, every path):
//   A shard holds nested norm-sorted row sets L_0 c L_1 c ... c L_last (random
//   samples of the shard, then the shard itself).
//   1. Scan L_0 with an infinite threshold; each query keeps the k-th
//      smallest (key, id) as its threshold T_0 (k rows of L_0 lie at or
//      below it, so at least k rows of every larger level do too).
//   2. For each following level, keep only the pairs with (key, id) <= T
//      as candidates and select their k-th smallest as the next threshold.
//   3. On the full shard the candidates' sorted first k entries are the
//      exact top-k: every pair left out ranks after T, which ranks after k
//      rows of the shard.
//   If a query's candidate list overflows on the full shard, the k-th
//   smallest stored entry is a strictly smaller valid threshold (ids make
//   keys unique); that query reruns with it until its list fits.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"

namespace mdh {

void ensure_speed_rows_u8(mdh_index* ix, Shard& sh);

namespace {

thread_local std::string g_last_error;
int g_scan_path = 0;  // 0 auto, 1 CUDA cores only, 2 tensor cores when possible
int g_cap_limit = 0;  // 0 = default candidate capacities
int g_verify = 0;     // queries per search re-checked by an exact unpruned scan (0 = off)
std::atomic<int> g_fault{kFaultNone};

constexpr int kCapMax = 16384;          // largest candidate list the selection kernel sorts
// Level-plan cost model (row-scan units per query): a level's fixed cost and
// one candidate's cost (epilogue expansion, re-key, selection), measured on
// B200 (u8 L2, 10K queries; the bf16 cosine scan and its rescore scale alike).
constexpr double kPlanLevelCost = 2.0e5;
constexpr double kPlanCandidateCost = 4.5e3;
int g_threshold_sharing = 1;  // ranks whose sample results set the full level's threshold
constexpr size_t kCandBudget = size_t(2) << 30;  // bytes of candidate lists per query chunk

template <class F>
mdh_status guard(F&& f) {
    try {
        f();
        g_last_error.clear();
        return MDH_OK;
    } catch (const Error& e) {
        g_last_error = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        g_last_error = "host allocation failed";
        return MDH_ERR_OOM;
    } catch (const std::exception& e) {
        g_last_error = e.what();
        return MDH_ERR_INTERNAL;
    }
}

int next_pow2(int64_t x) {
    int64_t p = 1;
    while (p < x) p <<= 1;
    return (int)p;
}

// What the queries of one call are and which arithmetic ranks them.
struct QueryPlan {
    bool integer = false;   // u8 integer path
    int kind = -1;          // ScoreKind for the float path
    bool asc = true;        // key ascends with the returned value (L2) or descends (scores)
    bool int_dist = false;  // returned value is an integer distance
};

// Levels scanned for one search: indices into shard.levels plus their
// candidate capacity.
struct LevelStep {
    int level;
    int cap;
    bool dense;  // infinite threshold (first level)
};

// sizes: the level row counts, ascending (the last is the whole shard).
std::vector<LevelStep> plan_levels(const std::vector<int64_t>& sizes, int64_t shard_rows, int k) {
    const int L = (int)sizes.size();
    std::vector<LevelStep> steps;
    // First level: the smallest with at least k rows whose dense candidate
    // list fits the selector.
    int i0 = -1;
    for (int i = 0; i < L; i++) {
        if (sizes[i] >= k || i == L - 1) {
            if (sizes[i] <= kCapMax) i0 = i;
            break;
        }
    }
    if (i0 < 0)
        throw Error(MDH_ERR_UNSUPPORTED, "k = " + std::to_string(k) +
                                             " is larger than this build's exact selector supports for a corpus of " +
                                             std::to_string(shard_rows) + " rows");
    // A list must hold more than k entries: the rerun threshold (k-th
    // smallest stored key) is then strictly below the largest stored key,
    // so every overflow round makes progress even when distances tie.
    const int cap_floor = next_pow2(std::max(k + 1, 64));
    auto limit = [&](int cap) { return g_cap_limit > 0 ? std::max(cap_floor, std::min(cap, g_cap_limit)) : cap; };
    steps.push_back({i0, limit(next_pow2(std::max<int64_t>(sizes[i0], k))), true});
    // The levels after the first: the cheapest chain to the full shard under
    // a cost model in row-scan units per query (measured on B200 with 10K
    // queries): each level scanned costs its rows plus a fixed kPlanLevelCost
    // (launches, selection), and each candidate it keeps costs
    // kPlanCandidateCost -- about k * (its rows / the previous level's rows)
    // candidates per query pass the previous level's threshold.  When the
    // ranks of a row split share their sample results (g_threshold_sharing =
    // G), the full level's threshold is the union's, G times tighter.  A step
    // is allowed only while its expected list fits the selector.
    const double rmax = std::max(4.0, (double)(kCapMax - 256) / (3.0 * k));
    std::vector<double> cost((size_t)L, 1e300);
    std::vector<int> prev((size_t)L, -1);
    cost[(size_t)i0] = (double)sizes[i0] + kPlanLevelCost;
    for (int j = i0 + 1; j < L; j++) {
        const double share = j == L - 1 ? (double)std::max(1, g_threshold_sharing) : 1.0;
        for (int i = i0; i < j; i++) {
            const double ratio = (double)sizes[j] / (double)std::max<int64_t>(sizes[i], 1);
            if (ratio > rmax && i != j - 1) continue;
            const double c = cost[(size_t)i] + (double)sizes[j] + kPlanLevelCost + kPlanCandidateCost * k * ratio / share;
            if (c < cost[(size_t)j]) {
                cost[(size_t)j] = c;
                prev[(size_t)j] = i;
            }
        }
    }
    std::vector<int> chain;
    for (int j = L - 1; j != i0; j = prev[(size_t)j]) chain.push_back(j);
    int cur = i0;
    for (auto it = chain.rbegin(); it != chain.rend(); ++it) {
        const int nxt = *it;
        const double ratio = (double)sizes[nxt] / (double)std::max<int64_t>(sizes[cur], 1);
        int cap = next_pow2((int64_t)(3.0 * k * ratio) + 256);
        cap = std::max(4096, std::min(kCapMax, cap));
        if (nxt == L - 1 && sizes[nxt] <= kCapMax) cap = std::max(cap, next_pow2(std::max<int64_t>(sizes[nxt], k)));
        cap = std::min(cap, kCapMax);
        steps.push_back({nxt, limit(cap), false});
        cur = nxt;
    }
    return steps;
}

std::vector<LevelStep> plan_levels(const Shard& sh, int k) {
    std::vector<int64_t> sizes;
    for (const Level& lv : sh.levels) sizes.push_back(lv.n);
    return plan_levels(sizes, sh.n, k);
}

void grow(void** p, size_t* have, size_t need) {
    if (need <= *have) return;
    if (take_fault(kFaultOom))
        throw Error(MDH_ERR_OOM, "device scratch allocation failed: injected out-of-memory (mdh_set_fault)");
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    size_t want = need + need / 4;
    cudaError_t e = cudaMalloc(p, want);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        throw Error(MDH_ERR_OOM, std::string("device scratch allocation failed: ") + cudaGetErrorString(e));
    }
    *have = want;
}
template <class T>
void growT(T** p, size_t* have, size_t need_bytes) {
    void* v = *p;
    grow(&v, have, need_bytes);
    *p = static_cast<T*>(v);
}

void ensure_status(Workspace& w) {
    if (!w.status) {
        MDH_CUDA(cudaMalloc(&w.status, kStatusWords * sizeof(int32_t)));
        MDH_CUDA(cudaHostAlloc(&w.h_status, kStatusWords * sizeof(int32_t), cudaHostAllocDefault));
    }
    for (cudaEvent_t* e : {&w.ev0, &w.ev1, &w.ev_start, &w.ev_sel, &w.ev_rescore, &w.ev_prep})
        if (!*e) MDH_CUDA(cudaEventCreate(e));
}

float event_ms(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.0f;
    MDH_CUDA(cudaEventElapsedTime(&ms, a, b));
    return ms;
}

// Run one level's filter for `nq` queries already staged in the workspace.
// dense: every row of the level is a candidate (first level, infinite
// thresholds, cap >= rows); the kernels write row r at slot r and the
// counts are set to the row count here.
// Returns the scan used: 1 CUDA cores, 2 tensor cores (one SM per tile),
// 3 tensor cores (SM pairs).  Auto takes the single-SM tensor scan for every
// batch size: on B200 it was measured faster than the SM-pair scan at every
// batch and faster than the streaming CUDA-core scan even for one query (at
// one query both read the corpus from HBM; TMA keeps more of it in flight).

// Error bound of the bf16 cosine pass for unit vectors: bf16 products carry a
// relative error of at most 2u + u^2 (u = 2^-8) and |sum q_j v_j| <= 1; the
// fp32 sums of the tensor core and of the reference add at most dim * 2^-24
// each.
float bf16_cos_eps(int dim) {
    return (float)((1.0 / 128 + 1.0 / 65536) * 1.001 + 2.0 * dim / 16777216.0 + 1e-6);
}

int run_filter(mdh_index* ix, Shard& sh, const Level& lv, const QueryPlan& qp, const uint8_t* q_u8,
               const int32_t* qn, const float* q_f32, int nq, const uint32_t* tk, const int32_t* ti, int cap,
               bool dense, const uint16_t* q_bf16 = nullptr, bool exact_only = false, int k_dense = 0) {
    Workspace& w = sh.ws;
    unsigned long long* bstats = reinterpret_cast<unsigned long long*>(w.status + kStatusBlockStats);
    const int d = dense ? 1 : 0;
    int used = 1;
    if (!qp.integer && qp.kind == kScoreSpeedCos && q_bf16 && !exact_only && g_scan_path != 1 &&
        lv.has_tmap_bf16 && tc_bf16_supported(ix, lv)) {
        // bf16 tensor pass keeps every pair within the error bound of the
        // threshold; the kept pairs are then rescored with the reference's
        // fp32 arithmetic.
        launch_filter_tc_bf16_cos(lv, ix->dim, q_bf16, nq, tk, w.counts, w.cand, cap, d, bf16_cos_eps(ix->dim),
                                  w.status, sh.stream);
        if (dense) launch_fill_u32(w.counts, nq, (uint32_t)lv.n, sh.stream);
        if (dense && k_dense > 0 && lv.n > k_dense) {
            // A dense list holds every row: rescore only the band of bf16
            // scores that can hold the exact top k.  The k-th bf16 key goes
            // through the thresholds, which are then reset, so the level's
            // exact selection starts from infinity again.
            launch_select(w.counts, w.cand, cap, lv.ids, nq, k_dense, 0, w.thr_key, w.thr_id, w.out_key, w.out_id,
                          w.flags, w.status + 1, nullptr, nullptr, sh.stream);
            launch_compact_bf16_band(w.counts, w.cand, cap, w.thr_key, 2.0f * bf16_cos_eps(ix->dim), nq, sh.stream);
            launch_fill_threshold(w.thr_key, w.thr_id, nq, kKeyInf, kIdInf, sh.stream);
        }
        MDH_CUDA(cudaEventRecord(w.ev_rescore, sh.stream));
        launch_rescore_speed_cos(w.counts, w.cand, cap, lv.rows_f32, ix->dim, q_f32, nq, sh.stream);
        return 4;
    }
    if (qp.integer) {
        if (ix->metric == MDH_METRIC_L2) {
            const bool can1 = lv.has_tmap && tc_supported(ix, lv);
            const bool can2 = lv.has_tmap_pair && tc2_supported(ix, lv);
            if (g_scan_path == 3 && can2)
                used = 3;
            else if (g_scan_path == 2 && can1)
                used = 2;
            else if (g_scan_path == 0)
                used = can1 ? 2 : 1;
            if (used == 3)
                launch_filter_tc2_u8_l2(lv, ix->dpad, q_u8, qn, nq, tk, ti, w.counts, w.cand, cap, d, w.status,
                                        sh.stream);
            else if (used == 2)
                launch_filter_tc_u8_l2(lv, ix->dpad, q_u8, qn, nq, tk, ti, w.counts, w.cand, cap, d, w.status, bstats,
                                       exact_only ? 1 : 0, sh.stream);
            else if (stream_supported(ix->dpad, lv))
                launch_scan_stream_u8(lv, ix->dpad, 0, q_u8, qn, nq, tk, ti, w.counts, w.cand, cap, d, w.status,
                                      sh.stream);
            else
                launch_filter_simt_u8_l2(lv, ix->dpad, q_u8, qn, nq, tk, ti, w.counts, w.cand, cap, d, sh.stream);
        } else if (stream_supported(ix->dpad, lv)) {
            launch_scan_stream_u8(lv, ix->dpad, 1, q_u8, qn, nq, tk, ti, w.counts, w.cand, cap, d, w.status, sh.stream);
        } else {
            launch_filter_simt_u8_cos(lv, ix->dpad, q_u8, qn, nq, tk, ti, w.counts, w.cand, cap, d, sh.stream);
        }
    } else {
        launch_filter_f32(lv, ix->dim, ix->dpad, qp.kind, q_f32, nq, tk, ti, w.counts, w.cand, cap, d, sh.stream);
    }
    if (dense) launch_fill_u32(w.counts, nq, (uint32_t)lv.n, sh.stream);
    return used;
}

struct ShardResult {
    int64_t pairs = 0;
    int levels = 0;
    bool tc = false;
    double scan_ms = 0.0;     // event time of the full-shard filter
    int64_t scan_pairs = 0;
    int scan_path = 0;        // run_filter's path for the full shard
    int64_t launches = 0;     // kernels launched
    int64_t candidates = 0;   // entries of the final candidate lists
    int64_t violations = 0;   // verification: rows misplaced relative to the results
    int64_t verified = 0;     // verification: queries re-checked
    double sample_ms = 0.0;   // event time of the sample levels (scans and selections)
    double select_ms = 0.0;   // final selection, overflow reruns included
    double rescore_ms = 0.0;  // exact rescore inside the full-level scan (bf16 path)
    int64_t tc_pairs = 0;     // pairs scanned by the 1-SM tensor scan (its block bound applies)
    int64_t blocks_tested = 0;
    int64_t blocks_passed = 0;
    int64_t pruned = 0;       // tc_pairs whose distance the block bound made unnecessary
};

// Phases of a search that ranks share their sample results in between
// (cooperative thresholds, mdh_search_u8_device_sample / _bounded).
enum SearchPhase { kPhaseAll = 0, kPhaseSample = 1, kPhaseBounded = 2 };

// Exact top-k for nq staged queries on one shard.  Results: ws.out_key /
// ws.out_id ([nq][k], device).  host_q_u8 / host_q_f32 hold the staged
// queries on the host for overflow reruns.
// phase kPhaseSample: the plan without its full level; the results are the
// exact top-k of the largest sample scanned (the whole shard when it has no
// sample).  kPhaseBounded: the full level alone, with each query's threshold
// the k-th entry of thr_lists ([nq][k] (distance, id) on the device, id -1 =
// empty); the results are the exact top-k among the rows at or under it.
ShardResult search_shard(mdh_index* ix, Shard& sh, const QueryPlan& qp, int nq, int k, const uint8_t* host_q_u8,
                         const float* host_q_f32, size_t f32_stride_floats, int phase = kPhaseAll,
                         const int32_t* thr_dist = nullptr, const int32_t* thr_ids = nullptr) {
    MDH_CUDA(cudaSetDevice(sh.device));
    Workspace& w = sh.ws;
    cudaStream_t st = sh.stream;
    ShardResult res;
    std::vector<LevelStep> steps = plan_levels(sh, k);
    if (phase == kPhaseSample && steps.size() > 1) steps.pop_back();
    if (phase == kPhaseBounded) steps = {LevelStep{(int)sh.levels.size() - 1, steps.back().cap, false}};
    int capmax = 0;
    for (auto& s : steps) capmax = std::max(capmax, s.cap);
    growT(&w.thr_key, &w.thr_key_bytes, (size_t)nq * 4);
    growT(&w.thr_id, &w.thr_id_bytes, (size_t)nq * 4);
    growT(&w.counts, &w.counts_bytes, (size_t)nq * 4);
    growT(&w.cand, &w.cand_bytes, (size_t)nq * capmax * sizeof(uint2));
    growT(&w.out_key, &w.out_key_bytes, (size_t)nq * k * 4);
    growT(&w.out_id, &w.out_id_bytes, (size_t)nq * k * 4);
    growT(&w.flags, &w.flags_bytes, (size_t)nq * 4);
    ensure_status(w);
    MDH_CUDA(cudaMemsetAsync(w.status, 0, 12 * sizeof(int32_t), st));
    unsigned long long* n_cand = reinterpret_cast<unsigned long long*>(w.status + 2);
    unsigned long long* n_viol = reinterpret_cast<unsigned long long*>(w.status + 4);
    // Tests of the 1-SM tensor scan's schedule form: every (query, 64-row block).
    auto count_tc = [&](const Level& lv, int used, int m) {
        if (used != 2) return;
        res.tc_pairs += lv.n * (int64_t)m;
        res.blocks_tested += lv.n_pad / 64 * (int64_t)m;
    };

    res.levels = (int)steps.size();
    MDH_CUDA(cudaEventRecord(w.ev_start, st));
    if (phase == kPhaseBounded) {
        launch_thresholds_from_lists(reinterpret_cast<const uint32_t*>(thr_dist), thr_ids, nq, k, w.thr_key, w.thr_id,
                                     st);
        res.launches++;
    }
    for (size_t si = 0; si < steps.size(); si++) {
        const LevelStep& s = steps[si];
        const Level& lv = sh.levels[s.level];
        if (s.dense) {
            launch_fill_threshold(w.thr_key, w.thr_id, nq, kKeyInf, kIdInf, st);
            res.launches++;
        }
        MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)nq * 4, st));
        const bool last_level = si + 1 == steps.size();
        if (last_level) {
            MDH_CUDA(cudaEventRecord(w.ev0, st));
        }
        const bool dense = s.dense && s.cap >= lv.n;
        const int used = run_filter(ix, sh, lv, qp, w.q_u8, w.qn, w.q_f32, nq, w.thr_key, w.thr_id, s.cap, dense,
                                    w.q_bf16, false, dense ? k : 0);
        count_tc(lv, used, nq);
        res.launches += (dense ? 2 : 1) + (used == 4 ? 1 : 0) + (used == 4 && dense && lv.n > k ? 3 : 0);
        if (last_level) {
            MDH_CUDA(cudaEventRecord(w.ev1, st));
            res.scan_pairs = lv.n * (int64_t)nq;
            res.scan_path = used;
        }
        res.pairs += lv.n * (int64_t)nq;
        if (used >= 2) res.tc = true;
        const bool final_ = si + 1 == steps.size();
        if (final_) MDH_CUDA(cudaMemsetAsync(w.status + 1, 0, sizeof(int32_t), st));
        launch_select(w.counts, w.cand, s.cap, lv.ids, nq, k, final_ ? 1 : 0, w.thr_key, w.thr_id, w.out_key,
                      w.out_id, w.flags, w.status + 1, nullptr, final_ ? n_cand : nullptr, st);
        res.launches++;
        if (final_) MDH_CUDA(cudaEventRecord(w.ev_sel, st));
    }
    // Status words: [0] device error of the tensor-core scan, [1] overflowed queries.
    MDH_CUDA(cudaMemcpyAsync(w.h_status, w.status, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    MDH_CUDA(cudaStreamSynchronize(st));
    if (w.h_status[0] != kDevOk)
        throw Error(w.h_status[0] == kDevTimeout ? MDH_ERR_TIMEOUT : MDH_ERR_INTERNAL,
                    "tensor-core scan reported device status " + std::to_string(w.h_status[0]));
    res.scan_ms = event_ms(w.ev0, w.ev1);
    res.sample_ms = steps.size() > 1 ? event_ms(w.ev_start, w.ev0) : 0.0;
    res.select_ms = event_ms(w.ev1, w.ev_sel);
    if (qp.kind == kScoreSpeedCos && res.scan_path == 4) res.rescore_ms = event_ms(w.ev_rescore, w.ev1);
    int flagged = w.h_status[1];
    const auto t_rerun = std::chrono::high_resolution_clock::now();
    const LevelStep last = steps.back();
    const Level& lv = sh.levels[last.level];
    int rounds = 0;
    while (flagged > 0) {
        MDH_REQUIRE(++rounds < 64, MDH_ERR_INTERNAL, "candidate overflow did not converge");
        std::vector<int32_t> hflags((size_t)nq), hti((size_t)nq);
        std::vector<uint32_t> htk((size_t)nq);
        MDH_CUDA(cudaMemcpyAsync(hflags.data(), w.flags, (size_t)nq * 4, cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaMemcpyAsync(htk.data(), w.thr_key, (size_t)nq * 4, cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaMemcpyAsync(hti.data(), w.thr_id, (size_t)nq * 4, cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaStreamSynchronize(st));
        std::vector<int32_t> list;
        for (int i = 0; i < nq; i++)
            if (hflags[(size_t)i]) list.push_back(i);
        const int m = (int)list.size();
        // Compact the flagged queries into the tail scratch (qlist + staged copies).
        std::vector<uint32_t> ctk((size_t)m);
        std::vector<int32_t> cti((size_t)m);
        for (int i = 0; i < m; i++) {
            ctk[(size_t)i] = htk[(size_t)list[(size_t)i]];
            cti[(size_t)i] = hti[(size_t)list[(size_t)i]];
        }
        growT(&w.qlist, &w.qlist_bytes, (size_t)m * 4 * 3);
        int32_t* d_list = w.qlist;
        uint32_t* d_tk = reinterpret_cast<uint32_t*>(w.qlist + m);
        int32_t* d_ti = w.qlist + 2 * m;
        MDH_CUDA(cudaMemcpyAsync(d_list, list.data(), (size_t)m * 4, cudaMemcpyHostToDevice, st));
        MDH_CUDA(cudaMemcpyAsync(d_tk, ctk.data(), (size_t)m * 4, cudaMemcpyHostToDevice, st));
        MDH_CUDA(cudaMemcpyAsync(d_ti, cti.data(), (size_t)m * 4, cudaMemcpyHostToDevice, st));
        // Staged query copies for the compact batch live in a separate buffer.
        uint8_t* cq_u8 = nullptr;
        int32_t* cqn = nullptr;
        float* cq_f32 = nullptr;
        void* tmpbuf = nullptr;
        size_t need = qp.integer ? (size_t)m * ix->dpad + (size_t)m * 4 + 256
                                 : (size_t)m * f32_stride_floats * 4 + (size_t)m * 4 + 256;
        grow(&w.tmp, &w.tmp_bytes, need);
        tmpbuf = w.tmp;
        if (qp.integer) {
            cq_u8 = static_cast<uint8_t*>(tmpbuf);
            cqn = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(tmpbuf) + round_up((size_t)m * ix->dpad, 256));
            launch_gather_queries_u8(w.q_u8, w.qn, d_list, m, ix->dpad, cq_u8, cqn, st);
            res.launches++;
        } else {
            // The flagged float queries, gathered from the staged batch: [m][dim] then [m] aux.
            cq_f32 = static_cast<float*>(tmpbuf);
            launch_gather_queries_f32(w.q_f32, nq, ix->dim, d_list, m, cq_f32, st);
            res.launches++;
        }
        MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)m * 4, st));
        count_tc(lv, run_filter(ix, sh, lv, qp, cq_u8, cqn, cq_f32, m, d_tk, d_ti, last.cap, false, nullptr, true), m);
        MDH_CUDA(cudaMemsetAsync(w.status + 1, 0, sizeof(int32_t), st));
        launch_select(w.counts, w.cand, last.cap, lv.ids, m, k, 1, w.thr_key, w.thr_id, w.out_key, w.out_id, w.flags,
                      w.status + 1, d_list, n_cand, st);
        res.launches += 2;  // filter + select
        MDH_CUDA(cudaMemcpyAsync(w.h_status, w.status, 2 * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaStreamSynchronize(st));
        if (w.h_status[0] != kDevOk)
            throw Error(MDH_ERR_TIMEOUT, "tensor-core scan reported device status " + std::to_string(w.h_status[0]));
        flagged = w.h_status[1];
        res.pairs += lv.n * (int64_t)m;
    }
    if (rounds > 0)
        res.select_ms += std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t_rerun)
                             .count();
    // Verification (opt-in): for up to g_verify queries, an exact scan with no
    // pruning (the CUDA-core kernels compare every row) counts the rows at or
    // before each query's k-th result by (key, id).  An exact result has
    // exactly k of them; any other count is reported as violations.
    if (g_verify > 0 && qp.integer && nq > 0 && phase == kPhaseAll) {
        const int m = std::min(nq, g_verify);
        std::vector<int32_t> list((size_t)m);
        for (int i = 0; i < m; i++) list[(size_t)i] = (int32_t)((int64_t)i * nq / m);
        growT(&w.qlist, &w.qlist_bytes, (size_t)m * 4 * 3);
        int32_t* d_list = w.qlist;
        uint32_t* d_tk = reinterpret_cast<uint32_t*>(w.qlist + m);
        int32_t* d_ti = w.qlist + 2 * m;
        MDH_CUDA(cudaMemcpyAsync(d_list, list.data(), (size_t)m * 4, cudaMemcpyHostToDevice, st));
        grow(&w.tmp, &w.tmp_bytes, round_up((size_t)m * ix->dpad, 256) + (size_t)m * 4 + 256);
        uint8_t* cq_u8 = static_cast<uint8_t*>(w.tmp);
        int32_t* cqn = reinterpret_cast<int32_t*>(cq_u8 + round_up((size_t)m * ix->dpad, 256));
        launch_gather_queries_u8(w.q_u8, w.qn, d_list, m, ix->dpad, cq_u8, cqn, st);
        launch_verify_thresholds(d_list, m, w.out_key, w.out_id, k, k, d_tk, d_ti, st);
        MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)m * 4, st));
        const int mode = ix->metric == MDH_METRIC_L2 ? 0 : 1;
        if (stream_supported(ix->dpad, lv))
            launch_scan_stream_u8(lv, ix->dpad, mode, cq_u8, cqn, m, d_tk, d_ti, w.counts, w.cand, 0, 0, w.status, st);
        else if (mode == 0)
            launch_filter_simt_u8_l2(lv, ix->dpad, cq_u8, cqn, m, d_tk, d_ti, w.counts, w.cand, 0, 0, st);
        else
            launch_filter_simt_u8_cos(lv, ix->dpad, cq_u8, cqn, m, d_tk, d_ti, w.counts, w.cand, 0, 0, st);
        launch_count_violations(w.counts, m, k, n_viol, st);
        res.launches += 4;
        res.verified = m;
    }
    MDH_CUDA(cudaMemcpyAsync(w.h_status, w.status, 12 * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
    MDH_CUDA(cudaStreamSynchronize(st));
    if (w.h_status[0] != kDevOk)
        throw Error(MDH_ERR_TIMEOUT, "scan reported device status " + std::to_string(w.h_status[0]));
    {
        unsigned long long cand_n = 0, viol_n = 0, bs[3] = {};
        std::memcpy(&cand_n, w.h_status + 2, 8);
        std::memcpy(&viol_n, w.h_status + 4, 8);
        std::memcpy(bs, w.h_status + kStatusBlockStats, sizeof(bs));
        res.candidates = (int64_t)cand_n;
        res.violations = (int64_t)viol_n;
        res.blocks_passed = (int64_t)bs[1];
        res.pruned = res.tc_pairs - (int64_t)bs[2];
    }
    (void)host_q_u8;
    return res;
}

// Prepare the float queries of one chunk following the reference formula.
// Output layout: [nq][dim] values, then [nq] aux (|q|^2 for cosine scores).
void prepare_float_queries(const mdh_index* ix, const QueryPlan& qp, const float* q, int nq, int mode,
                           std::vector<float>& out) {
    const int d = ix->dim;
    out.assign((size_t)nq * d + nq, 0.0f);
    for (int i = 0; i < nq; i++) {
        const float* src = q + (size_t)i * d;
        float* dst = &out[(size_t)i * d];
        std::memcpy(dst, src, (size_t)d * 4);
        if (qp.kind == kScoreSpeedCos) {
            // src/speed_cpu.cpp:278-287 (single query) and :365-372 (batch):
            // |q| by a sequential FMA chain, scaled by 1/|q|.
            float qn = 0.0f;
            for (int j = 0; j < d; j++) qn = std::fmaf(src[j], src[j], qn);
            float inv;
            if (mode == MDH_SCORE_SPEED_BATCH) {
                inv = qn > 1e-12f ? 1.0f / std::sqrt(qn) : 0.0f;  // batch path compares |q|^2
            } else {
                float s = std::sqrt(qn);
                inv = s > 1e-12f ? 1.0f / s : 0.0f;
            }
            for (int j = 0; j < d; j++) dst[j] = src[j] * inv;
        }
        if (qp.kind == kScoreCosU8 || qp.kind == kScoreExactCosF32) {
            float s = 0.0f;  // src/winnex_madhava.cpp:759
            for (int j = 0; j < d; j++) s = std::fmaf(src[j], src[j], s);
            out[(size_t)nq * d + i] = s;
        }
    }
}

QueryPlan plan_query(const mdh_index* ix, bool integral, int mode) {
    QueryPlan qp;
    const bool l2 = ix->metric == MDH_METRIC_L2;
    qp.asc = l2;
    if (!ix->is_f32 && integral && ix->dim <= 256 && (l2 || mode == MDH_SCORE_EXACT)) {
        qp.integer = true;
        qp.int_dist = l2;
        return qp;
    }
    if (ix->is_f32) {
        qp.kind = l2 ? kScoreSpeedL2 : kScoreSpeedCos;
        qp.asc = false;
    } else if (mode == MDH_SCORE_SPEED || mode == MDH_SCORE_SPEED_BATCH) {
        qp.kind = l2 ? kScoreSpeedL2 : kScoreSpeedCos;
        qp.asc = false;
    } else {
        qp.kind = l2 ? kScoreL2SqU8 : kScoreCosU8;
        qp.asc = l2;
    }
    return qp;
}

bool all_integral_u8(const float* q, size_t count) {
    for (size_t i = 0; i < count; i++) {
        float v = q[i];
        if (!(v >= 0.0f && v <= 255.0f) || v != std::floor(v)) return false;
    }
    return true;
}

// Full search of a batch: chunk queries, run every shard, merge.
// Exactly one of host_u8 / host_f32 is set.
void search_impl(mdh_index* ix, const uint8_t* host_u8, const float* host_f32, int nq, int k, int mode,
                 int32_t* out_ids, float* out_val_f, int32_t* out_val_i, mdh_stats* stats,
                 uint32_t* out_keys = nullptr, bool locked = false) {
    auto t0 = std::chrono::high_resolution_clock::now();
    MDH_REQUIRE(ix, MDH_ERR_INVALID_ARG, "null index");
    MDH_REQUIRE(nq >= 0, MDH_ERR_INVALID_ARG, "nq must be >= 0");
    MDH_REQUIRE(k >= 0, MDH_ERR_INVALID_ARG, "k must be >= 0");
    MDH_REQUIRE(nq == 0 || host_u8 || host_f32, MDH_ERR_INVALID_ARG, "null queries");
    MDH_REQUIRE(nq == 0 || k == 0 || out_ids, MDH_ERR_INVALID_ARG, "null output ids");
    std::unique_lock<std::mutex> lock(ix->mu, std::defer_lock);
    if (!locked) lock.lock();
    mdh_stats st{};
    const int dim = ix->dim, dpad = ix->dpad;
    const int kk = (int)std::min<int64_t>(k, ix->n);
    for (size_t i = 0; i < (size_t)nq * k; i++) out_ids[i] = -1;
    if (out_val_f)
        for (size_t i = 0; i < (size_t)nq * k; i++) out_val_f[i] = NAN;
    if (out_val_i)
        for (size_t i = 0; i < (size_t)nq * k; i++) out_val_i[i] = -1;
    if (nq == 0 || kk == 0) {
        if (stats) *stats = st;
        return;
    }
    bool integral = host_u8 != nullptr || (!ix->is_f32 && all_integral_u8(host_f32, (size_t)nq * dim));
    QueryPlan qp = plan_query(ix, integral, mode);
    MDH_REQUIRE(qp.integer || host_f32, MDH_ERR_NOT_INTEGRAL, "u8 queries need the integer path");
    if (qp.kind == kScoreSpeedCos && !ix->is_f32)
        for (auto& sh : ix->shards) ensure_speed_rows_u8(ix, sh);
    if (qp.kind == kScoreSpeedCos && g_scan_path != 1)
        for (auto& sh : ix->shards) ensure_bf16_rows(ix, sh);
    if (qp.kind == kScoreExactCosF32)
        throw Error(MDH_ERR_UNSUPPORTED, "float-row exact cosine is not built in this version");

    const int nshard = (int)ix->shards.size();
    // Query chunk: bounded candidate memory.
    int chunk = (int)std::max<size_t>(1, kCandBudget / ((size_t)kCapMax * sizeof(uint2)));
    chunk = std::min(chunk, nq);
    std::vector<uint8_t> qbuf_u8;
    std::vector<float> qbuf_f32;
    std::vector<uint32_t> hkey((size_t)chunk * kk);
    std::vector<int32_t> hid((size_t)chunk * kk);
    for (int c0 = 0; c0 < nq; c0 += chunk) {
        const auto t_chunk = std::chrono::high_resolution_clock::now();
        const int m = std::min(chunk, nq - c0);
        // This chunk's u8 queries with the padded row stride: the caller's
        // rows themselves when dim is already a multiple of the stride unit,
        // else a zero-padded host copy.
        const uint8_t* qsrc = nullptr;
        if (qp.integer) {
            if (host_u8 && dim == dpad) {
                qsrc = host_u8 + (size_t)c0 * dim;
            } else {
                qbuf_u8.assign((size_t)m * dpad, 0);
                for (int i = 0; i < m; i++) {
                    uint8_t* dst = qbuf_u8.data() + (size_t)i * dpad;
                    if (host_u8) {
                        std::memcpy(dst, host_u8 + (size_t)(c0 + i) * dim, (size_t)dim);
                    } else {
                        const float* src = host_f32 + (size_t)(c0 + i) * dim;
                        for (int j = 0; j < dim; j++) dst[j] = (uint8_t)src[j];
                    }
                }
                qsrc = qbuf_u8.data();
            }
        } else if (qp.kind != kScoreSpeedCos) {
            prepare_float_queries(ix, qp, host_f32 + (size_t)c0 * dim, m, mode, qbuf_f32);
        }
        const auto t_staged = std::chrono::high_resolution_clock::now();  // host part of the query staging
        std::vector<ShardResult> sres((size_t)nshard);
        std::vector<std::string> errs((size_t)nshard);
        std::vector<mdh_status> codes((size_t)nshard, MDH_OK);
        std::vector<int64_t> st_launch((size_t)nshard, 0);
        std::vector<double> st_prep((size_t)nshard, 0.0);
        auto run = [&](int si) {
            try {
                Shard& sh = ix->shards[(size_t)si];
                if (take_fault(kFaultShard))
                    throw Error(MDH_ERR_INTERNAL, "shard " + std::to_string(si) +
                                                      " search failed: injected fault (mdh_set_fault)");
                MDH_CUDA(cudaSetDevice(sh.device));
                Workspace& w = sh.ws;
                ensure_status(w);
                MDH_CUDA(cudaEventRecord(w.ev_prep, sh.stream));
                if (qp.integer) {
                    growT(&w.q_u8, &w.q_u8_bytes, (size_t)m * dpad);
                    growT(&w.qn, &w.qn_bytes, (size_t)m * 4);
                    MDH_CUDA(cudaMemcpyAsync(w.q_u8, qsrc, (size_t)m * dpad, cudaMemcpyHostToDevice, sh.stream));
                    launch_query_norms_u8(w.q_u8, m, dpad, w.qn, sh.stream);
                    st_launch[(size_t)si] = 1;
                } else if (qp.kind == kScoreSpeedCos) {
                    // Raw rows up, normalized on the device in the reference's
                    // order (no aux term for this score).
                    growT(&w.q_f32, &w.q_f32_bytes, ((size_t)m * dim + m) * 4);
                    MDH_CUDA(cudaMemcpyAsync(w.q_f32, host_f32 + (size_t)c0 * dim, (size_t)m * dim * 4,
                                             cudaMemcpyHostToDevice, sh.stream));
                    MDH_CUDA(cudaMemsetAsync(w.q_f32 + (size_t)m * dim, 0, (size_t)m * 4, sh.stream));
                    uint16_t* qb = nullptr;
                    if (ix->dim % 8 == 0) {
                        growT(&w.q_bf16, &w.q_bf16_bytes, (size_t)m * dim * 2);
                        qb = w.q_bf16;
                    }
                    launch_normalize_speed_cos(w.q_f32, m, dim, mode == MDH_SCORE_SPEED_BATCH ? 1 : 0, qb, sh.stream);
                    st_launch[(size_t)si] = 1;
                } else {
                    growT(&w.q_f32, &w.q_f32_bytes, qbuf_f32.size() * 4);
                    MDH_CUDA(cudaMemcpyAsync(w.q_f32, qbuf_f32.data(), qbuf_f32.size() * 4, cudaMemcpyHostToDevice,
                                             sh.stream));
                }
                sres[(size_t)si] = search_shard(ix, sh, qp, m, kk, qsrc, qbuf_f32.data(), (size_t)dim);
                st_prep[(size_t)si] = event_ms(w.ev_prep, w.ev_start);
            } catch (const Error& e) {
                codes[(size_t)si] = e.code;
                errs[(size_t)si] = e.what();
            } catch (const std::exception& e) {
                codes[(size_t)si] = MDH_ERR_INTERNAL;
                errs[(size_t)si] = e.what();
            }
        };
        if (nshard == 1) {
            run(0);
        } else {
            std::vector<std::thread> th;
            for (int si = 0; si < nshard; si++) th.emplace_back(run, si);
            for (auto& t : th) t.join();
        }
        for (int si = 0; si < nshard; si++)
            if (codes[(size_t)si] != MDH_OK) throw Error(codes[(size_t)si], errs[(size_t)si]);
        double chunk_scan_ms = 0.0, chunk_sample_ms = 0.0, chunk_select_ms = 0.0, chunk_rescore_ms = 0.0,
               chunk_prep_ms = 0.0;
        for (double p : st_prep) chunk_prep_ms = std::max(chunk_prep_ms, p);
        for (auto& r : sres) {
            chunk_sample_ms = std::max(chunk_sample_ms, r.sample_ms);
            chunk_select_ms = std::max(chunk_select_ms, r.select_ms);
            chunk_rescore_ms = std::max(chunk_rescore_ms, r.rescore_ms);
            st.blocks_tested += r.blocks_tested;
            st.blocks_passed += r.blocks_passed;
            st.pairs_pruned_by_bound += r.pruned;
            st.pairs_scored += r.pairs;
            st.levels = std::max(st.levels, r.levels);
            st.tensor_core_path = std::max(st.tensor_core_path, r.scan_path - 1);
            st.full_scan_pairs += r.scan_pairs;
            st.kernel_launches += r.launches;
            st.candidates += r.candidates;
            st.bound_violations += r.violations;
            st.verified_queries += r.verified;
            chunk_scan_ms = std::max(chunk_scan_ms, r.scan_ms);  // shards run concurrently
        }
        st.full_scan_ms += chunk_scan_ms;
        st.sample_ms += chunk_sample_ms;
        st.select_ms += chunk_select_ms;
        st.rescore_ms += chunk_rescore_ms;
        st.prep_ms += chunk_prep_ms +
                      std::chrono::duration<double, std::milli>(t_staged - t_chunk).count();
        for (int64_t l : st_launch) st.kernel_launches += l;
        // Gather / merge to the first shard's device.
        Shard& s0 = ix->shards[0];
        MDH_CUDA(cudaSetDevice(s0.device));
        const uint32_t* fkey = s0.ws.out_key;
        const int32_t* fid = s0.ws.out_id;
        if (nshard > 1) {
            size_t per = (size_t)m * kk;
            uint32_t* all_key = nullptr;
            int32_t* all_id = nullptr;
            growT(&s0.ws.tmp, &s0.ws.tmp_bytes, per * 8 * nshard + per * 8 + 1024);
            all_key = static_cast<uint32_t*>(s0.ws.tmp);
            all_id = reinterpret_cast<int32_t*>(all_key + per * nshard);
            uint32_t* mkey = reinterpret_cast<uint32_t*>(all_id + per * nshard);
            int32_t* mid = reinterpret_cast<int32_t*>(mkey + per);
            for (int si = 0; si < nshard; si++) {
                Shard& sh = ix->shards[(size_t)si];
                MDH_CUDA(cudaMemcpyPeerAsync(all_key + per * si, s0.device, sh.ws.out_key, sh.device, per * 4, s0.stream));
                MDH_CUDA(cudaMemcpyPeerAsync(all_id + per * si, s0.device, sh.ws.out_id, sh.device, per * 4, s0.stream));
            }
            launch_merge_topk(all_key, all_id, nshard, m, kk, mkey, mid, s0.stream);
            st.kernel_launches++;
            fkey = mkey;
            fid = mid;
        }
        MDH_CUDA(cudaMemcpyAsync(hkey.data(), fkey, (size_t)m * kk * 4, cudaMemcpyDeviceToHost, s0.stream));
        MDH_CUDA(cudaMemcpyAsync(hid.data(), fid, (size_t)m * kk * 4, cudaMemcpyDeviceToHost, s0.stream));
        MDH_CUDA(cudaStreamSynchronize(s0.stream));
        for (int i = 0; i < m; i++) {
            for (int j = 0; j < kk; j++) {
                const size_t src = (size_t)i * kk + j, dst = (size_t)(c0 + i) * k + j;
                const int32_t id = hid[src];
                out_ids[dst] = id;
                if (out_keys) out_keys[dst] = hkey[src];
                if (id < 0) continue;
                const uint32_t key = hkey[src];
                if (out_val_i) out_val_i[dst] = qp.int_dist ? (int32_t)key : -1;
                if (out_val_f) {
                    if (qp.int_dist)
                        out_val_f[dst] = (float)key;
                    else if (qp.integer)  // integer cosine: key encodes the descending float score
                        out_val_f[dst] = key_to_float_asc(~key);
                    else
                        out_val_f[dst] = qp.asc ? key_to_float_asc(key) : key_to_float_asc(~key);
                }
            }
        }
    }
    st.latency_ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0).count();
    if (stats) *stats = st;
}

// Audited search (MadhavaL2::search_audited / search_with_commitment,
// src/winnex_madhava.cpp:1258-1591) on the exact engine, one query at a time:
//   1. the exact top-(k + max_records): its first k are the result, its
//      k-th key is the threshold T, and the rest are the excluded rows
//      nearest the cut, in (key, id) order (the deterministic sample);
//   2. the audit pass: every shard's whole level scanned once more with the
//      threshold (T, any id) and no candidate storage, so the counters give
//      the rows at or within T -- every other row is provably outside the
//      top k -- and, on the tensor-core path, the real rows of the 64-row
//      blocks whose bound could not settle them; the rest were excluded by
//      the block bound alone.
constexpr int64_t kAuditRecordSearchMax = int64_t(1) << 18;

void audit_impl(mdh_index* ix, const uint8_t* host_u8, const float* host_f32, int nq, int k, int max_records,
                int32_t* out_ids, float* out_val_f, int32_t* out_val_i, int32_t* rec_ids, float* rec_val_f,
                int32_t* rec_val_i, mdh_audit* audit, mdh_stats* stats) {
    auto t0 = std::chrono::high_resolution_clock::now();
    MDH_REQUIRE(ix, MDH_ERR_INVALID_ARG, "null index");
    MDH_REQUIRE(nq >= 0 && k >= 1 && max_records >= 0, MDH_ERR_INVALID_ARG,
                "nq and max_records must be >= 0, k >= 1");
    MDH_REQUIRE(nq == 0 || ((host_u8 || host_f32) && out_ids && audit), MDH_ERR_INVALID_ARG,
                "null queries or outputs");
    MDH_REQUIRE(nq == 0 || max_records == 0 || rec_ids, MDH_ERR_INVALID_ARG, "null record ids");
    std::lock_guard<std::mutex> lock(ix->mu);
    mdh_stats total{};
    const int dim = ix->dim;
    const int64_t n = ix->n;
    const int kk = (int)std::min<int64_t>(k, n);
    const int m = (int)std::max<int64_t>(0, std::min<int64_t>(max_records, n - kk));
    const int k2 = kk + m;
    std::vector<int32_t> ids2((size_t)std::max(k2, 1)), vi2((size_t)std::max(k2, 1));
    std::vector<float> vf2((size_t)std::max(k2, 1));
    std::vector<uint32_t> keys2((size_t)std::max(k2, 1));
    for (int i = 0; i < nq; i++) {
        mdh_audit& a = audit[i];
        a = mdh_audit{};
        a.rows = n;
        for (int j = 0; j < k; j++) {
            out_ids[(size_t)i * k + j] = -1;
            if (out_val_f) out_val_f[(size_t)i * k + j] = NAN;
            if (out_val_i) out_val_i[(size_t)i * k + j] = -1;
        }
        for (int j = 0; j < max_records; j++) {
            rec_ids[(size_t)i * max_records + j] = -1;
            if (rec_val_f) rec_val_f[(size_t)i * max_records + j] = NAN;
            if (rec_val_i) rec_val_i[(size_t)i * max_records + j] = -1;
        }
        if (kk == 0) continue;
        const uint8_t* qu = host_u8 ? host_u8 + (size_t)i * dim : nullptr;
        const float* qf = host_f32 ? host_f32 + (size_t)i * dim : nullptr;
        mdh_stats st{};
        search_impl(ix, qu, qf, 1, k2, MDH_SCORE_EXACT, ids2.data(), vf2.data(), vi2.data(), &st, keys2.data(), true);
        total.pairs_scored += st.pairs_scored;
        total.pairs_pruned_by_bound += st.pairs_pruned_by_bound;
        total.full_scan_pairs += st.full_scan_pairs;
        total.kernel_launches += st.kernel_launches;
        total.candidates += st.candidates;
        total.blocks_tested += st.blocks_tested;
        total.blocks_passed += st.blocks_passed;
        total.full_scan_ms += st.full_scan_ms;
        total.sample_ms += st.sample_ms;
        total.select_ms += st.select_ms;
        total.prep_ms += st.prep_ms;
        total.levels = std::max(total.levels, st.levels);
        total.tensor_core_path = std::max(total.tensor_core_path, st.tensor_core_path);
        for (int j = 0; j < kk; j++) {
            out_ids[(size_t)i * k + j] = ids2[(size_t)j];
            if (out_val_f) out_val_f[(size_t)i * k + j] = vf2[(size_t)j];
            if (out_val_i) out_val_i[(size_t)i * k + j] = vi2[(size_t)j];
        }
        const uint32_t T = keys2[(size_t)kk - 1];
        // An integer distance where the path returns one, else the float score.
        a.threshold = vi2[(size_t)kk - 1] >= 0 ? (double)vi2[(size_t)kk - 1] : (double)vf2[(size_t)kk - 1];
        int r = 0;
        for (int j = kk; j < k2; j++) {
            if (ids2[(size_t)j] < 0 || keys2[(size_t)j] <= T) continue;  // ties with the k-th are not excluded
            rec_ids[(size_t)i * max_records + r] = ids2[(size_t)j];
            if (rec_val_f) rec_val_f[(size_t)i * max_records + r] = vf2[(size_t)j];
            if (rec_val_i) rec_val_i[(size_t)i * max_records + r] = vi2[(size_t)j];
            r++;
        }
        a.n_records = r;
        // The audit pass over every shard's whole level, on the query the
        // search just staged in each shard's workspace.
        const bool integral = host_u8 != nullptr || (!ix->is_f32 && all_integral_u8(qf, (size_t)dim));
        const QueryPlan qp = plan_query(ix, integral, MDH_SCORE_EXACT);
        int64_t within = 0, unsettled_rows = 0;
        bool bounded = true;
        for (Shard& sh : ix->shards) {
            MDH_CUDA(cudaSetDevice(sh.device));
            Workspace& w = sh.ws;
            const Level& lv = sh.levels.back();
            const uint32_t tk = T;
            const int32_t ti = 0x7fffffff;
            MDH_CUDA(cudaMemcpyAsync(w.thr_key, &tk, 4, cudaMemcpyHostToDevice, sh.stream));
            MDH_CUDA(cudaMemcpyAsync(w.thr_id, &ti, 4, cudaMemcpyHostToDevice, sh.stream));
            MDH_CUDA(cudaMemsetAsync(w.counts, 0, 4, sh.stream));
            MDH_CUDA(cudaMemsetAsync(w.status, 0, kStatusWords * sizeof(int32_t), sh.stream));
            const int used = run_filter(ix, sh, lv, qp, w.q_u8, w.qn, w.q_f32, 1, w.thr_key, w.thr_id, 0, false,
                                        nullptr, true);
            uint32_t cnt = 0;
            MDH_CUDA(cudaMemcpyAsync(&cnt, w.counts, 4, cudaMemcpyDeviceToHost, sh.stream));
            MDH_CUDA(cudaMemcpyAsync(w.h_status, w.status, kStatusWords * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                     sh.stream));
            MDH_CUDA(cudaStreamSynchronize(sh.stream));
            if (w.h_status[0] != kDevOk)
                throw Error(w.h_status[0] == kDevTimeout ? MDH_ERR_TIMEOUT : MDH_ERR_INTERNAL,
                            "audit scan reported device status " + std::to_string(w.h_status[0]));
            unsigned long long bs[3] = {};
            std::memcpy(bs, w.h_status + kStatusBlockStats, sizeof(bs));
            within += (int64_t)cnt;
            if (used == 2)
                unsettled_rows += (int64_t)bs[2];
            else
                bounded = false;
            total.pairs_scored += lv.n;
            total.kernel_launches += 1;
        }
        // Rows tied with the k-th result fill the list before any excluded
        // row: then the records come from the top (within + max_records),
        // past the ties (a bounded search; beyond the bound the records stop
        // short).
        if (r < m && within > (int64_t)kk && within + m <= std::min<int64_t>(n, kAuditRecordSearchMax)) {
            const int k3 = (int)(within + m);
            std::vector<int32_t> ids3((size_t)k3), vi3((size_t)k3);
            std::vector<float> vf3((size_t)k3);
            std::vector<uint32_t> keys3((size_t)k3);
            mdh_stats st3{};
            search_impl(ix, qu, qf, 1, k3, MDH_SCORE_EXACT, ids3.data(), vf3.data(), vi3.data(), &st3, keys3.data(),
                        true);
            total.pairs_scored += st3.pairs_scored;
            total.kernel_launches += st3.kernel_launches;
            r = 0;
            for (int j = (int)within; j < k3 && r < m; j++) {
                if (ids3[(size_t)j] < 0 || keys3[(size_t)j] <= T) continue;
                rec_ids[(size_t)i * max_records + r] = ids3[(size_t)j];
                if (rec_val_f) rec_val_f[(size_t)i * max_records + r] = vf3[(size_t)j];
                if (rec_val_i) rec_val_i[(size_t)i * max_records + r] = vi3[(size_t)j];
                r++;
            }
            a.n_records = r;
        }
        a.within = within;
        a.excluded = n - within;
        a.excluded_by_bound = bounded ? n - unsettled_rows : -1;
        // Every returned row is at or within T, so fewer than k such rows
        // would mean a row the search missed or mis-scored.
        a.violations = within < kk ? kk - within : 0;
        total.bound_violations += a.violations;
        total.verified_queries += 1;
    }
    total.latency_ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0).count();
    if (stats) *stats = total;
}

void create_impl(const void* host, bool f32, int64_t n, int32_t dim, int32_t metric, const int32_t* devices,
                 int32_t ndev, int64_t id_offset, mdh_index** out) {
    MDH_REQUIRE(out, MDH_ERR_INVALID_ARG, "null output pointer");
    *out = nullptr;
    MDH_REQUIRE(n >= 0, MDH_ERR_INVALID_ARG, "n must be >= 0");
    MDH_REQUIRE(n == 0 || host, MDH_ERR_INVALID_ARG, "null corpus");
    MDH_REQUIRE(dim >= 1 && dim <= 4096, MDH_ERR_INVALID_ARG, "dim must be in [1, 4096]");
    MDH_REQUIRE(metric == MDH_METRIC_COSINE || metric == MDH_METRIC_L2, MDH_ERR_INVALID_ARG, "metric must be 0 or 1");
    MDH_REQUIRE(id_offset >= 0 && n + id_offset <= 0x7FFFFFFF, MDH_ERR_INVALID_ARG,
                "row ids must fit in int32 (n + id_offset <= 2^31 - 1)");
    std::vector<int> devs;
    if (devices && ndev > 0) {
        for (int i = 0; i < ndev; i++) devs.push_back(devices[i]);
    } else {
        int cur = 0;
        cudaError_t e = cudaGetDevice(&cur);
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw Error(MDH_ERR_CUDA, "no CUDA device is available (this library has no CPU fallback)");
        }
        devs.push_back(cur);
    }
    for (int d : devs) check_device_usable(d);
    std::unique_ptr<mdh_index> ix(new mdh_index());
    ix->n = n;
    ix->dim = dim;
    ix->dpad = (int)round_up(dim, kRowAlign);
    ix->metric = metric;
    ix->is_f32 = f32;
    const int nd = (int)devs.size();
    ix->shards.resize((size_t)nd);
    try {
        for (int i = 0; i < nd; i++) {
            Shard& sh = ix->shards[(size_t)i];
            sh.device = devs[(size_t)i];
            MDH_CUDA(cudaSetDevice(sh.device));
            MDH_CUDA(cudaStreamCreateWithFlags(&sh.stream, cudaStreamNonBlocking));
            const int64_t r0 = n * i / nd, r1 = n * (i + 1) / nd;
            sh.id_base = id_offset + r0;
            if (f32)
                build_shard_f32(ix.get(), sh, static_cast<const float*>(host) + (size_t)r0 * dim, r1 - r0);
            else
                build_shard_u8(ix.get(), sh, static_cast<const uint8_t*>(host) + (size_t)r0 * dim, r1 - r0);
        }
    } catch (...) {
        for (auto& sh : ix->shards) free_shard(sh);
        throw;
    }
    *out = ix.release();
}

}  // namespace

bool take_fault(int site) {
    int want = site;
    return g_fault.load() == site && g_fault.compare_exchange_strong(want, kFaultNone);
}

[[noreturn]] void throw_cuda(cudaError_t e, const char* what, const char* file, int line) {
    cudaGetLastError();
    mdh_status code = (e == cudaErrorMemoryAllocation) ? MDH_ERR_OOM : MDH_ERR_CUDA;
    throw Error(code, std::string("CUDA error ") + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ") in " + what +
                          " at " + file + ":" + std::to_string(line));
}

void check_device_usable(int dev) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        throw Error(MDH_ERR_CUDA, "no CUDA device is available (this library has no CPU fallback)");
    }
    MDH_REQUIRE(dev >= 0 && dev < count, MDH_ERR_INVALID_ARG, "device ordinal out of range");
    cudaDeviceProp p;
    MDH_CUDA(cudaGetDeviceProperties(&p, dev));
    if (p.major != 10 || p.minor != 0)
        throw Error(MDH_ERR_CUDA, "this library is built for sm_100a (B200); device " + std::to_string(dev) +
                                      " is sm_" + std::to_string(p.major) + std::to_string(p.minor));
}

int device_sm_count(int dev) {
    static int cache[64] = {0};
    if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
    int v = 0;
    MDH_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    if (dev >= 0 && dev < 64) cache[dev] = v;
    return v;
}

void ensure(void** p, size_t* have, size_t need) { grow(p, have, need); }

mdh_status run_guarded(void (*fn)(void*), void* ctx) {
    return guard([&] { fn(ctx); });
}

}  // namespace mdh

using namespace mdh;

extern "C" {

mdh_status mdh_index_create_u8(const uint8_t* host_corpus, int64_t n, int32_t dim, int32_t metric,
                               const int32_t* devices, int32_t ndev, int64_t id_offset, mdh_index** out) {
    return guard([&] { create_impl(host_corpus, false, n, dim, metric, devices, ndev, id_offset, out); });
}

mdh_status mdh_index_create_f32(const float* host_corpus, int64_t n, int32_t dim, int32_t metric,
                                const int32_t* devices, int32_t ndev, int64_t id_offset, mdh_index** out) {
    return guard([&] { create_impl(host_corpus, true, n, dim, metric, devices, ndev, id_offset, out); });
}

mdh_status mdh_index_create_u8_device(const uint8_t* dev_corpus, int64_t n, int32_t dim, int32_t metric,
                                      int64_t id_offset, mdh_index** out) {
    return guard([&] {
        if (n > 0) {
            cudaPointerAttributes a;
            MDH_CUDA(cudaPointerGetAttributes(&a, dev_corpus));
            MDH_REQUIRE(a.type == cudaMemoryTypeDevice, MDH_ERR_INVALID_ARG, "dev_corpus is not device memory");
            int32_t dev = a.device;
            create_impl(dev_corpus, false, n, dim, metric, &dev, 1, id_offset, out);
        } else {
            create_impl(dev_corpus, false, n, dim, metric, nullptr, 0, id_offset, out);
        }
    });
}

mdh_status mdh_index_destroy(mdh_index* index) {
    return guard([&] {
        if (!index) return;
        for (auto& sh : index->shards) free_shard(sh);
        delete index;
    });
}

mdh_status mdh_index_info(const mdh_index* index, int64_t* n, int32_t* dim, int32_t* metric, int32_t* ndev) {
    return guard([&] {
        MDH_REQUIRE(index, MDH_ERR_INVALID_ARG, "null index");
        if (n) *n = index->n;
        if (dim) *dim = index->dim;
        if (metric) *metric = index->metric;
        if (ndev) *ndev = (int32_t)index->shards.size();
    });
}

mdh_status mdh_index_memory(const mdh_index* index, int64_t* level_bytes, int64_t* workspace_bytes) {
    return guard([&] {
        MDH_REQUIRE(index, MDH_ERR_INVALID_ARG, "null index");
        int64_t lv_b = 0, ws_b = 0;
        for (const Shard& sh : index->shards) {
            for (const Level& lv : sh.levels) {
                if (!lv.owns) continue;
                if (lv.rows) lv_b += lv.n_pad * index->dpad + lv.n_pad * 4;
                if (lv.ids) lv_b += lv.n_pad * 4;
                if (lv.rows_f32) lv_b += lv.n_pad * (int64_t)index->dim * 4 + lv.n_pad * 4;
                if (lv.rows_bf16) lv_b += lv.n_pad * (int64_t)index->dim * 2;
            }
            const Workspace& w = sh.ws;
            for (size_t b : {w.q_u8_bytes, w.q_f32_bytes, w.q_bf16_bytes, w.qn_bytes, w.thr_key_bytes, w.thr_id_bytes,
                             w.counts_bytes, w.cand_bytes, w.out_key_bytes, w.out_id_bytes, w.flags_bytes,
                             w.qlist_bytes, w.tmp_bytes})
                ws_b += (int64_t)b;
            if (w.status) ws_b += kStatusWords * 4;
        }
        if (level_bytes) *level_bytes = lv_b;
        if (workspace_bytes) *workspace_bytes = ws_b;
    });
}

mdh_status mdh_index_id_base(const mdh_index* index, int64_t* first_id) {
    return guard([&] {
        MDH_REQUIRE(index && first_id, MDH_ERR_INVALID_ARG, "null argument");
        *first_id = index->shards.empty() ? 0 : index->shards[0].id_base;
    });
}

mdh_status mdh_search_f32(mdh_index* index, const float* host_queries, int32_t nq, int32_t k, int32_t mode,
                          int32_t* out_ids, float* out_dist, mdh_stats* stats) {
    return guard([&] {
        MDH_REQUIRE(mode == MDH_SCORE_EXACT || mode == MDH_SCORE_SPEED || mode == MDH_SCORE_SPEED_BATCH,
                    MDH_ERR_INVALID_ARG, "mode must be an mdh_score_mode value");
        search_impl(index, nullptr, host_queries, nq, k, mode, out_ids, out_dist, nullptr, stats);
    });
}

mdh_status mdh_search_u8(mdh_index* index, const uint8_t* host_queries, int32_t nq, int32_t k, int32_t* out_ids,
                         int32_t* out_dist, mdh_stats* stats) {
    return guard([&] {
        MDH_REQUIRE(index && !index->is_f32, MDH_ERR_INVALID_ARG, "u8 queries need a u8 index");
        search_impl(index, host_queries, nullptr, nq, k, MDH_SCORE_EXACT, out_ids, nullptr, out_dist, stats);
    });
}

mdh_status mdh_audit_f32(mdh_index* index, const float* host_queries, int32_t nq, int32_t k, int32_t max_records,
                         int32_t* out_ids, float* out_values, int32_t* rec_ids, float* rec_values, mdh_audit* audit,
                         mdh_stats* stats) {
    return guard([&] {
        audit_impl(index, nullptr, host_queries, nq, k, max_records, out_ids, out_values, nullptr, rec_ids,
                   rec_values, nullptr, audit, stats);
    });
}

mdh_status mdh_audit_u8(mdh_index* index, const uint8_t* host_queries, int32_t nq, int32_t k, int32_t max_records,
                        int32_t* out_ids, int32_t* out_dist, int32_t* rec_ids, int32_t* rec_dist, mdh_audit* audit,
                        mdh_stats* stats) {
    return guard([&] {
        audit_impl(index, host_queries, nullptr, nq, k, max_records, out_ids, nullptr, out_dist, rec_ids, nullptr,
                   rec_dist, audit, stats);
    });
}

}  // extern "C"

namespace mdh {
namespace {

// The device-resident u8 search (mdh_search_u8_device) and its cooperative
// phases (mdh_search_u8_device_sample / _bounded): queries, results and the
// threshold lists are device pointers on the index's device.
void device_search(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k, int phase,
                   const int32_t* thr_dist, const int32_t* thr_ids, int32_t* dev_ids, int32_t* dev_dist, void* stream,
                   mdh_stats* stats) {
        auto t0 = std::chrono::high_resolution_clock::now();
        MDH_REQUIRE(index && !index->is_f32, MDH_ERR_INVALID_ARG, "u8 queries need a u8 index");
        MDH_REQUIRE(index->shards.size() == 1, MDH_ERR_UNSUPPORTED, "device search needs a single-device index");
        MDH_REQUIRE(index->dim <= 256, MDH_ERR_UNSUPPORTED, "device u8 search supports dim <= 256");
        MDH_REQUIRE(nq >= 0 && k >= 0, MDH_ERR_INVALID_ARG, "nq and k must be >= 0");
        MDH_REQUIRE(nq == 0 || (dev_queries && dev_ids), MDH_ERR_INVALID_ARG, "null device buffer");
        std::lock_guard<std::mutex> lock(index->mu);
        Shard& sh = index->shards[0];
        MDH_CUDA(cudaSetDevice(sh.device));
        mdh_stats st{};
        const int kk = (int)std::min<int64_t>(k, index->n);
        cudaStream_t user = static_cast<cudaStream_t>(stream);
        cudaStream_t saved = sh.stream;
        if (user) sh.stream = user;
        try {
            if (nq > 0 && k > 0) {
                Workspace& w = sh.ws;
                const int dpad = index->dpad;
                ensure_status(w);
                MDH_CUDA(cudaEventRecord(w.ev_prep, sh.stream));
                growT(&w.q_u8, &w.q_u8_bytes, (size_t)nq * dpad);
                growT(&w.qn, &w.qn_bytes, (size_t)nq * 4);
                if (dpad != index->dim) MDH_CUDA(cudaMemsetAsync(w.q_u8, 0, (size_t)nq * dpad, sh.stream));
                MDH_CUDA(cudaMemcpy2DAsync(w.q_u8, dpad, dev_queries, index->dim, index->dim, nq,
                                           cudaMemcpyDeviceToDevice, sh.stream));
                launch_query_norms_u8(w.q_u8, nq, dpad, w.qn, sh.stream);
                QueryPlan qp;
                qp.integer = true;
                qp.int_dist = index->metric == MDH_METRIC_L2;
                ShardResult r;
                if (kk > 0) r = search_shard(index, sh, qp, nq, kk, nullptr, nullptr, 0, phase, thr_dist, thr_ids);
                st.pairs_scored = r.pairs;
                st.levels = r.levels;
                st.tensor_core_path = std::max(0, r.scan_path - 1);
                st.full_scan_ms = r.scan_ms;
                st.full_scan_pairs = r.scan_pairs;
                st.kernel_launches = 1 + r.launches;  // query norms + the shard's search
                st.candidates = r.candidates;
                st.bound_violations = r.violations;
                st.verified_queries = r.verified;
                st.sample_ms = r.sample_ms;
                st.select_ms = r.select_ms;
                st.blocks_tested = r.blocks_tested;
                st.blocks_passed = r.blocks_passed;
                st.pairs_pruned_by_bound = r.pruned;
                if (kk > 0) st.prep_ms = event_ms(w.ev_prep, w.ev_start);
                if (kk == k) {
                    MDH_CUDA(cudaMemcpyAsync(dev_ids, w.out_id, (size_t)nq * k * 4, cudaMemcpyDeviceToDevice, sh.stream));
                    if (dev_dist)
                        MDH_CUDA(cudaMemcpyAsync(dev_dist, w.out_key, (size_t)nq * k * 4, cudaMemcpyDeviceToDevice,
                                                 sh.stream));
                } else {
                    MDH_CUDA(cudaMemsetAsync(dev_ids, 0xFF, (size_t)nq * k * 4, sh.stream));
                    MDH_CUDA(cudaMemcpy2DAsync(dev_ids, (size_t)k * 4, w.out_id, (size_t)kk * 4, (size_t)kk * 4, nq,
                                               cudaMemcpyDeviceToDevice, sh.stream));
                    if (dev_dist) {
                        MDH_CUDA(cudaMemsetAsync(dev_dist, 0xFF, (size_t)nq * k * 4, sh.stream));
                        MDH_CUDA(cudaMemcpy2DAsync(dev_dist, (size_t)k * 4, w.out_key, (size_t)kk * 4, (size_t)kk * 4,
                                                   nq, cudaMemcpyDeviceToDevice, sh.stream));
                    }
                }
                MDH_CUDA(cudaStreamSynchronize(sh.stream));
            }
        } catch (...) {
            sh.stream = saved;
            throw;
        }
        sh.stream = saved;
        st.latency_ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0).count();
        if (stats) *stats = st;
}

}  // namespace
}  // namespace mdh

extern "C" {

mdh_status mdh_search_u8_device(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                int32_t* dev_ids, int32_t* dev_dist, void* stream, mdh_stats* stats) {
    return guard([&] {
        device_search(index, dev_queries, nq, k, kPhaseAll, nullptr, nullptr, dev_ids, dev_dist, stream, stats);
    });
}

mdh_status mdh_search_u8_device_sample(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                       int32_t* dev_ids, int32_t* dev_dist, void* stream, mdh_stats* stats) {
    return guard([&] {
        device_search(index, dev_queries, nq, k, kPhaseSample, nullptr, nullptr, dev_ids, dev_dist, stream, stats);
    });
}

mdh_status mdh_search_u8_device_bounded(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                        const int32_t* dev_thr_dist, const int32_t* dev_thr_ids, int32_t* dev_ids,
                                        int32_t* dev_dist, void* stream, mdh_stats* stats) {
    return guard([&] {
        MDH_REQUIRE(nq == 0 || k == 0 || (dev_thr_dist && dev_thr_ids), MDH_ERR_INVALID_ARG,
                    "null threshold lists");
        device_search(index, dev_queries, nq, k, kPhaseBounded, dev_thr_dist, dev_thr_ids, dev_ids, dev_dist,
                      stream, stats);
    });
}

mdh_status mdh_merge_topk_device(const int32_t* dev_dist_all, const int32_t* dev_ids_all, int32_t nshard, int32_t nq,
                                 int32_t k, int32_t* dev_dist_out, int32_t* dev_ids_out, void* stream) {
    return guard([&] {
        MDH_REQUIRE(nshard >= 1 && nq >= 0 && k >= 0, MDH_ERR_INVALID_ARG, "bad merge shape");
        MDH_REQUIRE(nq == 0 || k == 0 || (dev_dist_all && dev_ids_all && dev_dist_out && dev_ids_out),
                    MDH_ERR_INVALID_ARG, "null device buffer");
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        launch_merge_topk(reinterpret_cast<const uint32_t*>(dev_dist_all), dev_ids_all, nshard, nq, k,
                          reinterpret_cast<uint32_t*>(dev_dist_out), dev_ids_out, st);
        MDH_CUDA(cudaStreamSynchronize(st));
    });
}

mdh_status mdh_set_scan_path(int32_t path) {
    return guard([&] {
        MDH_REQUIRE(path >= 0 && path <= 3, MDH_ERR_INVALID_ARG, "path must be 0, 1, 2 or 3");
        g_scan_path = path;
    });
}

mdh_status mdh_set_verify(int32_t max_queries) {
    return guard([&] {
        MDH_REQUIRE(max_queries >= 0 && max_queries <= 65536, MDH_ERR_INVALID_ARG, "max_queries must be in [0, 65536]");
        g_verify = max_queries;
    });
}

mdh_status mdh_set_fault(int32_t site) {
    return guard([&] {
        MDH_REQUIRE(site >= kFaultNone && site <= kFaultIvfChunks, MDH_ERR_INVALID_ARG, "site must be 0 .. 3");
        g_fault.store(site);
    });
}

mdh_status mdh_check_wait_timeout(int32_t device, int64_t budget_cycles) {
    return guard([&] {
        MDH_REQUIRE(budget_cycles >= 1000 && budget_cycles <= (int64_t)1 << 32, MDH_ERR_INVALID_ARG,
                    "budget_cycles must be in [1000, 2^32]");
        int dev = device;
        if (dev < 0) MDH_CUDA(cudaGetDevice(&dev));
        check_device_usable(dev);
        MDH_CUDA(cudaSetDevice(dev));
        int32_t* d = nullptr;
        MDH_CUDA(cudaMalloc(&d, 2 * sizeof(int32_t)));
        int32_t h[2] = {-1, -1};
        cudaError_t e = cudaMemset(d, 0, 2 * sizeof(int32_t));
        if (e == cudaSuccess) {
            try {
                launch_wait_timeout_probe((long long)budget_cycles, d, nullptr);
            } catch (...) {
                cudaFree(d);
                throw;
            }
            e = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
        }
        cudaFree(d);
        MDH_CUDA(e);
        MDH_REQUIRE(h[1] == 0, MDH_ERR_INTERNAL, "the probe's barrier completed: nothing should arrive on it");
        if (h[0] == kDevTimeout)
            throw Error(MDH_ERR_TIMEOUT, "bounded device wait gave up after " + std::to_string(budget_cycles) +
                                             " cycles (expected: nothing arrives on the probe's barrier)");
        throw Error(MDH_ERR_INTERNAL, "bounded device wait returned without recording a timeout");
    });
}

mdh_status mdh_set_threshold_sharing(int32_t ranks) {
    return guard([&] {
        MDH_REQUIRE(ranks >= 1 && ranks <= 4096, MDH_ERR_INVALID_ARG, "ranks must be in [1, 4096]");
        g_threshold_sharing = ranks;
    });
}

mdh_status mdh_set_sample_ratio(int32_t ratio) {
    return guard([&] {
        MDH_REQUIRE(ratio == 0 || (ratio >= 2 && ratio <= 65536), MDH_ERR_INVALID_ARG,
                    "ratio must be 0 or in [2, 65536]");
        g_sample_top_ratio = ratio == 0 ? kSampleTopRatioDefault : ratio;
    });
}

int32_t mdh_plan_level_count(int64_t shard_rows, int32_t k) {
    if (shard_rows <= 0 || k <= 0) return 0;
    try {
        std::vector<int64_t> sizes = plan_samples(shard_rows);
        sizes.push_back(shard_rows);
        return (int32_t)plan_levels(sizes, shard_rows, (int)std::min<int64_t>(k, shard_rows)).size();
    } catch (...) {
        return -1;
    }
}

mdh_status mdh_set_candidate_cap_limit(int32_t cap) {
    return guard([&] {
        MDH_REQUIRE(cap == 0 || (cap >= 64 && cap <= kCapMax && (cap & (cap - 1)) == 0), MDH_ERR_INVALID_ARG,
                    "cap must be 0 or a power of two in [64, 16384]");
        g_cap_limit = cap;
    });
}

int32_t mdh_device_count(void) {
    int c = 0;
    if (cudaGetDeviceCount(&c) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return c;
}

const char* mdh_last_error(void) { return g_last_error.c_str(); }

const char* mdh_version(void) { return "winnex-madhava-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
