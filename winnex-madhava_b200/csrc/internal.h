// Internal host-side interfaces shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace mdh {

// A norm-sorted row set on one device: either a nested random sample of the
// shard (used to find per-query distance thresholds) or the whole shard.
struct Level {
    int64_t n = 0;           // real rows
    int64_t n_pad = 0;       // rows padded to kTileRows (pad rows: zero bytes, kNormPad, id -1)
    uint8_t* rows = nullptr; // [n_pad][dpad] u8, ascending (|v|^2, id)
    int32_t* norms = nullptr;// [n_pad] |v|^2
    int32_t* ids = nullptr;  // [n_pad] global row id
    float* rows_f32 = nullptr;   // [n_pad][dim] float rows (float corpora / float-score paths)
    float* norms_f32 = nullptr;  // [n_pad] float |v|^2 (SpeedEngine semantics)
    CUtensorMap tmap_rows;   // TMA map over `rows` (1-SM tensor-core scan), valid if has_tmap
    bool has_tmap = false;
    CUtensorMap tmap_rows_pair;  // TMA map over `rows` with half-tile boxes (2-SM scan)
    bool has_tmap_pair = false;
    uint16_t* rows_bf16 = nullptr;  // [n_pad][dim] bf16 copy of rows_f32 (approximate tensor scan)
    CUtensorMap tmap_bf16;          // TMA map over rows_bf16, 64 x 128 boxes, 128-byte swizzle
    bool has_tmap_bf16 = false;
    bool owns = true;        // false when aliasing another level's buffers
};

// Reusable per-device scratch.  Grown on demand, never shrunk.
struct Workspace {
    uint8_t* q_u8 = nullptr;     size_t q_u8_bytes = 0;     // [nq][dpad]
    float* q_f32 = nullptr;      size_t q_f32_bytes = 0;    // [nq][dim]
    uint16_t* q_bf16 = nullptr;  size_t q_bf16_bytes = 0;   // [nq][dim] bf16 of q_f32
    int32_t* qn = nullptr;       size_t qn_bytes = 0;       // [nq] |q|^2
    uint32_t* thr_key = nullptr; size_t thr_key_bytes = 0;  // [nq]
    int32_t* thr_id = nullptr;   size_t thr_id_bytes = 0;   // [nq]
    uint32_t* counts = nullptr;  size_t counts_bytes = 0;   // [nq]
    uint2* cand = nullptr;       size_t cand_bytes = 0;     // [nq][cap]
    uint32_t* out_key = nullptr; size_t out_key_bytes = 0;  // [nq][k]
    int32_t* out_id = nullptr;   size_t out_id_bytes = 0;   // [nq][k]
    int32_t* flags = nullptr;    size_t flags_bytes = 0;    // [nq] overflow flags
    int32_t* qlist = nullptr;    size_t qlist_bytes = 0;    // [nq] query index list
    int32_t* status = nullptr;   // [kStatusWords] device status words: [0] scan error, [1] overflowed
                                 // queries, [2..3] u64 final candidates, [4..5] u64 violations,
                                 // [6..11] u64 block-bound counts (tests, unsettled, rows formed),
                                 // [12] chunk-buffer overflow and [13] entry counter of a
                                 // deferred unit scan
    int32_t* h_status = nullptr;                             // pinned mirror
    void* tmp = nullptr;         size_t tmp_bytes = 0;      // CUB / misc scratch
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;               // brackets the full-shard scan
    cudaEvent_t ev_start = nullptr, ev_sel = nullptr;       // first level's start; end of the final selection
    cudaEvent_t ev_rescore = nullptr, ev_prep = nullptr;    // start of the rescore; start of query staging
};
// Fault injection (host side, one shot, mdh_set_fault): the next workspace
// growth reports OOM; the next shard search thread fails before it scans; the
// next IVF search gets a chunk buffer of one block per pass (its deferred
// passes overflow and pass 2 reruns with keys formed in the scan).
enum FaultSite : int { kFaultNone = 0, kFaultOom = 1, kFaultShard = 2, kFaultIvfChunks = 3 };
// True once for an armed site (and disarms it).
bool take_fault(int site);

constexpr int kStatusWords = 16;
constexpr int kStatusBlockStats = 6;   // first word of the three u64 block-bound counters
constexpr int kStatusChunkOverflow = 12;
constexpr int kStatusChunkCounter = 13;  // u32 entry counter of a deferred unit scan

struct Shard {
    int device = 0;
    cudaStream_t stream = nullptr;
    int64_t n = 0;           // rows in this shard
    int64_t id_base = 0;     // global id of the shard's first row
    std::vector<Level> levels;   // ascending size; levels.back() is the whole shard
    Workspace ws;
};

}  // namespace mdh

struct mdh_index {
    int64_t n = 0;
    int32_t dim = 0;
    int32_t dpad = 0;        // u8 row stride (bytes), multiple of kRowAlign
    int32_t metric = MDH_METRIC_L2;
    bool is_f32 = false;     // built from a float corpus
    std::vector<mdh::Shard> shards;
    std::mutex mu;           // one search at a time per index
};

namespace mdh {

// ---- index build (index.cu) ----
// Largest sample of a shard of n rows is about n / g_sample_top_ratio rows
// (process-wide; read when samples are built: index create and load).
constexpr int kSampleTopRatioDefault = 8;
extern int g_sample_top_ratio;
std::vector<int64_t> plan_samples(int64_t n);   // nested sample sizes, ascending
void build_shard_u8(mdh_index* ix, Shard& sh, const uint8_t* host_rows, int64_t n);
void build_shard_f32(mdh_index* ix, Shard& sh, const float* host_rows, int64_t n);
// Device buffers of a level of n rows padded to kTileRows (pad rows: zero
// bytes, kNormPad, id -1); u8 = rows + norms, f32 = float rows + float norms.
void alloc_level(Level& lv, int64_t n, int dpad, int dim, bool u8, bool f32, cudaStream_t st);
// Given sh.levels = {the full level}: adds the nested sample levels and the
// TMA maps, then waits for the shard's stream.
void finish_shard(mdh_index* ix, Shard& sh, bool u8, bool f32);
void free_shard(Shard& sh);
void free_level_buffers(Level& lv);   // frees owned buffers, resets lv
void free_workspace(Workspace& w);    // frees every buffer, resets w

// ---- workspace (capi.cu) ----
void ensure(void** p, size_t* have, size_t need);

// ---- CUDA-core scan kernels (scan_simt.cu) ----
void launch_query_norms_u8(const uint8_t* q, int nq, int dpad, int32_t* qn, cudaStream_t st);
// Append every pair with (key, id) <= per-query threshold to the candidate lists.
// dense = 1: every row is a candidate (infinite threshold, cap >= rows): the
// candidate of row r is written at slot r without atomics and the caller
// sets counts to the row count afterwards.
void launch_filter_simt_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                              const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts,
                              uint2* cand, int cap, int dense, cudaStream_t st);
void launch_filter_simt_u8_cos(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                               const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts,
                               uint2* cand, int cap, int dense, cudaStream_t st);
// Streaming CUDA-core scan for small batches over 128-byte rows
// (scan_stream.cu): mode 0 = L2, 1 = integer cosine.
bool stream_supported(int dpad, const Level& lv);
void launch_scan_stream_u8(const Level& lv, int dpad, int mode, const uint8_t* q, const int32_t* qn, int nq,
                           const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap,
                           int dense, int32_t* status, cudaStream_t st);
// Float replicas of the reference arithmetic (float queries).
void launch_filter_f32(const Level& lv, int dim, int dpad, int score_kind, const float* q, int nq,
                       const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand,
                       int cap, int dense, cudaStream_t st);

// score_kind values for launch_filter_f32
enum ScoreKind : int {
    kScoreL2SqU8 = 0,      // l2_sq_avx over u8 rows (MadhavaL2 L2, float query)
    kScoreCosU8 = 1,       // exact_score cosine over u8 rows (MadhavaL2 cosine, float query)
    kScoreSpeedL2 = 2,     // 2*dot_f32 - |v|^2 over float rows (SpeedEngine L2)
    kScoreSpeedCos = 3,    // dot_f32 over normalized float rows, normalized query (SpeedEngine cosine)
    kScoreExactCosF32 = 4, // exact_score cosine over float rows (MadhavaL2 float corpus, quant none)
};

// ---- tensor-core scan (scan_tc.cu) ----
// TMA map over a row-major 2-D array of u8 (bf16 = 0) or bf16 (bf16 = 1)
// elements, 128-byte swizzle, boxes of box_inner x box_rows elements.
void encode_tmap_2d_sw128(CUtensorMap* map, int bf16, const void* base, uint64_t inner, uint64_t rows,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows);
// TMA map over u8 rows [rows][dpad], 128-byte swizzle, boxes of box_rows rows.
void encode_u8_rows_tmap(CUtensorMap* map, const void* base, int64_t rows, int dpad, int box_rows);
// Corpus chunks per query group for a schedule of groups x chunks units on
// `workers` CTAs; every unit keeps at least min_unit_tiles tiles.
int choose_scan_chunks(int groups, int n_tiles, int workers, int min_unit_tiles);
bool tc_supported(const mdh_index* ix, const Level& lv);
void make_tmap_rows(Level& lv, int dpad);
// One CTA runs the scans' bounded mbarrier wait on a barrier that never
// completes, with `budget` cycles: status[0] gets kDevTimeout when it gives up.
void launch_wait_timeout_probe(long long budget, int32_t* status, cudaStream_t st);
// block_stats (may be null): [0] += bound tests counted by the kernel (unit
// tables only; the schedule form tests every (query, 64-row block)), [1] +=
// tests the bound did not settle, [2] += real rows of those blocks (pairs whose
// exact distance was formed).
// The lists come back holding exact keys.  exact = 0: they hold every row the
// block bound could not exclude (a superset of the rows at or under the
// threshold; keys are formed by a pass after the scan).  exact = 1 (overflow
// reruns): only the rows at or under the threshold.
void launch_filter_tc_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                            const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts,
                            uint2* cand, int cap, int dense, int32_t* status, unsigned long long* block_stats,
                            int exact, cudaStream_t st);
// Unit-table form of the tensor-core scan (used by the IVF search, ivf.cu):
// unit u scans query rows [q_row, q_row + q_count) of `qmat` (row i is query
// qmap[i]; thresholds, norms and candidate lists are indexed by that query)
// against corpus tiles [t0, t1) of 256 rows, rows at or past row_end masked.
// n_units bounds the table (it sizes the grid); when n_units_dev is given the
// kernel reads the table's length from it (tables built on the device).  When
// unit_counter is given (one int of device memory, reset by the launch), the
// CTAs take units in table order as each finishes its previous one, instead
// of fixed shares.
struct ScanUnit {
    int32_t q_row;
    int32_t q_count;   // <= 128
    int32_t t0, t1;
    int32_t row_end;
    int32_t pad;
};
// Passing chunks of a deferred unit scan: entry e holds the 32 dot products
// of one (query, 32-row chunk) whose block bound could not settle it
// (x[8e .. 8e+8) as u32 x 32) and hdr[e] = {query, first row position, valid
// rows, 0}.  CTAs' warps take 64-entry blocks from *counter; capacity is a
// multiple of 64, and a block past it is dropped and flags
// status[kStatusChunkOverflow].  nq: the number of candidate lists (query
// indices in the entries are below it).
struct ChunkOut {
    uint4* x = nullptr;
    int4* hdr = nullptr;
    uint32_t* counter = nullptr;
    uint32_t capacity = 0;
    int32_t nq = 0;
};
constexpr int kChunkBlock = 64;
// With `defer` null the scan forms exact keys in its epilogue (the form the
// overflow reruns use).  With it, the scan writes the passing chunks to
// *defer and a re-key pass (k_rekey_chunks) forms the same candidates:
// every row of those chunks with (key, id) <= the query's threshold.
void launch_filter_tc_u8_l2_units(const Level& lv, int dpad, const uint8_t* qmat, int qmat_rows, const int32_t* qmap,
                                  const int32_t* qn, const ScanUnit* units, int n_units, const int32_t* n_units_dev,
                                  int32_t* unit_counter, const uint32_t* thr_key, const int32_t* thr_id,
                                  uint32_t* counts, uint2* cand, int cap, int32_t* status,
                                  unsigned long long* block_stats, const ChunkOut* defer, cudaStream_t st);
// ---- tensor-core scan on SM pairs (scan_tc2.cu) ----
bool tc2_supported(const mdh_index* ix, const Level& lv);
void make_tmap_rows_pair(Level& lv, int dpad);
void launch_filter_tc2_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                             const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts,
                             uint2* cand, int cap, int dense, int32_t* status, cudaStream_t st);

// ---- approximate bf16 tensor-core scan for float cosine scores (scan_tc_bf16.cu) ----
// Every row whose bf16 score is >= T - eps (T = the query's threshold score)
// is appended with its row position; launch_rescore_speed_cos then replaces
// the candidates' keys by the exact float score of the reference.
bool tc_bf16_supported(const mdh_index* ix, const Level& lv);
void ensure_bf16_rows(mdh_index* ix, Shard& sh);
void launch_convert_bf16(const float* src, int64_t count, uint16_t* dst, cudaStream_t st);
// Dense bf16 lists: keep only rows within two_eps of each list's k-th bf16
// score (thr_key), the only rows that can be in the exact top k.
void launch_compact_bf16_band(uint32_t* counts, uint2* cand, int cap, const uint32_t* thr_key, float two_eps, int nq,
                              cudaStream_t st);
void launch_filter_tc_bf16_cos(const Level& lv, int dim, const uint16_t* q_bf16, int nq, const uint32_t* thr_key,
                               uint32_t* counts, uint2* cand, int cap, int dense, float eps, int32_t* status,
                               cudaStream_t st);
// SpeedEngine cosine query normalization in place ([nq][dim] fp32, the
// reference's arithmetic; batch_guard: search_batch's |q|^2 > 1e-12 test),
// plus the bf16 copy when q_bf16 is not null.
void launch_normalize_speed_cos(float* q, int nq, int dim, int batch_guard, uint16_t* q_bf16, cudaStream_t st);
void launch_rescore_speed_cos(const uint32_t* counts, uint2* cand, int cap, const float* rows_f32, int dim,
                              const float* q_f32, int nq, cudaStream_t st);

// ---- selection (select.cu) ----
void launch_fill_threshold(uint32_t* thr_key, int32_t* thr_id, int nq, uint32_t key, int32_t id,
                           cudaStream_t st);
// final == 0: write the k-th smallest stored (key, id) per query into thr.
// final == 1: write the sorted top-k to out_key/out_id; set flags[q] = 1 and
//             thr[q] when the candidate list overflowed (result not final).
void launch_fill_u32(uint32_t* p, int n, uint32_t v, cudaStream_t st);
// Candidates hold {key, row position in the scanned level}; ids maps positions to global ids.
void launch_select(const uint32_t* counts, const uint2* cand, int cap, const int32_t* ids, int nq, int k, int final_,
                   uint32_t* thr_key, int32_t* thr_id, uint32_t* out_key, int32_t* out_id,
                   int32_t* flags, int32_t* n_flagged, const int32_t* qmap, unsigned long long* n_cand,
                   cudaStream_t st);
// thr[q] = the k-th entry (key, id) of list q of [nq][k] (key, id) lists,
// or infinity when that entry is empty (id -1).
void launch_thresholds_from_lists(const uint32_t* keys, const int32_t* ids, int nq, int k, uint32_t* thr_key,
                                  int32_t* thr_id, cudaStream_t st);
// Verification of results (capi.cu, search with verification on).
void launch_verify_thresholds(const int32_t* list, int m, const uint32_t* out_key, const int32_t* out_id, int k, int kk,
                              uint32_t* thr_key, int32_t* thr_id, cudaStream_t st);
void launch_count_violations(const uint32_t* counts, int m, int kk, unsigned long long* violations, cudaStream_t st);
void launch_merge_topk(const uint32_t* key_all, const int32_t* id_all, int nshard, int nq, int k,
                       uint32_t* key_out, int32_t* id_out, cudaStream_t st);
// Float query rows [nq][dim] + [nq] aux -> the listed m rows, same layout.
void launch_gather_queries_f32(const float* src, int nq, int dim, const int32_t* list, int m, float* dst,
                               cudaStream_t st);
void launch_gather_queries_u8(const uint8_t* src, const int32_t* qn_src, const int32_t* list, int m,
                              int dpad, uint8_t* dst, int32_t* qn_dst, cudaStream_t st);

int device_sm_count(int dev);
// Throws unless `dev` is a visible sm_100 device.
void check_device_usable(int dev);

// Runs fn(ctx) under the C ABI's error convention (status code, and the
// message for mdh_last_error) without allocating on success.
mdh_status run_guarded(void (*fn)(void*), void* ctx);

}  // namespace mdh
