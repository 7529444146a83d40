/*
 * winnex_madhava_b200.h -- C ABI of the B200 exact top-K scan library
 * (libwinnex_madhava_b200.so).
 *
 * Plain C: pointers, sizes and status codes only.  Every entry point returns
 * an mdh_status; on failure mdh_last_error() holds a message for the calling
 * thread.  There is no CPU fallback: without a usable sm_100 GPU every search
 * entry point fails with MDH_ERR_CUDA.
 *
 * Each declaration names the reference interface it replaces
 * (winnex-madhava, paths relative to that project).
 *
 * Result convention (all searches): out_ids[q*k + j], j < min(k, n), is the
 * j-th best corpus row for query q; rows past min(k, n) are -1.  L2 results
 * ascend by (squared distance, row id): the lower id wins a tie, as in
 * MadhavaL2::search_exact's pair<float,int> partial_sort
 * (src/winnex_madhava.cpp:1237-1239).  Score results (cosine / inner product)
 * descend by score with the same lower-id tie break.
 */
#ifndef WINNEX_MADHAVA_B200_H
#define WINNEX_MADHAVA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    MDH_OK = 0,
    MDH_ERR_INVALID_ARG = 1,   /* bad pointer / size / shape */
    MDH_ERR_CUDA = 2,          /* CUDA runtime error, or no usable GPU */
    MDH_ERR_NCCL = 3,          /* collective failure (multi-device merge) */
    MDH_ERR_OOM = 4,           /* device allocation failed */
    MDH_ERR_TIMEOUT = 5,       /* a bounded device-side wait expired */
    MDH_ERR_NOT_INTEGRAL = 6,  /* an integer-only entry point got non-integral data */
    MDH_ERR_UNSUPPORTED = 7,   /* valid request outside what this build implements */
    MDH_ERR_INTERNAL = 8,
    MDH_ERR_IO = 9             /* index file: cannot open / read / write, bad header, truncated,
                                  or rows that fail the load-time integrity check */
} mdh_status;

/* Metric values match the reference enum (include/winnex_madhava/winnex_madhava.hpp:38-41). */
typedef enum { MDH_METRIC_COSINE = 0, MDH_METRIC_L2 = 1 } mdh_metric;

/* Score semantics of a float query -- which reference formula the float
 * arithmetic reproduces when the query is not a u8 vector.
 *   MDH_SCORE_EXACT: MadhavaL2::exact_score (src/winnex_madhava.cpp:710-763):
 *                    L2 = l2_sq_avx, cosine = dot / sqrt(|v|^2 |q|^2).
 *   MDH_SCORE_SPEED: SpeedEngine::search (src/speed_cpu.cpp:271-353): score =
 *                    2*dot_f32 - |v|^2 (L2) or dot of normalized vectors.
 *   MDH_SCORE_SPEED_BATCH: SpeedEngine::search_batch (src/speed_cpu.cpp:356-398),
 *                    identical except the cosine query-normalization guard
 *                    (|q|^2 > 1e-12 instead of |q| > 1e-12). */
typedef enum { MDH_SCORE_EXACT = 0, MDH_SCORE_SPEED = 1, MDH_SCORE_SPEED_BATCH = 2 } mdh_score_mode;

typedef struct mdh_index mdh_index;

/* Per-call statistics; maps onto SearchResult / SpeedResult fields
 * (include/winnex_madhava/winnex_madhava.hpp:118-164, speed_engine.hpp:36-41). */
typedef struct {
    double latency_ms;            /* host wall time of the call (SearchResult::latency_ms) */
    int64_t pairs_scored;         /* (query, row) pairs scanned, every level (bound_pairs) */
    int64_t pairs_pruned_by_bound;/* scanned pairs the tensor scan's block bound excluded without forming their
                                     distance: the block's smallest |v|^2 and largest q.v prove every key in it
                                     above the query's threshold (SearchResult::pruned_by_bound); the rest,
                                     pairs_scored - pairs_pruned_by_bound, had their exact distance formed
                                     (SearchResult::exact_evals).  0 on the CUDA-core and bf16 paths, which
                                     form every distance */
    int64_t bound_violations;     /* rows misplaced relative to the returned top-K, counted for the
                                     verified queries by an exact unpruned scan (mdh_set_verify); 0 */
    int64_t candidates;           /* pairs that passed the threshold filter into the final selection */
    int32_t tensor_core_path;     /* full-corpus scan: 0 CUDA cores, 1 tcgen05 per SM, 2 tcgen05 on SM pairs,
                                     3 bf16 tcgen05 pass + exact fp32 rescore (float cosine scores) */
    int32_t levels;               /* threshold-refinement levels run */
    double full_scan_ms;          /* CUDA-event time of the full-corpus scan kernel(s) on their stream */
    int64_t full_scan_pairs;      /* (query, row) pairs that kernel scored */
    int64_t kernel_launches;      /* this library's kernels launched by the call */
    int64_t verified_queries;     /* queries re-checked by the verification scan (mdh_set_verify) */
    /* Stage times, CUDA events on the search's stream (slowest shard per query chunk, summed over chunks): */
    double sample_ms;             /* sample levels: their scans and threshold selections */
    double select_ms;             /* final selection of the full level, overflow reruns included */
    double rescore_ms;            /* exact fp32 rescore of the bf16 pass's candidates (float cosine); also
                                     inside full_scan_ms */
    double prep_ms;               /* query staging: host conversion and padding (wall time) plus the upload
                                     and |q|^2 on the stream (events) */
    int64_t blocks_tested;        /* (query, row block) bound tests of the 1-SM tensor scan, every level */
    int64_t blocks_passed;        /* tests the bound did not settle; their rows' distances were formed */
} mdh_stats;

/* Build an index over a row-major u8 corpus [n][dim] held in host memory.
 * The library copies the corpus into device memory (norm-sorted rows, integer
 * |v|^2, row ids) and does not keep the host pointer.
 * devices/ndev: GPUs to shard rows over (contiguous id ranges); NULL/0 = the
 * current device.  id_offset is added to every returned row id (a rank that
 * holds rows [off, off+n) of a larger corpus passes off).
 * Replaces SpeedEngine::SpeedEngine(const uint8_t*, ...) (src/speed_cpu.cpp:117-144)
 * and MadhavaL2::build (src/winnex_madhava.cpp:487), bound via
 * bindings/py_module.cpp:98-107 and :303-313. */
mdh_status mdh_index_create_u8(const uint8_t* host_corpus, int64_t n, int32_t dim, int32_t metric,
                               const int32_t* devices, int32_t ndev, int64_t id_offset,
                               mdh_index** out);

/* Build from a row-major float32 corpus [n][dim].  Replaces
 * SpeedEngine::SpeedEngine(const float*, ...) (src/speed_cpu.cpp:81-115):
 * cosine rows are normalized with the reference's arithmetic. */
mdh_status mdh_index_create_f32(const float* host_corpus, int64_t n, int32_t dim, int32_t metric,
                                const int32_t* devices, int32_t ndev, int64_t id_offset,
                                mdh_index** out);

/* Build a single-device index from a u8 corpus [n][dim] already in device
 * memory on the current device (e.g. a tensor produced on the GPU).  Same
 * layout and semantics as mdh_index_create_u8; the device buffer is copied
 * and may be freed afterwards.  No counterpart in the reference (its corpus
 * always starts on the host). */
mdh_status mdh_index_create_u8_device(const uint8_t* dev_corpus, int64_t n, int32_t dim, int32_t metric,
                                      int64_t id_offset, mdh_index** out);

mdh_status mdh_index_destroy(mdh_index* index);

/* Shape of an index. */
mdh_status mdh_index_info(const mdh_index* index, int64_t* n, int32_t* dim, int32_t* metric,
                          int32_t* ndev);

/* Device memory an index holds (host only; no GPU work): level_bytes for its
 * rows, norms and ids (samples included), workspace_bytes for the per-device
 * scratch that searches grow on demand and keep (query staging, thresholds,
 * candidate lists, results).  Either output may be NULL.  No counterpart in
 * the reference. */
mdh_status mdh_index_memory(const mdh_index* index, int64_t* level_bytes, int64_t* workspace_bytes);

/* First global row id of an index: its rows carry ids [first_id, first_id + n)
 * (the id_offset it was built with, or the first id of the file it was loaded
 * from).  No counterpart in the reference (its ids always start at 0). */
mdh_status mdh_index_id_base(const mdh_index* index, int64_t* first_id);

/* Index files.  A file holds, per shard, the norm-sorted rows with their
 * padded stride, the integer |v|^2 and the global row ids (float corpora:
 * float rows, float norms, ids), behind a fixed little-endian header:
 *   0  char[8] "MDHB200I"   8  u32 version (1)   12 u32 kind (0 u8, 1 float32)
 *   16 i64 n   24 i32 dim   28 i32 row stride (u8: dim rounded up to 128
 *   bytes; float32: dim)   32 i32 metric   36 i32 shards   40 u64 data offset
 *   48 u64 file size   56 u64 0;  64: shards x {i64 rows, i64 id_base,
 *   u64 offset, u64 bytes};  each shard's data at its 4096-aligned offset:
 *   rows [rows][stride], norms [rows] (4 bytes), ids [rows] (int32).
 * The shards' id ranges tile one run [first id, first id + n) in file order.
 * Loading skips the sort: it streams each shard to its GPU, checks every row
 * against its stored norm and order, and that the shard's ids are a
 * permutation of its id range, on the device, and rebuilds
 * the sample levels (they are chosen by a hash of the row id, so they come
 * out the same).  Search results after a load equal those before the save.
 *
 * mdh_index_save writes `path` through a temporary file renamed into place.
 * Replaces MadhavaL2::save_index (src/winnex_madhava.cpp:1120-1149, bound at
 * bindings/py_module.cpp:227-230); the reference file holds the bound
 * engine's projections and leaves the corpus out, this one holds the corpus
 * in the order the scan reads it. */
mdh_status mdh_index_save(mdh_index* index, const char* path);

/* devices/ndev: one GPU per shard of the file, in file order; NULL/0 = every
 * shard on the current device.  Replaces MadhavaL2::load_index
 * (src/winnex_madhava.cpp:1151-1217, bound at bindings/py_module.cpp:232-235). */
mdh_status mdh_index_load(const char* path, const int32_t* devices, int32_t ndev, mdh_index** out);

/* Header of an index file (host only; no GPU needed).  Any output may be NULL.
 * is_float: 1 for a float32 corpus. */
mdh_status mdh_index_file_info(const char* path, int64_t* n, int32_t* dim, int32_t* metric, int32_t* shards,
                               int32_t* is_float);

/* Search with float32 host queries [nq][dim]; results to host buffers.
 * A query whose values are all integers in [0,255] runs the integer u8 path
 * (exact for every mode); other queries run float arithmetic that reproduces
 * the reference formula selected by `mode`.
 * out_dist (may be NULL) receives the value the ranking used: the squared L2
 * distance (MDH_SCORE_EXACT, L2), the cosine score (cosine metrics), or the
 * SpeedEngine score 2*dot - |v|^2 (MDH_SCORE_SPEED* on float arithmetic).
 * Replaces MadhavaL2::search_exact / search / search_batch
 * (src/winnex_madhava.cpp:1219-1246, :766, :1094; py_module.cpp:136-151, :219-226)
 * and SpeedEngine::search / search_batch (src/speed_cpu.cpp:425-449;
 * py_module.cpp:314-335). */
mdh_status mdh_search_f32(mdh_index* index, const float* host_queries, int32_t nq, int32_t k,
                          int32_t mode, int32_t* out_ids, float* out_dist, mdh_stats* stats);

/* Search with u8 host queries [nq][dim] (the integer path only).
 * out_dist: exact squared L2 distance (int32) for L2; NULL allowed. */
mdh_status mdh_search_u8(mdh_index* index, const uint8_t* host_queries, int32_t nq, int32_t k,
                         int32_t* out_ids, int32_t* out_dist, mdh_stats* stats);

/* Audited search: replaces MadhavaL2::search_audited / audit_json /
 * search_with_commitment (src/winnex_madhava.cpp:1258-1591,
 * include/winnex_madhava/winnex_madhava.hpp:172-234).  The reference
 * certifies its Stage-1 projection bound; this engine is exact, so the audit
 * certifies the exact top k against a second GPU pass over every row with
 * the final threshold.  Per query:
 *   threshold          the k-th result's distance (L2) or score (cosine);
 *   within             rows whose (exact) key is at or within the threshold:
 *                      the k results and rows tied with the k-th;
 *   excluded           rows - within: rows strictly worse than the k-th
 *                      result, i.e. provably outside the top k (the
 *                      reference's audit_excluded / total_excluded_count);
 *   excluded_by_bound  of those, the rows the 64-row block bound of the
 *                      tensor-core scan settled without a key (-1 when the
 *                      scan path has no block bound);
 *   violations         max(0, k - within): 0 for a correct result;
 *   n_records          the excluded rows nearest the threshold written to
 *                      rec_ids / rec values (ascending key, then id; at most
 *                      max_records), the deterministic sample of the
 *                      commitment; fewer only when more than 2^18 rows tie
 *                      with the k-th result.
 * Queries run one at a time.  mdh_audit_f32 ranks by MDH_SCORE_EXACT. */
typedef struct mdh_audit {
    int64_t rows;
    int64_t within;
    int64_t excluded;
    int64_t excluded_by_bound;
    int64_t violations;
    double threshold;
    int32_t n_records;
    int32_t reserved;
} mdh_audit;

mdh_status mdh_audit_f32(mdh_index* index, const float* host_queries, int32_t nq, int32_t k, int32_t max_records,
                         int32_t* out_ids, float* out_values, int32_t* rec_ids, float* rec_values,
                         mdh_audit* audit, mdh_stats* stats);
mdh_status mdh_audit_u8(mdh_index* index, const uint8_t* host_queries, int32_t nq, int32_t k, int32_t max_records,
                        int32_t* out_ids, int32_t* out_dist, int32_t* rec_ids, int32_t* rec_dist,
                        mdh_audit* audit, mdh_stats* stats);

/* Device-resident variant of mdh_search_u8 for a single-device index:
 * queries, ids and distances are device pointers on the index's device;
 * work is enqueued on `stream` (a cudaStream_t, NULL = the index's stream)
 * and the call returns after the results are written (stream synchronized).
 * No counterpart in the reference (its GPU path always copies from the host,
 * src/speed_gpu.cu:194-227); used for HBM-resident throughput measurement. */
mdh_status mdh_search_u8_device(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                int32_t* dev_ids, int32_t* dev_dist, void* stream, mdh_stats* stats);

/* Cooperative thresholds for a corpus sharded over ranks (one index per rank,
 * global row ids).  Phase 1, mdh_search_u8_device_sample, scans only this
 * shard's sample levels and writes each query's exact top-k (distance, id) of
 * the largest sample scanned ([nq][k], id -1 past its rows).  The ranks
 * exchange these lists (all_gather) and merge them (mdh_merge_topk_device):
 * the merged list's k-th entry is the k-th best of the union of every rank's
 * sample, a valid distance threshold for the whole corpus and tighter than
 * any one rank's own.  Phase 2, mdh_search_u8_device_bounded, takes the merged
 * lists (dev_thr_dist / dev_thr_ids, [nq][k]) and scans the full shard under
 * that threshold: its results are the exact top-k among this shard's rows at
 * or under it (-1 past them).  Merging the ranks' phase-2 lists gives the
 * exact global top-k.  A rank's sample then only needs 1/G of the rows that
 * one rank alone would need for the same threshold, G = the number of ranks.
 * Single-device indexes; device pointers and stream as mdh_search_u8_device.
 * No counterpart in the reference (it has no multi-GPU path,
 * src/speed_gpu.cu:113-117). */
mdh_status mdh_search_u8_device_sample(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                       int32_t* dev_ids, int32_t* dev_dist, void* stream, mdh_stats* stats);
mdh_status mdh_search_u8_device_bounded(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                        const int32_t* dev_thr_dist, const int32_t* dev_thr_ids, int32_t* dev_ids,
                                        int32_t* dev_dist, void* stream, mdh_stats* stats);

/* mdh_search_u8_device without any allocation: no cudaMalloc / cudaFree
 * or allocating library call; scratch is a fixed 9 MiB __device__ array per
 * device.  For callers that must not allocate (a serving loop beside a
 * caching allocator that holds most of HBM; a latency-bound loop where
 * cudaFree would synchronize the device).  Limits: L2 index on one device,
 * dim <= 256, nq <= 256, k <= 256 (MDH_ERR_UNSUPPORTED beyond).  The first
 * call on a device resolves the scratch address (cudaGetSymbolAddress): make
 * it before any stream capture.  Calls share the scratch, so they are
 * serialized by a process-wide lock; each returns after its work on `stream`
 * completed.  No counterpart in the reference. */
mdh_status mdh_search_u8_device_noalloc(mdh_index* index, const uint8_t* dev_queries, int32_t nq, int32_t k,
                                        int32_t* dev_ids, int32_t* dev_dist, void* stream, mdh_stats* stats);

/* Merge per-shard top-k lists (device pointers on the current device):
 * dist_all/ids_all are [nshard][nq][k] (int32 squared distance, int32 row id,
 * id -1 = empty), the output [nq][k] keeps the k smallest (dist, id).
 * The exchange step of the row-sharded multi-GPU scan. */
mdh_status mdh_merge_topk_device(const int32_t* dev_dist_all, const int32_t* dev_ids_all, int32_t nshard,
                                 int32_t nq, int32_t k, int32_t* dev_dist_out, int32_t* dev_ids_out,
                                 void* stream);

/* ---------------------------------------------------------------- IVF
 * Clustered index over a u8 corpus: the GPU form of MadHybrid's uint8 path
 * (python/winnex_madhava/__init__.py:547-654).  The caller supplies the
 * cells: centroids [nlist][dim] float32 and one label per row (the reference
 * computes them with MiniBatchKMeans, __init__.py:577-593).  A query goes to
 * the nprobe cells with the largest centroid inner product (the reference's
 * `centroids @ q`, :631-632; here in fp64, ties to the lower cell id) and the
 * result is the exact top-k over the union of those cells: by (squared L2
 * distance, row id) for metric L2, or by (inner product q.v descending, row
 * id) for metric COSINE -- the ranking MadHybrid's merge uses for a u8 corpus
 * under metric "cosine", `corpus[ids].astype(float32) @ q` (:640-646), which
 * is exact in integers for u8 rows and integral queries.  dim <= 128,
 * nlist <= 8192, nprobe <= 1024, k <= 4096. */
typedef struct mdh_ivf mdh_ivf;

/* device: GPU ordinal, -1 = the current device.  Row ids are 0..n-1.
 * metric: MDH_METRIC_L2 or MDH_METRIC_COSINE (inner-product ranking, above).
 * Replaces MadHybrid.__init__'s per-cell engines (__init__.py:600-608). */
mdh_status mdh_ivf_create_u8_metric(const uint8_t* host_corpus, int64_t n, int32_t dim, const float* centroids,
                                    int32_t nlist, const int32_t* labels, int32_t metric, int32_t device,
                                    mdh_ivf** out);
/* mdh_ivf_create_u8_metric with MDH_METRIC_L2. */
mdh_status mdh_ivf_create_u8(const uint8_t* host_corpus, int64_t n, int32_t dim, const float* centroids,
                             int32_t nlist, const int32_t* labels, int32_t device, mdh_ivf** out);
/* out_cells [nq][nprobe]: the cells each query probes, best first. */
mdh_status mdh_ivf_route_u8(mdh_ivf* index, const uint8_t* host_queries, int32_t nq, int32_t nprobe,
                            int32_t* out_cells);
/* u8 host queries [nq][dim]; out_ids / out_dist [nq][k] (NULL allowed; the
 * exact squared L2 distance, or the exact inner product for metric COSINE),
 * -1 past the rows of the probed cells.  Replaces MadHybrid.search
 * (__init__.py:625-654). */
mdh_status mdh_ivf_search_u8(mdh_ivf* index, const uint8_t* host_queries, int32_t nq, int32_t k, int32_t nprobe,
                             int32_t* out_ids, int32_t* out_dist, mdh_stats* stats);
/* cell_rows (NULL allowed): [nlist] rows per cell. */
mdh_status mdh_ivf_info(const mdh_ivf* index, int64_t* n, int32_t* dim, int32_t* nlist, int64_t* cell_rows);
mdh_status mdh_ivf_destroy(mdh_ivf* index);

/* Clustered search over a float32 corpus: replaces MadHybrid's float path
 * (python/winnex_madhava/__init__.py:547-654: routing `centroids @ q` at
 * :631-632, per-cell float64 scores `vecs @ q` at :526, merge by score at
 * :650).  Every row of the probed cells is scored, so the result is the
 * exact top k of their union by (float64 inner product descending, row id
 * ascending); routing and scores are fp64 with one fused multiply-add per
 * dimension in dimension order.  labels[i] in [0, nlist) is row i's cell;
 * dim <= 4096; k in [1, 16] (MDH_ERR_UNSUPPORTED above); out_scores may be
 * null.  Rows past the probed cells' total come back as id -1. */
typedef struct mdh_ivf_f32 mdh_ivf_f32;
mdh_status mdh_ivf_create_f32(const float* host_rows, int64_t n, int32_t dim, const float* centroids, int32_t nlist,
                              const int32_t* labels, int32_t device, mdh_ivf_f32** out);
mdh_status mdh_ivf_search_f32(mdh_ivf_f32* index, const float* host_queries, int32_t nq, int32_t k, int32_t nprobe,
                              int32_t* out_ids, double* out_scores, mdh_stats* stats);
mdh_status mdh_ivf_destroy_f32(mdh_ivf_f32* index);

/* Options (process-wide): force the scan path for testing and measurement.
 * path: 0 = automatic, 1 = CUDA-core scan only, 2 = tensor-core scan on
 * single SMs, 3 = tensor-core scan on SM pairs (each whenever the shape
 * allows; otherwise the CUDA-core scan). */
mdh_status mdh_set_scan_path(int32_t path);

/* Options (process-wide): verification.  max_queries > 0 makes every u8
 * integer search re-check up to that many of its queries (spread evenly over
 * the batch) with an exact CUDA-core scan that prunes nothing: it counts the
 * rows at or before each query's k-th result by (distance, id), and any count
 * other than k adds to mdh_stats.bound_violations.  0 = off (default).  The
 * reference declares bound_violations but never measures it
 * (include/winnex_madhava/winnex_madhava.hpp:125). */
mdh_status mdh_set_verify(int32_t max_queries);

/* Options (process-wide): upper bound on a query's candidate list length
 * (a power of two in [64, 16384]; 0 = automatic).  A list that overflows is
 * rerun with a strictly tighter threshold, so results stay exact; small
 * limits trade speed for scratch memory and exercise that rerun path. */
mdh_status mdh_set_candidate_cap_limit(int32_t cap);

/* Failure handling, exercised without a device fault.
 * mdh_set_fault(site): a one-shot host-side fault for tests.  site 1: the
 * next growth of a search workspace fails as out of memory (MDH_ERR_OOM);
 * site 2: the next shard search thread fails before it scans
 * (MDH_ERR_INTERNAL); site 3: the next IVF search gets a one-block chunk
 * buffer, so its deferred scans overflow it and pass 2 reruns with keys
 * formed in the scan (the results stay exact).  0 clears it.  The index
 * stays usable afterwards.
 * mdh_check_wait_timeout(device, budget_cycles): runs the scans' bounded
 * mbarrier wait on a barrier that nothing arrives on, with a budget of
 * budget_cycles (1,000 .. 2^32 clock cycles; the scans use ~4e9): it must
 * give up and record the timeout, and the call returns MDH_ERR_TIMEOUT; any
 * other status means the timeout path is broken.  device -1 = current.
 * No counterpart in the reference. */
mdh_status mdh_set_fault(int32_t site);
mdh_status mdh_check_wait_timeout(int32_t device, int64_t budget_cycles);

/* Options (process-wide): sample plan.  An index shard of n rows keeps
 * nested random samples of 1024 * 4^j rows up to n / ratio rows (default
 * ratio 8; 0 restores it).  Read when samples are built (index create and
 * load).  A search scans a chain of them, smallest first, to set each
 * query's distance threshold: the chain is the cheapest under a measured
 * cost model (a level costs its rows plus a fixed overhead, and a level
 * keeps about k * (its rows / the previous level's) candidates per query,
 * each costing ~4,500 row scans), so its largest sample is about
 * sqrt(4,500 k n) rows.
 * mdh_set_threshold_sharing(ranks): the full level's threshold comes from the
 * union of `ranks` ranks' samples (mdh_search_u8_device_sample), so the
 * chain's last step expects `ranks` times fewer candidates and stops at a
 * smaller sample.  1 (default) for a shard searched alone.  Read at search. */
mdh_status mdh_set_threshold_sharing(int32_t ranks);
mdh_status mdh_set_sample_ratio(int32_t ratio);

/* Levels (samples, then the whole shard) a top-k search scans on one shard
 * of shard_rows rows with the current sample plan, from the nominal sample
 * sizes (host only; no GPU needed).  0 for an empty request, -1 when k is
 * beyond what the selector supports for that shard. */
int32_t mdh_plan_level_count(int64_t shard_rows, int32_t k);

/* Number of CUDA devices visible (0 when none). */
int32_t mdh_device_count(void);

/* Message of the last failed call on this thread ("" if none). */
const char* mdh_last_error(void);

/* Library version string. */
const char* mdh_version(void);

#ifdef __cplusplus
}
#endif

#endif /* WINNEX_MADHAVA_B200_H */
