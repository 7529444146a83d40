/*
 * Oracle for the exact top-K scan -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is a plain-C restatement of the reference's CPU exact-scan
 * arithmetic (winnex-madhava, src/winnex_madhava.cpp and src/speed_cpu.cpp).
 * It exists so the test suite, the smoke check and the bench's cpu_baseline
 * leg have an independent checker.  Nothing in the product links it or calls
 * it: the CUDA library in winnex-madhava_b200/ never falls back to this code.
 *
 * Every function below names the reference lines it restates.  The float
 * arithmetic follows the reference's evaluation order exactly (8 FMA lanes,
 * then a left-to-right lane sum), so for float queries the oracle's distances
 * are bit-identical to the reference built with -O3 -mavx2 -mfma.  For u8
 * corpora with integral queries every intermediate value is an integer below
 * 2^24, so the result is exact and independent of evaluation order.
 *
 * Ranking rules:
 *   L2 (MadhavaL2::search_exact):   ascending (distance, index) -- the
 *       reference sorts std::pair<float,int>, so ties go to the lower index
 *       (src/winnex_madhava.cpp:1237-1239).
 *   score metrics (SpeedEngine, cosine): descending score; the reference's
 *       comparator looks at the score only, leaving tie order unspecified
 *       (src/speed_cpu.cpp:346-347).  The oracle breaks those ties by the
 *       lower index, which is one of the orders the reference may produce.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Distance / score kernels (one corpus row against one float query).        */
/* ------------------------------------------------------------------------ */

/* l2_sq_avx, src/winnex_madhava.cpp:119-146: 16 bytes per step, split into a
 * low and a high group of 8; lane l accumulates fma(d[j+l]^2) then
 * fma(d[j+8+l]^2); the 8 lanes are summed left to right; scalar tail. */
float oracle_l2_sq_u8(const uint8_t* v, const float* q, int d) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j + 16 <= d; j += 16) {
        for (int l = 0; l < 8; l++) {
            float dl = (float)v[j + l] - q[j + l];
            lane[l] = fmaf(dl, dl, lane[l]);
        }
        for (int l = 0; l < 8; l++) {
            float dh = (float)v[j + 8 + l] - q[j + 8 + l];
            lane[l] = fmaf(dh, dh, lane[l]);
        }
    }
    float r = lane[0] + lane[1] + lane[2] + lane[3] + lane[4] + lane[5] + lane[6] + lane[7];
    for (; j < d; j++) {
        float dd = (float)v[j] - q[j];
        r = fmaf(dd, dd, r); /* g++ contracts `r += dd*dd` under -mfma */
    }
    return r;
}

/* dot_f32, src/speed_cpu.cpp:60-76: 8 FMA lanes over steps of 8, lanes summed
 * left to right, scalar tail. */
float oracle_dot_f32(const float* a, const float* b, int d) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= d; i += 8)
        for (int l = 0; l < 8; l++) lane[l] = fmaf(a[i + l], b[i + l], lane[l]);
    float r = lane[0] + lane[1] + lane[2] + lane[3] + lane[4] + lane[5] + lane[6] + lane[7];
    for (; i < d; i++) r = fmaf(a[i], b[i], r);
    return r;
}

/* exact_score cosine over a u8 row, src/winnex_madhava.cpp:714-763 (the
 * base_ branch, taken whenever corpus_f32_ is null or quant != None).  dot
 * and |v|^2 use the same 16-byte lane split as l2_sq_avx; |q|^2 is a scalar
 * loop; score = dot / sqrt(|v|^2 * |q|^2), or 0 when that is <= 1e-10. */
float oracle_cosine_u8(const uint8_t* v, const float* q, int d, float qn2) {
    float sd[8] = {0, 0, 0, 0, 0, 0, 0, 0}, sv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j + 16 <= d; j += 16) {
        for (int l = 0; l < 8; l++) {
            float f = (float)v[j + l];
            sd[l] = fmaf(f, q[j + l], sd[l]);
        }
        for (int l = 0; l < 8; l++) {
            float f = (float)v[j + 8 + l];
            sd[l] = fmaf(f, q[j + 8 + l], sd[l]);
        }
        for (int l = 0; l < 8; l++) {
            float f = (float)v[j + l];
            sv[l] = fmaf(f, f, sv[l]);
        }
        for (int l = 0; l < 8; l++) {
            float f = (float)v[j + 8 + l];
            sv[l] = fmaf(f, f, sv[l]);
        }
    }
    float dot = 0.0f, vn2 = 0.0f;
    for (int l = 0; l < 8; l++) { dot += sd[l]; vn2 += sv[l]; }
    for (; j < d; j++) {
        float f = (float)v[j];
        dot = fmaf(f, q[j], dot);
        vn2 = fmaf(f, f, vn2);
    }
    float denom = sqrtf(vn2 * qn2);
    return denom > 1e-10f ? dot / denom : 0.0f;
}

/* |q|^2 scalar loop used by the cosine score (src/winnex_madhava.cpp:759). */
float oracle_qn2(const float* q, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; j++) s = fmaf(q[j], q[j], s);
    return s;
}

/* ------------------------------------------------------------------------ */
/* Top-k selection helpers.                                                  */
/* ------------------------------------------------------------------------ */

typedef struct { float key; int32_t id; } kv_t;

/* "a ranks before b": ascending key, then ascending id. */
static int kv_before_asc(kv_t a, kv_t b) {
    return a.key < b.key || (a.key == b.key && a.id < b.id);
}

/* Bounded max-heap keeping the k best (smallest under kv_before_asc). */
static void heap_push_asc(kv_t* h, int* size, int k, kv_t x) {
    if (*size < k) {
        int i = (*size)++;
        h[i] = x;
        while (i > 0) {
            int p = (i - 1) / 2;
            if (kv_before_asc(h[p], h[i])) { kv_t t = h[p]; h[p] = h[i]; h[i] = t; i = p; }
            else break;
        }
        return;
    }
    if (!kv_before_asc(x, h[0])) return;
    h[0] = x;
    int i = 0;
    for (;;) {
        int l = 2 * i + 1, r = l + 1, m = i;
        if (l < k && kv_before_asc(h[m], h[l])) m = l;
        if (r < k && kv_before_asc(h[m], h[r])) m = r;
        if (m == i) break;
        kv_t t = h[m]; h[m] = h[i]; h[i] = t; i = m;
    }
}

static int cmp_kv_asc(const void* pa, const void* pb) {
    kv_t a = *(const kv_t*)pa, b = *(const kv_t*)pb;
    if (kv_before_asc(a, b)) return -1;
    if (kv_before_asc(b, a)) return 1;
    return 0;
}

/* Select the k best of `keys` (n entries, id = position) in ascending
 * (key, id) order.  Returns the number written (min(k, n)). */
static int select_topk_asc(const float* keys, int64_t n, int k, int32_t* out_ids, float* out_keys) {
    if (k > n) k = (int)n;
    if (k <= 0) return 0;
    kv_t* h = (kv_t*)malloc(sizeof(kv_t) * (size_t)k);
    int size = 0;
    for (int64_t i = 0; i < n; i++) {
        kv_t x = {keys[i], (int32_t)i};
        heap_push_asc(h, &size, k, x);
    }
    qsort(h, (size_t)size, sizeof(kv_t), cmp_kv_asc);
    for (int i = 0; i < size; i++) {
        out_ids[i] = h[i].id;
        if (out_keys) out_keys[i] = h[i].key;
    }
    free(h);
    return size;
}

/* ------------------------------------------------------------------------ */
/* Public oracle entry points (one call = nq queries).                       */
/* ------------------------------------------------------------------------ */

/* MadhavaL2::search_exact with Metric::L2 on a u8 corpus
 * (src/winnex_madhava.cpp:1224-1246).  out_ids/out_dist: [nq][k]; entries
 * beyond min(k, n) are set to -1 / INFINITY. */
void oracle_l2_exact_u8(const uint8_t* corpus, int64_t n, int d, const float* queries, int nq,
                        int k, int32_t* out_ids, float* out_dist) {
    float* dist = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    for (int qi = 0; qi < nq; qi++) {
        const float* q = queries + (size_t)qi * d;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) dist[i] = oracle_l2_sq_u8(corpus + (size_t)i * d, q, d);
        int m = select_topk_asc(dist, n, k, out_ids + (size_t)qi * k, out_dist + (size_t)qi * k);
        for (int j = m; j < k; j++) { out_ids[(size_t)qi * k + j] = -1; out_dist[(size_t)qi * k + j] = INFINITY; }
    }
    free(dist);
}

/* SpeedEngine exact scan (no anchors), src/speed_cpu.cpp:271-398.
 * corpus_f32 is the engine's internal float corpus (u8 cast to float, or the
 * row-normalized float corpus for cosine).  norms are |v|^2 (L2) and are
 * ignored for cosine.  Score = ip (cosine) or 2*ip - |v|^2 (L2); the query is
 * normalized for cosine (src/speed_cpu.cpp:278-287).  Output is descending
 * score, ties to the lower index; out_score is that score. */
void oracle_speed_exact(const float* corpus_f32, const float* norms, int64_t n, int d, int is_cosine,
                        const float* queries, int nq, int k, int32_t* out_ids, float* out_score) {
    float* neg = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    float* qbuf = (float*)malloc(sizeof(float) * (size_t)d);
    for (int qi = 0; qi < nq; qi++) {
        const float* q = queries + (size_t)qi * d;
        if (is_cosine) {
            float qn = 0.0f;
            for (int j = 0; j < d; j++) qn = fmaf(q[j], q[j], qn);
            qn = sqrtf(qn);
            float inv = qn > 1e-12f ? 1.0f / qn : 0.0f;
            for (int j = 0; j < d; j++) qbuf[j] = q[j] * inv;
            q = qbuf;
        }
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) {
            float ip = oracle_dot_f32(corpus_f32 + (size_t)i * d, q, d);
            float s = is_cosine ? ip : (float)(2.0 * (double)ip - (double)norms[i]);
            neg[i] = -s;
        }
        int m = select_topk_asc(neg, n, k, out_ids + (size_t)qi * k, out_score + (size_t)qi * k);
        for (int j = 0; j < m; j++) out_score[(size_t)qi * k + j] = -out_score[(size_t)qi * k + j];
        for (int j = m; j < k; j++) { out_ids[(size_t)qi * k + j] = -1; out_score[(size_t)qi * k + j] = -INFINITY; }
    }
    free(neg);
    free(qbuf);
}

/* SpeedEngine u8 constructor's float copy and norms, src/speed_cpu.cpp:117-140:
 * dst = (float)v; norm accumulates dst*dst left to right; cosine rows are
 * scaled by 1/sqrt(norm) and get norm 1; L2 rows keep norm = |v|^2. */
void oracle_speed_prepare_u8(const uint8_t* corpus, int64_t n, int d, int is_cosine, float* out_f32,
                             float* out_norms) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const uint8_t* v = corpus + (size_t)i * d;
        float* dst = out_f32 + (size_t)i * d;
        float norm = 0.0f;
        for (int j = 0; j < d; j++) { dst[j] = (float)v[j]; norm = fmaf(dst[j], dst[j], norm); }
        if (is_cosine) {
            norm = sqrtf(norm);
            if (norm > 1e-12f) {
                float inv = 1.0f / norm;
                for (int j = 0; j < d; j++) dst[j] *= inv;
            }
            out_norms[i] = 1.0f;
        } else {
            out_norms[i] = norm;
        }
    }
}

/* SpeedEngine float constructor, src/speed_cpu.cpp:81-115. */
void oracle_speed_prepare_f32(const float* corpus, int64_t n, int d, int is_cosine, float* out_f32,
                              float* out_norms) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const float* v = corpus + (size_t)i * d;
        float* dst = out_f32 + (size_t)i * d;
        float norm = 0.0f;
        if (is_cosine) {
            for (int j = 0; j < d; j++) { dst[j] = v[j]; norm = fmaf(v[j], v[j], norm); }
            norm = sqrtf(norm);
            if (norm > 1e-12f) {
                float inv = 1.0f / norm;
                for (int j = 0; j < d; j++) dst[j] *= inv;
            }
            out_norms[i] = 1.0f;
        } else {
            for (int j = 0; j < d; j++) { dst[j] = v[j]; norm = fmaf(dst[j], dst[j], norm); }
            out_norms[i] = norm;
        }
    }
}

/* MadhavaL2::search_exact with Metric::Cosine on a u8 base
 * (src/winnex_madhava.cpp:1224-1246 with exact_score :714-763).  Descending
 * score, ties to the lower index. */
void oracle_cosine_exact_u8(const uint8_t* corpus, int64_t n, int d, const float* queries, int nq, int k,
                            int32_t* out_ids, float* out_score) {
    float* neg = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    for (int qi = 0; qi < nq; qi++) {
        const float* q = queries + (size_t)qi * d;
        float qn2 = oracle_qn2(q, d);
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) neg[i] = -oracle_cosine_u8(corpus + (size_t)i * d, q, d, qn2);
        int m = select_topk_asc(neg, n, k, out_ids + (size_t)qi * k, out_score + (size_t)qi * k);
        for (int j = 0; j < m; j++) out_score[(size_t)qi * k + j] = -out_score[(size_t)qi * k + j];
        for (int j = m; j < k; j++) { out_ids[(size_t)qi * k + j] = -1; out_score[(size_t)qi * k + j] = -INFINITY; }
    }
    free(neg);
}

/* Integer exact L2 for u8 queries: int64 distances, ascending (dist, index).
 * Same ranking as oracle_l2_exact_u8 for integral queries, without float. */
void oracle_l2_exact_u8_int(const uint8_t* corpus, int64_t n, int d, const uint8_t* queries, int nq, int k,
                            int32_t* out_ids, int64_t* out_dist) {
    float* key = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    int64_t* dist = (int64_t*)malloc(sizeof(int64_t) * (size_t)(n > 0 ? n : 1));
    for (int qi = 0; qi < nq; qi++) {
        const uint8_t* q = queries + (size_t)qi * d;
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < n; i++) {
            const uint8_t* v = corpus + (size_t)i * d;
            int64_t s = 0;
            for (int j = 0; j < d; j++) { int64_t t = (int64_t)v[j] - (int64_t)q[j]; s += t * t; }
            dist[i] = s;
            key[i] = (float)s; /* exact: s < 2^24 for d <= 258 */
        }
        int32_t* ids = out_ids + (size_t)qi * k;
        int m = select_topk_asc(key, n, k, ids, NULL);
        for (int j = 0; j < m; j++) out_dist[(size_t)qi * k + j] = dist[ids[j]];
        for (int j = m; j < k; j++) { ids[j] = -1; out_dist[(size_t)qi * k + j] = -1; }
    }
    free(key);
    free(dist);
}

/* The same integer ranking as oracle_l2_exact_u8_int (ascending (distance,
 * index), MadhavaL2::search_exact, src/winnex_madhava.cpp:1224-1246), folded
 * into a running top-k so a corpus can be checked one slice at a time:
 * rows [0, n) of `corpus` carry the global ids id_base .. id_base + n - 1, and
 * ids_io / dist_io ([nq][k]) hold the best k seen so far on entry (id -1 for
 * an empty slot) and the best k including this slice on return.  Every
 * thread scans a contiguous row range against all queries (each row is read
 * once per call) into private lists, which are then merged; the result does
 * not depend on the thread count.  Distances are exact: d * 255^2 < 2^31 for
 * d <= 33025. */
typedef struct { int64_t dist; int32_t id; } dk_t;

static int dk_before(dk_t a, dk_t b) { return a.dist < b.dist || (a.dist == b.dist && a.id < b.id); }

/* Insert x into the sorted list l of size *m (capacity k). */
static void dk_insert(dk_t* l, int* m, int k, dk_t x) {
    if (*m == k && !dk_before(x, l[k - 1])) return;
    int i = *m < k ? (*m)++ : k - 1;
    while (i > 0 && dk_before(x, l[i - 1])) { l[i] = l[i - 1]; i--; }
    l[i] = x;
}

__attribute__((optimize("O3"))) void oracle_l2_topk_u8_update(const uint8_t* corpus, int64_t n, int d,
                                                               int64_t id_base, const uint8_t* queries, int nq,
                                                               int k, int32_t* ids_io, int64_t* dist_io) {
    if (k <= 0 || nq <= 0) return;
    int nt = 1;
#ifdef _OPENMP
    nt = omp_get_max_threads();
#endif
    dk_t* lists = (dk_t*)malloc(sizeof(dk_t) * (size_t)nt * nq * k);
    int* sizes = (int*)calloc((size_t)nt * nq, sizeof(int));
#pragma omp parallel num_threads(nt)
    {
        int t = 0;
#ifdef _OPENMP
        t = omp_get_thread_num();
#endif
        const int64_t r0 = n * t / nt, r1 = n * (t + 1) / nt;
        dk_t* my = lists + (size_t)t * nq * k;
        int* msz = sizes + (size_t)t * nq;
        for (int64_t i = r0; i < r1; i++) {
            const uint8_t* v = corpus + (size_t)i * d;
            for (int qi = 0; qi < nq; qi++) {
                const uint8_t* q = queries + (size_t)qi * d;
                int32_t s = 0;
                for (int j = 0; j < d; j++) { int32_t e = (int32_t)v[j] - (int32_t)q[j]; s += e * e; }
                dk_t x = {s, (int32_t)(id_base + i)};
                dk_insert(my + (size_t)qi * k, msz + qi, k, x);
            }
        }
    }
    dk_t* merged = (dk_t*)malloc(sizeof(dk_t) * (size_t)k);
    for (int qi = 0; qi < nq; qi++) {
        int m = 0;
        for (int j = 0; j < k; j++) {
            int32_t id = ids_io[(size_t)qi * k + j];
            if (id < 0) break;
            dk_t x = {dist_io[(size_t)qi * k + j], id};
            dk_insert(merged, &m, k, x);
        }
        for (int t = 0; t < nt; t++) {
            const dk_t* l = lists + ((size_t)t * nq + qi) * k;
            for (int j = 0; j < sizes[(size_t)t * nq + qi]; j++) dk_insert(merged, &m, k, l[j]);
        }
        for (int j = 0; j < k; j++) {
            ids_io[(size_t)qi * k + j] = j < m ? merged[j].id : -1;
            dist_io[(size_t)qi * k + j] = j < m ? merged[j].dist : -1;
        }
    }
    free(merged);
    free(sizes);
    free(lists);
}

/* Score given row ids of one query with the reference arithmetic.
 * kind 0: l2_sq_avx over u8 rows (MadhavaL2 L2);
 * kind 1: exact_score cosine over u8 rows (MadhavaL2 cosine);
 * kind 2: SpeedEngine score over the prepared float rows (cosine: the query
 *         is normalized as in src/speed_cpu.cpp:278-287; L2: 2*ip - |v|^2).
 * Ids < 0 score NAN. */
void oracle_score_ids(int kind, int is_cosine, const uint8_t* corpus_u8, const float* corpus_f32,
                      const float* norms, int d, const float* q, const int32_t* ids, int m, float* out) {
    float* qbuf = (float*)malloc(sizeof(float) * (size_t)d);
    const float* qq = q;
    if (kind == 2 && is_cosine) {
        float qn = 0.0f;
        for (int j = 0; j < d; j++) qn = fmaf(q[j], q[j], qn);
        qn = sqrtf(qn);
        float inv = qn > 1e-12f ? 1.0f / qn : 0.0f;
        for (int j = 0; j < d; j++) qbuf[j] = q[j] * inv;
        qq = qbuf;
    }
    float qn2 = oracle_qn2(q, d);
    for (int i = 0; i < m; i++) {
        int64_t r = ids[i];
        if (r < 0) { out[i] = NAN; continue; }
        if (kind == 0) out[i] = oracle_l2_sq_u8(corpus_u8 + (size_t)r * d, q, d);
        else if (kind == 1) out[i] = oracle_cosine_u8(corpus_u8 + (size_t)r * d, q, d, qn2);
        else {
            float ip = oracle_dot_f32(corpus_f32 + (size_t)r * d, qq, d);
            out[i] = is_cosine ? ip : (float)(2.0 * (double)ip - (double)norms[r]);
        }
    }
    free(qbuf);
}

/* MadHybrid routing, python/winnex_madhava/__init__.py:631-632:
 * sims = centroids @ q, then the nprobe largest (argsort(-sims)[:nprobe]).
 * The reference evaluates the product in float32 through BLAS, whose
 * summation order is unspecified; this restatement fixes it: fp64
 * multiply-adds in dimension order from 0.0, ties to the lower cell id.
 * out_cells: [nq][nprobe], best first. */
/* Float-query routing and the exact inner-product ranking of float32 IVF
 * cells (MadHybrid over a float corpus, python/winnex_madhava/__init__.py:
 * routing `centroids @ q` at :631-632; each cell scores its rows by
 * `vecs @ q` in float64 at :526 and the merge orders by score at :650).
 * Here every row of the probed cells is scored (the exact top-k over their
 * union): s = sum_j fma(row[j], q[j]) in float64 in dimension order, ranked
 * by (s descending, row id ascending).  Routing as oracle_ivf_route. */
void oracle_ivf_route_f32(const float* centroids, int nlist, int d, const float* queries, int nq, int nprobe,
                          int32_t* out_cells) {
#pragma omp parallel
    {
        double* sims = (double*)malloc(sizeof(double) * (size_t)nlist);
#pragma omp for schedule(dynamic, 4)
        for (int qi = 0; qi < nq; qi++) {
            const float* q = queries + (size_t)qi * d;
            for (int c = 0; c < nlist; c++) {
                const float* cr = centroids + (size_t)c * d;
                double acc = 0.0;
                for (int j = 0; j < d; j++) acc = fma((double)q[j], (double)cr[j], acc);
                sims[c] = acc;
            }
            for (int p = 0; p < nprobe; p++) {
                int bi = -1;
                for (int c = 0; c < nlist; c++)
                    if (bi < 0 || sims[c] > sims[bi]) bi = c;
                out_cells[(size_t)qi * nprobe + p] = bi;
                sims[bi] = -INFINITY;
            }
        }
        free(sims);
    }
}

void oracle_ivf_ip_f32(const float* rows, int64_t n, int d, const int32_t* labels, const int32_t* cells, int nprobe,
                       const float* queries, int nq, int k, int32_t* out_ids, double* out_scores) {
#pragma omp parallel
    {
        double* ts = (double*)malloc(sizeof(double) * (size_t)k);
        int32_t* ti = (int32_t*)malloc(sizeof(int32_t) * (size_t)k);
#pragma omp for schedule(dynamic, 1)
        for (int qi = 0; qi < nq; qi++) {
            const float* q = queries + (size_t)qi * d;
            const int32_t* cq = cells + (size_t)qi * nprobe;
            int cnt = 0;
            for (int64_t r = 0; r < n; r++) {
                int hit = 0;
                for (int p = 0; p < nprobe; p++) hit |= labels[r] == cq[p];
                if (!hit) continue;
                const float* v = rows + (size_t)r * d;
                double s = 0.0;
                for (int j = 0; j < d; j++) s = fma((double)v[j], (double)q[j], s);
                /* insert (s, r) into the descending list (ties: lower id first) */
                int pos = cnt < k ? cnt : k;
                while (pos > 0 && (ts[pos - 1] < s)) pos--;
                if (pos >= k) continue;
                int last = cnt < k ? cnt : k - 1;
                for (int m = last; m > pos; m--) {
                    ts[m] = ts[m - 1];
                    ti[m] = ti[m - 1];
                }
                ts[pos] = s;
                ti[pos] = (int32_t)r;
                if (cnt < k) cnt++;
            }
            for (int m = 0; m < k; m++) {
                out_ids[(size_t)qi * k + m] = m < cnt ? ti[m] : -1;
                out_scores[(size_t)qi * k + m] = m < cnt ? ts[m] : -INFINITY;
            }
        }
        free(ts);
        free(ti);
    }
}

void oracle_ivf_route(const float* centroids, int nlist, int d, const uint8_t* queries, int nq, int nprobe,
                      int32_t* out_cells) {
#pragma omp parallel
    {
        double* sims = (double*)malloc(sizeof(double) * (size_t)nlist);
#pragma omp for schedule(dynamic, 4)
        for (int qi = 0; qi < nq; qi++) {
            const uint8_t* q = queries + (size_t)qi * d;
            for (int c = 0; c < nlist; c++) {
                const float* cr = centroids + (size_t)c * d;
                double acc = 0.0;
                for (int j = 0; j < d; j++) acc = fma((double)q[j], (double)cr[j], acc);
                sims[c] = acc;
            }
            for (int p = 0; p < nprobe; p++) {
                int bi = -1;
                for (int c = 0; c < nlist; c++)
                    if (bi < 0 || sims[c] > sims[bi]) bi = c; /* first maximum = lower id */
                out_cells[(size_t)qi * nprobe + p] = bi;
                sims[bi] = -INFINITY;
            }
        }
        free(sims);
    }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
