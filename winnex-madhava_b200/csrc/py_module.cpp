// _winnex_madhava: pybind11 module over the C ABI (include/winnex_madhava_b200.h).
//
// Mirrors the reference module of the same name (bindings/py_module.cpp):
// the enums, Config, SearchResult, MadhavaL2, SpeedEngine and the metric
// helpers keep their names, argument names, defaults and error messages.
// Search runs on the GPU through libwinnex_madhava_b200.so with the GIL
// released.  What changes by design:
//   * MadhavaL2.search / search_batch return the exact top-K (the same list
//     as search_exact); k1 = k2 = N; pruned_by_bound = pairs the tensor
//     scan's block bound proved outside the top-K without forming their
//     distance (a Cauchy-Schwarz-style certificate on norm-sorted rows);
//     k3 = exact_evals = the pairs whose exact distance was formed;
//     bound_violations is measured when verification is on (set_verify) and
//     is 0 otherwise;
//   * SpeedEngine always runs on the GPU (has_gpu() is True); n_anchors is
//     accepted, and the scan stays exact.  The reference does the same when
//     a CUDA device is present: enable_gpu sets use_gpu_ (src/speed_gpu.cu:
//     136-160) and search / search_batch then take the brute-force
//     scores_gpu_topk (src/speed_cpu.cpp:426-448); only its CPU single-query
//     path routes through the anchor cells (:295-328);
//   * save_index / load_index write and read this library's index file (the
//     norm-sorted corpus, norms and ids; no re-attached base is needed);
//   * audit certificates and commitments (search_audited, audit_json,
//     search_with_commitment) certify the exact result against a second GPU
//     pass over every row with the k-th result's value as the threshold;
//     their sample is the excluded rows nearest that threshold, in
//     (value, id) order;
//   * projection bases and residuals (bound-engine internals) raise
//     NotImplementedError.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "winnex_madhava_b200.h"

namespace py = pybind11;

namespace {

enum class Metric { Cosine = 0, L2 = 1 };
enum class QuantMode { Int8 = 0, None = 1 };
enum class BasisMode { Random = 0, PCACorpus = 1 };

// Field set and defaults of the reference Config
// (include/winnex_madhava/winnex_madhava.hpp:73-113).
struct Config {
    int dim = 128;
    int seed = 42;
    int pca_sample = 10000;
    Metric metric = Metric::Cosine;
    QuantMode quant = QuantMode::Int8;
    BasisMode basis = BasisMode::Random;
    int stage1_dim = 64;
    int stage2_dim = 128;
    int k = 10;
    double k1_fraction = 0.05;
    double k2_fraction = 0.01;
    int k1_min = 100;
    int k2_min = 10;
    int k2_max = 2000;
    bool modulation = true;
    bool postfilter = true;
    bool normalize_input = true;
    bool early_exit = false;
    int n_threads = 0;
};

// Field set of the reference SearchResult (winnex_madhava.hpp:118-164).
struct SearchResult {
    std::vector<int> indices;
    int k1 = 0, k2 = 0, k3 = 0;
    double latency_ms = 0.0;
    long long bound_pairs = 0;
    long long bound_violations = 0;
    double modulation_gain = 0.0;
    long long pruned_by_bound = 0;
    long long pruned_by_prefilter = 0;
    long long exact_evals = 0;
    double audit_threshold = 0.0;
    std::vector<int64_t> audit_ids;
    std::vector<float> audit_ubs;
    std::vector<float> audit_l2_lbs;
    std::vector<float> audit_residuals;
};

void check(mdh_status s) {
    if (s == MDH_OK) return;
    std::string msg = mdh_last_error();
    if (s == MDH_ERR_OOM) throw std::bad_alloc();
    throw std::runtime_error(msg.empty() ? std::string("winnex_madhava_b200 error ") + std::to_string((int)s) : msg);
}

[[noreturn]] void not_implemented(const char* what) {
    PyErr_SetString(PyExc_NotImplementedError, what);
    throw py::error_already_set();
}

using F32Array = py::array_t<float, py::array::c_style | py::array::forcecast>;
using U8Array = py::array_t<uint8_t, py::array::c_style | py::array::forcecast>;

struct IndexHandle {
    mdh_index* ix = nullptr;
    ~IndexHandle() {
        if (ix) mdh_index_destroy(ix);
    }
    void reset(mdh_index* p) {
        if (ix) mdh_index_destroy(ix);
        ix = p;
    }
};

std::vector<int32_t> parse_devices(const py::object& devices) {
    std::vector<int32_t> d;
    if (devices.is_none()) return d;
    if (py::isinstance<py::int_>(devices)) {
        int n = devices.cast<int>();
        for (int i = 0; i < n; i++) d.push_back(i);
        return d;
    }
    for (auto h : devices) d.push_back(h.cast<int>());
    return d;
}

// ---------------------------------------------------------------------------
class MadhavaL2 {
public:
    explicit MadhavaL2(const Config& cfg) : cfg_(cfg) {}

    void build_u8(const uint8_t* data, int n) {
        auto t0 = std::chrono::high_resolution_clock::now();
        mdh_index* p = nullptr;
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_index_create_u8(data, n, cfg_.dim, (int32_t)cfg_.metric, devices_.empty() ? nullptr : devices_.data(),
                                    (int32_t)devices_.size(), 0, &p);
        }
        check(s);
        h_.reset(p);
        n_ = n;
        built_ = true;
        build_s_ = std::chrono::duration<double>(std::chrono::high_resolution_clock::now() - t0).count();
    }

    // MadhavaL2::build_float32 (src/winnex_madhava.cpp:433-468): the float
    // rows are re-quantized with u8 = clamp((v + 1) * 127.5, 0, 255) and the
    // exact scores run over those bytes.
    void build_f32(const float* data, int n) {
        const int D = cfg_.dim;
        std::vector<uint8_t> q((size_t)n * D);
        for (size_t i = 0; i < (size_t)n * D; i++) {
            float v = data[i];
            float t = (v + 1.0f) * 127.5f;
            if (t < 0.0f) t = 0.0f;
            if (t > 255.0f) t = 255.0f;
            q[i] = (uint8_t)t;
        }
        if (cfg_.quant == QuantMode::None && cfg_.metric == Metric::Cosine)
            not_implemented("MadhavaL2.build_float32 with quant='none' and metric='cosine' (float-row exact cosine) "
                            "is not implemented in this build");
        build_u8(q.data(), n);
    }

    SearchResult search_one(const F32Array& q) const {
        auto info = q.request();
        if (info.ndim != 1 || (int)info.shape[0] != cfg_.dim)
            throw std::runtime_error("query must be float32 of length dim");
        SearchResult out;
        if (!built_) return out;
        std::vector<int32_t> ids((size_t)cfg_.k);
        mdh_stats st{};
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_search_f32(h_.ix, (const float*)info.ptr, 1, cfg_.k, MDH_SCORE_EXACT, ids.data(), nullptr, &st);
        }
        check(s);
        for (int32_t id : ids)
            if (id >= 0) out.indices.push_back(id);
        out.k1 = n_;
        out.k2 = n_;
        const int64_t formed = st.pairs_scored - st.pairs_pruned_by_bound;
        out.k3 = (int)std::min<int64_t>(formed, 0x7fffffff);
        out.bound_pairs = n_;
        out.exact_evals = formed;
        out.bound_violations = st.bound_violations;
        out.pruned_by_bound = st.pairs_pruned_by_bound;
        out.latency_ms = st.latency_ms;
        return out;
    }

    // One audited query (mdh_audit_f32): the top min(k, config.k) and the
    // excluded rows nearest the threshold, at most max_records of them.
    struct Audit {
        std::vector<int32_t> ids, rec_ids;
        std::vector<float> vals, rec_vals;
        mdh_audit a{};
        mdh_stats st{};
        int k = 0;
    };
    Audit audit_one(const F32Array& q, int64_t k, int64_t max_records) const {
        auto info = q.request();
        if (info.ndim != 1 || (int)info.shape[0] != cfg_.dim)
            throw std::runtime_error("query must be float32 of length dim");
        Audit r;
        if (!built_) return r;
        r.k = (int)std::max<int64_t>(1, std::min<int64_t>(k > 0 ? k : cfg_.k, cfg_.k));
        const int mr = (int)std::max<int64_t>(0, std::min<int64_t>(max_records, 0x7fffffff));
        r.ids.assign((size_t)r.k, -1);
        r.vals.assign((size_t)r.k, 0.0f);
        r.rec_ids.assign((size_t)std::max(mr, 1), -1);
        r.rec_vals.assign((size_t)std::max(mr, 1), 0.0f);
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_audit_f32(h_.ix, (const float*)info.ptr, 1, r.k, mr, r.ids.data(), r.vals.data(),
                              r.rec_ids.data(), r.rec_vals.data(), &r.a, &r.st);
        }
        check(s);
        return r;
    }

    std::vector<int> search_batch(const F32Array& q, int nq, int k) const {
        auto info = q.request();
        if (info.ndim != 2 || (int)info.shape[0] != nq || (int)info.shape[1] != cfg_.dim)
            throw std::runtime_error("queries must be (nq, dim) float32");
        std::vector<int> all;
        if (!built_ || nq <= 0 || k <= 0) return all;
        std::vector<int32_t> ids((size_t)nq * k);
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_search_f32(h_.ix, (const float*)info.ptr, nq, k, MDH_SCORE_EXACT, ids.data(), nullptr, nullptr);
        }
        check(s);
        all.assign(ids.begin(), ids.end());
        return all;
    }

    // MadhavaL2::save_index (src/winnex_madhava.cpp:1120-1149): false when the
    // engine is not built or the file cannot be written.  The file holds the
    // norm-sorted corpus itself, so a loaded engine needs no re-attached base.
    bool save_index(const std::string& path) const {
        if (!built_) return false;
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_index_save(h_.ix, path.c_str());
        }
        if (s == MDH_ERR_IO) return false;
        check(s);
        return true;
    }

    // MadhavaL2::load_index (src/winnex_madhava.cpp:1151-1217): drops the
    // current state first, then returns false when the file cannot be read or
    // fails its header or integrity checks.  dim and metric come from the file.
    bool load_index(const std::string& path) {
        h_.reset(nullptr);
        built_ = false;
        n_ = 0;
        mdh_index* p = nullptr;
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_index_load(path.c_str(), devices_.empty() ? nullptr : devices_.data(), (int32_t)devices_.size(), &p);
        }
        if (s == MDH_ERR_IO) return false;
        check(s);
        h_.reset(p);
        // Engine results index the corpus from row 0; a file holding another
        // id range (one rank's rows of a larger corpus) cannot back it.
        int64_t first = 0;
        check(mdh_index_id_base(p, &first));
        if (first != 0) {
            h_.reset(nullptr);
            return false;
        }
        int64_t n = 0;
        int32_t dim = 0, metric = 0;
        check(mdh_index_info(p, &n, &dim, &metric, nullptr));
        n_ = (int)n;
        cfg_.dim = dim;
        cfg_.metric = (Metric)metric;
        built_ = true;
        return true;
    }

    int num_vectors() const { return n_; }
    int dim() const { return cfg_.dim; }
    const Config& config() const { return cfg_; }
    double build_seconds() const { return build_s_; }
    bool built() const { return built_; }
    void set_devices(std::vector<int32_t> d) { devices_ = std::move(d); }
    mdh_index* handle() const { return h_.ix; }

private:
    Config cfg_;
    IndexHandle h_;
    int n_ = 0;
    bool built_ = false;
    double build_s_ = 0.0;
    std::vector<int32_t> devices_;
};

// ---------------------------------------------------------------------------
// GPU IVF index (MadHybrid's uint8 L2 path): cells given as centroids + labels.
class IvfIndex {
public:
    IvfIndex(const U8Array& corpus, const F32Array& centroids, py::array_t<int32_t, py::array::c_style |
                                                                             py::array::forcecast> labels,
             int device, int metric) {
        auto ic = corpus.request(), ie = centroids.request(), il = labels.request();
        if (ic.ndim != 2) throw std::runtime_error("corpus must be a 2-D uint8 array");
        if (ie.ndim != 2 || ie.shape[1] != ic.shape[1]) throw std::runtime_error("centroids must be [nlist][dim]");
        if (il.size != ic.shape[0]) throw std::runtime_error("labels must hold one cell per row");
        n_ = (int64_t)ic.shape[0];
        dim_ = (int)ic.shape[1];
        nlist_ = (int)ie.shape[0];
        mdh_ivf* p = nullptr;
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_ivf_create_u8_metric((const uint8_t*)ic.ptr, n_, dim_, (const float*)ie.ptr, nlist_,
                                         (const int32_t*)il.ptr, metric, device, &p);
        }
        check(s);
        ix_ = p;
    }
    ~IvfIndex() {
        if (ix_) mdh_ivf_destroy(ix_);
    }
    IvfIndex(const IvfIndex&) = delete;
    IvfIndex& operator=(const IvfIndex&) = delete;

    // queries [nq][dim] u8 -> (ids, dists) [nq][k] and the call's stats
    py::tuple search(const U8Array& q, int k, int nprobe) const {
        auto info = q.request();
        const int nq = info.ndim == 1 ? 1 : (int)info.shape[0];
        if ((size_t)info.size != (size_t)nq * dim_) throw std::runtime_error("queries must be uint8 [nq][dim]");
        py::array_t<int32_t> ids({nq, k}), dist({nq, k});
        mdh_stats st{};
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_ivf_search_u8(ix_, (const uint8_t*)info.ptr, nq, k, nprobe, ids.mutable_data(),
                                  dist.mutable_data(), &st);
        }
        check(s);
        py::dict d;
        d["latency_ms"] = st.latency_ms;
        d["pairs_scored"] = (long long)st.pairs_scored;
        d["pruned_by_bound"] = (long long)st.pairs_pruned_by_bound;
        d["blocks_tested"] = (long long)st.blocks_tested;
        d["blocks_passed"] = (long long)st.blocks_passed;
        d["bound_violations"] = (long long)st.bound_violations;
        d["full_scan_ms"] = st.full_scan_ms;
        d["kernel_launches"] = (long long)st.kernel_launches;
        return py::make_tuple(ids, dist, d);
    }
    py::array_t<int32_t> route(const U8Array& q, int nprobe) const {
        auto info = q.request();
        const int nq = info.ndim == 1 ? 1 : (int)info.shape[0];
        if ((size_t)info.size != (size_t)nq * dim_) throw std::runtime_error("queries must be uint8 [nq][dim]");
        py::array_t<int32_t> cells({nq, nprobe});
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_ivf_route_u8(ix_, (const uint8_t*)info.ptr, nq, nprobe, cells.mutable_data());
        }
        check(s);
        return cells;
    }
    int64_t num_vectors() const { return n_; }
    int nlist() const { return nlist_; }

private:
    mdh_ivf* ix_ = nullptr;
    int64_t n_ = 0;
    int dim_ = 0, nlist_ = 0;
};

// The float32 clustered index (mdh_ivf_*_f32): MadHybrid over a float
// corpus, every probed row scored in float64.
class IvfIndexF32 {
public:
    IvfIndexF32(const F32Array& corpus, const F32Array& centroids,
                py::array_t<int32_t, py::array::c_style | py::array::forcecast> labels, int device) {
        auto ic = corpus.request(), ie = centroids.request(), il = labels.request();
        if (ic.ndim != 2) throw std::runtime_error("corpus must be a 2-D float32 array");
        if (ie.ndim != 2 || ie.shape[1] != ic.shape[1]) throw std::runtime_error("centroids must be [nlist][dim]");
        if (il.size != ic.shape[0]) throw std::runtime_error("labels must hold one cell per row");
        n_ = (int64_t)ic.shape[0];
        dim_ = (int)ic.shape[1];
        nlist_ = (int)ie.shape[0];
        mdh_ivf_f32* p = nullptr;
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_ivf_create_f32((const float*)ic.ptr, n_, dim_, (const float*)ie.ptr, nlist_,
                                   (const int32_t*)il.ptr, device, &p);
        }
        check(s);
        ix_ = p;
    }
    ~IvfIndexF32() {
        if (ix_) mdh_ivf_destroy_f32(ix_);
    }
    IvfIndexF32(const IvfIndexF32&) = delete;
    IvfIndexF32& operator=(const IvfIndexF32&) = delete;

    // queries [nq][dim] float32 -> (ids, scores float64) [nq][k] and stats
    py::tuple search(const F32Array& q, int k, int nprobe) const {
        auto info = q.request();
        const int nq = info.ndim == 1 ? 1 : (int)info.shape[0];
        if ((size_t)info.size != (size_t)nq * dim_) throw std::runtime_error("queries must be float32 [nq][dim]");
        py::array_t<int32_t> ids({nq, k});
        py::array_t<double> sc({nq, k});
        mdh_stats st{};
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_ivf_search_f32(ix_, (const float*)info.ptr, nq, k, nprobe, ids.mutable_data(), sc.mutable_data(),
                                   &st);
        }
        check(s);
        py::dict d;
        d["latency_ms"] = st.latency_ms;
        d["pairs_scored"] = (long long)st.pairs_scored;
        d["kernel_launches"] = (long long)st.kernel_launches;
        return py::make_tuple(ids, sc, d);
    }
    int64_t num_vectors() const { return n_; }
    int nlist() const { return nlist_; }

private:
    mdh_ivf_f32* ix_ = nullptr;
    int64_t n_ = 0;
    int dim_ = 0, nlist_ = 0;
};

// ---------------------------------------------------------------------------
class SpeedEngine {
public:
    SpeedEngine(const void* data, bool is_f32, int n, int dim, int metric, std::vector<int32_t> devices)
        : n_(n), dim_(dim) {
        if (metric != 0 && metric != 1) throw std::runtime_error("metric must be 0 (cosine) or 1 (l2)");
        mdh_index* p = nullptr;
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            if (is_f32)
                s = mdh_index_create_f32((const float*)data, n, dim, metric, devices.empty() ? nullptr : devices.data(),
                                         (int32_t)devices.size(), 0, &p);
            else
                s = mdh_index_create_u8((const uint8_t*)data, n, dim, metric, devices.empty() ? nullptr : devices.data(),
                                        (int32_t)devices.size(), 0, &p);
        }
        check(s);
        h_.reset(p);
    }

    py::dict search(const F32Array& q, int k) const {
        auto info = q.request();
        if ((size_t)info.size != (size_t)dim_) throw std::runtime_error("query must be float32 of length dim");
        std::vector<int32_t> ids((size_t)std::max(k, 0));
        mdh_stats st{};
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_search_f32(h_.ix, (const float*)info.ptr, 1, k, MDH_SCORE_SPEED, ids.data(), nullptr, &st);
        }
        check(s);
        std::vector<int> out;
        for (int32_t id : ids)
            if (id >= 0) out.push_back(id);
        py::dict d;
        d["indices"] = out;
        d["latency_ms"] = st.latency_ms;
        d["bound_pairs"] = (long long)n_;
        d["bound_violations"] = (long long)st.bound_violations;
        d["pruned_by_bound"] = (long long)st.pairs_pruned_by_bound;
        d["verified_queries"] = (long long)st.verified_queries;
        return d;
    }

    py::dict search_batch(const F32Array& q, int nq, int k) const {
        auto info = q.request();
        if ((size_t)info.size != (size_t)nq * dim_) throw std::runtime_error("queries must be (nq, dim) float32");
        int kk = std::min(std::max(k, 0), n_);
        std::vector<int32_t> ids((size_t)nq * std::max(k, 0));
        mdh_stats st{};
        mdh_status s;
        {
            py::gil_scoped_release nogil;
            s = mdh_search_f32(h_.ix, (const float*)info.ptr, nq, k, MDH_SCORE_SPEED_BATCH, ids.data(), nullptr, &st);
        }
        check(s);
        // SpeedResult::indices is the concatenation of min(k, N) ids per query
        // (src/speed_cpu.cpp:393).
        std::vector<int> out;
        out.reserve((size_t)nq * kk);
        for (int i = 0; i < nq; i++)
            for (int j = 0; j < kk; j++) out.push_back(ids[(size_t)i * k + j]);
        // The reference returns indices and latency_ms here; the counters
        // below are this library's additions (bound_pairs as in search()).
        py::dict d;
        d["indices"] = out;
        d["latency_ms"] = st.latency_ms;
        d["bound_pairs"] = (long long)n_ * nq;
        d["bound_violations"] = (long long)st.bound_violations;
        d["pruned_by_bound"] = (long long)st.pairs_pruned_by_bound;
        d["verified_queries"] = (long long)st.verified_queries;
        return d;
    }

    int num_vectors() const { return n_; }
    int dim() const { return dim_; }

private:
    IndexHandle h_;
    int n_, dim_;
};

// ---------------------------------------------------------------------------
// Metric helpers with the reference's definitions (src/winnex_madhava.cpp:320-377).
double recall_at_k(const std::vector<int>& result, const std::vector<int>& gt_set, int k) {
    int hits = 0;
    for (int ri : result)
        for (int vi : gt_set)
            if (ri == vi) {
                hits++;
                break;
            }
    int denom = std::min(k, (int)gt_set.size());
    return denom > 0 ? (double)hits / (double)denom : 0.0;
}

double ndcg_at_k(const std::vector<int>& result, const std::vector<int>& gt_set, int k) {
    double dcg = 0, idcg = 0;
    int top = std::min(k, (int)gt_set.size());
    for (int j = 0; j < top && j < (int)result.size(); j++) {
        int rel = 0;
        for (int vi : gt_set)
            if (result[j] == vi) {
                rel = 1;
                break;
            }
        dcg += (std::pow(2, rel) - 1) / std::log2(j + 2);
    }
    for (int j = 0; j < top; j++) idcg += 1.0 / std::log2(j + 2);
    return idcg > 0 ? dcg / idcg : 0.0;
}

float l2_sq(const U8Array& v_raw, const F32Array& q, int dim) {
    auto iv = v_raw.request();
    auto iq = q.request();
    if (iv.size < dim || iq.size < dim) throw std::runtime_error("l2_sq: inputs shorter than dim");
    const uint8_t* v = (const uint8_t*)iv.ptr;
    const float* qq = (const float*)iq.ptr;
    float s = 0;
    for (int j = 0; j < dim; j++) {
        float d = (float)v[j] - qq[j];
        s = std::fma(d, d, s);  // the reference build contracts `s += d * d` (-mfma)
    }
    return s;
}

std::vector<std::vector<int>> read_bigann_groundtruth(const std::string& path, int n_queries) {
    std::vector<std::vector<int>> gt;
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return gt;
    int32_t nq = 0, dim = 0;
    if (std::fread(&nq, 4, 1, f) != 1 || std::fread(&dim, 4, 1, f) != 1 || nq < 0 || dim < 0) {
        std::fclose(f);
        return gt;
    }
    int want = n_queries > 0 ? std::min(n_queries, (int)nq) : (int)nq;
    gt.resize((size_t)want);
    std::vector<int32_t> ids((size_t)dim);
    std::vector<float> dists((size_t)dim);
    for (int gi = 0; gi < want; gi++) {
        if (std::fread(ids.data(), 4, (size_t)dim, f) != (size_t)dim) break;
        if (std::fread(dists.data(), 4, (size_t)dim, f) != (size_t)dim) break;
        gt[(size_t)gi].assign(ids.begin(), ids.end());
    }
    std::fclose(f);
    return gt;
}

}  // namespace

PYBIND11_MODULE(_winnex_madhava, m) {
    m.doc() = "winnex-madhava exact top-K search on B200 (sm_100a CUDA kernels behind a C ABI)";

    py::enum_<Metric>(m, "Metric").value("COSINE", Metric::Cosine).value("L2", Metric::L2).export_values();
    py::enum_<QuantMode>(m, "QuantMode").value("INT8", QuantMode::Int8).value("NONE", QuantMode::None).export_values();
    py::enum_<BasisMode>(m, "BasisMode")
        .value("RANDOM", BasisMode::Random)
        .value("PCA_CORPUS", BasisMode::PCACorpus)
        .export_values();

    py::class_<Config>(m, "Config")
        .def(py::init<>())
        .def_readwrite("dim", &Config::dim)
        .def_readwrite("seed", &Config::seed)
        .def_readwrite("metric", &Config::metric)
        .def_readwrite("quant", &Config::quant)
        .def_readwrite("basis", &Config::basis)
        .def_readwrite("pca_sample", &Config::pca_sample)
        .def_readwrite("stage1_dim", &Config::stage1_dim)
        .def_readwrite("stage2_dim", &Config::stage2_dim)
        .def_readwrite("k", &Config::k)
        .def_readwrite("k1_fraction", &Config::k1_fraction)
        .def_readwrite("k2_fraction", &Config::k2_fraction)
        .def_readwrite("k1_min", &Config::k1_min)
        .def_readwrite("k2_min", &Config::k2_min)
        .def_readwrite("k2_max", &Config::k2_max)
        .def_readwrite("modulation", &Config::modulation)
        .def_readwrite("postfilter", &Config::postfilter)
        .def_readwrite("normalize_input", &Config::normalize_input)
        .def_readwrite("early_exit", &Config::early_exit)
        .def_readwrite("n_threads", &Config::n_threads);

    py::class_<SearchResult>(m, "SearchResult")
        .def_readonly("indices", &SearchResult::indices)
        .def_readonly("k1", &SearchResult::k1)
        .def_readonly("k2", &SearchResult::k2)
        .def_readonly("k3", &SearchResult::k3)
        .def_readonly("latency_ms", &SearchResult::latency_ms)
        .def_readonly("bound_pairs", &SearchResult::bound_pairs)
        .def_readonly("bound_violations", &SearchResult::bound_violations)
        .def_readonly("modulation_gain", &SearchResult::modulation_gain)
        .def_readonly("pruned_by_bound", &SearchResult::pruned_by_bound)
        .def_readonly("pruned_by_prefilter", &SearchResult::pruned_by_prefilter)
        .def_readonly("exact_evals", &SearchResult::exact_evals)
        .def_readonly("audit_threshold", &SearchResult::audit_threshold)
        .def_readonly("audit_ids", &SearchResult::audit_ids)
        .def_readonly("audit_ubs", &SearchResult::audit_ubs)
        .def_readonly("audit_l2_lbs", &SearchResult::audit_l2_lbs)
        .def_readonly("audit_residuals", &SearchResult::audit_residuals);

    py::class_<MadhavaL2>(m, "MadhavaL2")
        .def(py::init<const Config&>())
        .def(
            "build",
            [](MadhavaL2& self, py::bytes raw, int n, int dim) {
                char* buf = nullptr;
                Py_ssize_t len = 0;
                PyBytes_AsStringAndSize(raw.ptr(), &buf, &len);
                if ((size_t)len < (size_t)n * dim) throw std::runtime_error("raw buffer too small for n*dim");
                self.build_u8((const uint8_t*)buf, n);
            },
            py::arg("raw"), py::arg("n"), py::arg("dim"))
        .def(
            "build_numpy",
            [](MadhavaL2& self, U8Array arr) {
                auto info = arr.request();
                if (info.ndim != 2) throw std::runtime_error("expected 2D uint8 array (n, dim)");
                int n = (int)info.shape[0];
                if ((int)info.shape[1] != self.dim()) throw std::runtime_error("array dim does not match Config.dim");
                self.build_u8((const uint8_t*)info.ptr, n);
                return n;
            },
            py::arg("arr"))
        .def(
            "build_float32",
            [](MadhavaL2& self, F32Array arr) {
                auto info = arr.request();
                if (info.ndim != 2) throw std::runtime_error("expected 2D float32 array (n, dim)");
                int n = (int)info.shape[0];
                if ((int)info.shape[1] != self.dim()) throw std::runtime_error("array dim does not match Config.dim");
                self.build_f32((const float*)info.ptr, n);
                return n;
            },
            py::arg("arr"))
        .def(
            "set_basis", [](MadhavaL2&, py::object, py::object) { not_implemented("MadhavaL2.set_basis (bound-engine projection basis) is not part of the exact engine"); },
            py::arg("P1"), py::arg("P2") = py::none())
        .def("search", &MadhavaL2::search_one, py::arg("query"))
        .def("search_exact", &MadhavaL2::search_one, py::arg("query"))
        // Audits on the exact engine (mdh_audit_f32): the certificate covers
        // the returned top k (stage "in_topk") and the excluded rows nearest
        // the threshold (stage "exact": their exact value is the bound that
        // excludes them), at most max_audit_records of those; audit_excluded
        // counts every row strictly worse than the k-th result, from a second
        // GPU pass over all rows with that threshold.
        .def(
            "search_audited",
            [](const MadhavaL2& self, const F32Array& q, int64_t k, int64_t max_audit_records) -> py::dict {
                auto r = self.audit_one(q, k, max_audit_records);
                py::dict d;
                py::list audit;
                std::vector<int> idx;
                for (int j = 0; j < r.k; j++)
                    if (r.ids[(size_t)j] >= 0) idx.push_back(r.ids[(size_t)j]);
                for (int j = 0; j < r.a.n_records; j++) {
                    py::dict rd;
                    const double v = r.rec_vals[(size_t)j];
                    rd["doc_id"] = (int64_t)r.rec_ids[(size_t)j];
                    rd["true_cosine"] = v;
                    rd["projected_cosine"] = v;
                    rd["residual_norm"] = 0.0;
                    rd["upper_bound"] = v;
                    rd["threshold"] = r.a.threshold;
                    rd["excluded"] = true;
                    rd["stage"] = "exact";
                    audit.append(rd);
                }
                for (int j = 0; j < (int)idx.size(); j++) {
                    py::dict rd;
                    rd["doc_id"] = (int64_t)idx[(size_t)j];
                    rd["true_cosine"] = (double)r.vals[(size_t)j];
                    rd["projected_cosine"] = 0.0;
                    rd["residual_norm"] = 0.0;
                    rd["upper_bound"] = 0.0;
                    rd["threshold"] = r.a.threshold;
                    rd["excluded"] = false;
                    rd["stage"] = "in_topk";
                    audit.append(rd);
                }
                d["indices"] = idx;
                d["latency_ms"] = r.st.latency_ms;
                d["bound_violations"] = r.a.violations;
                d["bound_pairs"] = r.a.rows;
                d["audit_candidates"] = r.a.rows;
                d["audit_excluded"] = r.a.excluded;
                d["audit_excluded_by_bound"] = r.a.excluded_by_bound;
                d["audit_threshold"] = r.a.threshold;
                d["audit"] = audit;
                return d;
            },
            py::arg("query"), py::arg("k") = 10, py::arg("max_audit_records") = 500)
        .def(
            "audit_json",
            [](const MadhavaL2& self, const F32Array& q, int64_t k, int64_t max_audit_records) -> std::string {
                auto r = self.audit_one(q, k, max_audit_records);
                auto num = [](double x) {
                    char b[64];
                    std::snprintf(b, sizeof(b), "%f", x);
                    return std::string(b);
                };
                std::string j = "{\n  \"query_id\": \"madhava_audit\",\n";
                j += "  \"latency_ms\": " + num(r.st.latency_ms) + ",\n";
                j += "  \"bound_violations\": " + std::to_string(r.a.violations) + ",\n";
                j += "  \"audit_excluded\": " + std::to_string(r.a.excluded) + ",\n";
                j += "  \"results\": [";
                int rank = 0;
                for (int i = 0; i < r.k; i++) {
                    if (r.ids[(size_t)i] < 0) continue;
                    if (rank > 0) j += ",";
                    j += "\n    {\"rank\": " + std::to_string(rank + 1) +
                         ", \"doc_id\": " + std::to_string(r.ids[(size_t)i]) + "}";
                    rank++;
                }
                j += "\n  ],\n  \"audit_trail\": [\n";
                int count = 0;
                auto rec = [&](int64_t id, double v, double ub, bool excl, const char* stage) {
                    if (count++ > 0) j += ",\n";
                    j += "    {\"doc_id\": " + std::to_string(id) + ", \"true_cosine\": " + num(v) +
                         ", \"upper_bound\": " + num(ub) + ", \"threshold\": " + num(r.a.threshold) +
                         ", \"excluded\": " + (excl ? "true" : "false") + ", \"stage\": \"" + stage + "\"}";
                };
                for (int i = 0; i < r.a.n_records; i++)
                    rec(r.rec_ids[(size_t)i], r.rec_vals[(size_t)i], r.rec_vals[(size_t)i], true, "exact");
                for (int i = 0; i < r.k; i++)
                    if (r.ids[(size_t)i] >= 0) rec(r.ids[(size_t)i], r.vals[(size_t)i], 0.0, false, "in_topk");
                j += "\n  ]\n}\n";
                return j;
            },
            py::arg("query"), py::arg("k") = 10, py::arg("max_audit_records") = 500)
        .def(
            "search_with_commitment",
            [](const MadhavaL2& self, const F32Array& q, int64_t k, int64_t max_sample) -> py::dict {
                auto r = self.audit_one(q, k, max_sample);
                py::dict d;
                std::vector<int> idx;
                for (int j = 0; j < r.k; j++)
                    if (r.ids[(size_t)j] >= 0) idx.push_back(r.ids[(size_t)j]);
                d["indices"] = idx;
                d["bound_pairs"] = r.a.rows;
                d["bound_violations"] = r.a.violations;
                d["latency_ms"] = r.st.latency_ms;
                d["total_excluded_count"] = r.a.excluded;
                d["excluded_by_bound"] = r.a.excluded_by_bound;
                d["global_threshold"] = r.a.threshold;
                py::list samples;
                for (int j = 0; j < r.a.n_records; j++) {
                    py::dict sd;
                    sd["doc_id"] = (int64_t)r.rec_ids[(size_t)j];
                    sd["upper_bound"] = (double)r.rec_vals[(size_t)j];
                    sd["excluded"] = true;
                    samples.append(sd);
                }
                d["sampled_records"] = samples;
                return d;
            },
            py::arg("query"), py::arg("k") = 10, py::arg("max_sample") = 50)
        .def("search_batch", &MadhavaL2::search_batch, py::arg("queries"), py::arg("nq"), py::arg("k"))
        .def("save_index", &MadhavaL2::save_index, py::arg("path"))
        .def("load_index", &MadhavaL2::load_index, py::arg("path"))
        .def("num_vectors", &MadhavaL2::num_vectors)
        .def("dim", &MadhavaL2::dim)
        .def("config", &MadhavaL2::config)
        .def("build_seconds", &MadhavaL2::build_seconds)
        .def("built", &MadhavaL2::built)
        .def("basis1", [](const MadhavaL2&) -> py::array { not_implemented("MadhavaL2.basis1: the exact engine has no projection basis"); })
        .def("basis2", [](const MadhavaL2&) -> py::array { not_implemented("MadhavaL2.basis2: the exact engine has no projection basis"); })
        .def("residuals1", [](const MadhavaL2&) -> py::array { not_implemented("MadhavaL2.residuals1: the exact engine has no projection residuals"); })
        .def("residuals2", [](const MadhavaL2&) -> py::array { not_implemented("MadhavaL2.residuals2: the exact engine has no projection residuals"); })
        .def("_set_devices", [](MadhavaL2& self, py::object d) { self.set_devices(parse_devices(d)); }, py::arg("devices"));

    py::class_<IvfIndex>(m, "IvfIndex")
        .def(py::init<const U8Array&, const F32Array&, py::array_t<int32_t, py::array::c_style | py::array::forcecast>,
                      int, int>(),
             py::arg("corpus"), py::arg("centroids"), py::arg("labels"), py::arg("device") = -1,
             py::arg("metric") = 1)
        .def("search", &IvfIndex::search, py::arg("queries"), py::arg("k"), py::arg("nprobe"))
        .def("route", &IvfIndex::route, py::arg("queries"), py::arg("nprobe"))
        .def("num_vectors", &IvfIndex::num_vectors)
        .def("nlist", &IvfIndex::nlist);

    py::class_<IvfIndexF32>(m, "IvfIndexF32")
        .def(py::init<const F32Array&, const F32Array&, py::array_t<int32_t, py::array::c_style | py::array::forcecast>,
                      int>(),
             py::arg("corpus"), py::arg("centroids"), py::arg("labels"), py::arg("device") = -1)
        .def("search", &IvfIndexF32::search, py::arg("queries"), py::arg("k"), py::arg("nprobe"))
        .def("num_vectors", &IvfIndexF32::num_vectors)
        .def("nlist", &IvfIndexF32::nlist);

    py::class_<SpeedEngine>(m, "SpeedEngine")
        .def(py::init([](py::array_t<float, py::array::c_style> arr, int dim, int metric, int n_anchors, int nprobe,
                         bool require_gpu, const std::string& opencl_lib, py::object devices) {
                 (void)n_anchors; (void)nprobe; (void)require_gpu; (void)opencl_lib;
                 auto info = arr.request();
                 return new SpeedEngine(info.ptr, true, (int)info.shape[0], dim, metric, parse_devices(devices));
             }),
             py::arg("corpus_f32"), py::arg("dim"), py::arg("metric"), py::arg("n_anchors") = 0, py::arg("nprobe") = 4,
             py::arg("require_gpu") = false, py::arg("opencl_lib") = "", py::arg("devices") = py::none())
        .def(py::init([](py::array_t<uint8_t, py::array::c_style> arr, int dim, int metric, int n_anchors, int nprobe,
                         bool require_gpu, const std::string& opencl_lib, py::object devices) {
                 (void)n_anchors; (void)nprobe; (void)require_gpu; (void)opencl_lib;
                 auto info = arr.request();
                 return new SpeedEngine(info.ptr, false, (int)info.shape[0], dim, metric, parse_devices(devices));
             }),
             py::arg("corpus_u8"), py::arg("dim"), py::arg("metric"), py::arg("n_anchors") = 0, py::arg("nprobe") = 4,
             py::arg("require_gpu") = false, py::arg("opencl_lib") = "", py::arg("devices") = py::none())
        .def("search", &SpeedEngine::search, py::arg("query"), py::arg("k"))
        .def("search_batch", &SpeedEngine::search_batch, py::arg("queries"), py::arg("nq"), py::arg("k"))
        .def("num_vectors", &SpeedEngine::num_vectors)
        .def("dim", &SpeedEngine::dim)
        .def("has_gpu", [](const SpeedEngine&) { return true; })
        .def("backend_name", [](const SpeedEngine&) { return "gpu"; })
        .def("gpu_reason", [](const SpeedEngine&) { return std::string(); });

    m.def("recall_at_k", &recall_at_k, py::arg("result"), py::arg("gt_set"), py::arg("k"));
    m.def("ndcg_at_k", &ndcg_at_k, py::arg("result"), py::arg("gt_set"), py::arg("k"));
    m.def("l2_sq", &l2_sq, py::arg("v_raw"), py::arg("q"), py::arg("dim"));
    m.def("read_bigann_groundtruth", &read_bigann_groundtruth, py::arg("path"), py::arg("n_queries"));
    m.def("device_count", &mdh_device_count);
    m.def("version", &mdh_version);
    m.def("set_scan_path", [](int p) { check(mdh_set_scan_path(p)); }, py::arg("path"));
    m.def("set_verify", [](int n) { check(mdh_set_verify(n)); }, py::arg("max_queries"),
          "Re-check up to max_queries queries of every search with an exact unpruned scan; misplaced rows are "
          "counted in bound_violations (0 = off).");
}
