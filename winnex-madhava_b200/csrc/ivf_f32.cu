// Clustered (IVF) search over a float32 corpus: MadHybrid's float path
// (python/winnex_madhava/__init__.py:547-654).  The reference routes a query
// to the nprobe cells with the largest centroid inner product (:631-632),
// scores each probed cell's rows by the float64 inner product vecs @ q
// (:526, after an approximate per-cell cascade) and merges the cells by that
// score (:650).  Here every row of the probed cells is scored, so the result
// is the exact top k of their union by (score descending, row id ascending).
//
// Layout: rows in cell order (within a cell, by row id), with each position's
// row id and the cells' first positions.  Search, per batch of queries:
//   1. k_route_sims_f32: fp64 query . centroid, one fused multiply-add per
//      dimension in dimension order (the u8 IVF's routing arithmetic);
//   2. k_route_top_f32: a warp per query takes the nprobe largest, ties to the
//      lower cell id;
//   3. k_ivf_f32_topk: a block per query scores the rows of its cells (fp64,
//      dimension order), each thread keeps its best kIvfF32MaxK, and the
//      block merges them by (score, id).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"

struct mdh_ivf_f32 {
    int device = 0;
    cudaStream_t stream = nullptr;
    int64_t n = 0;
    int32_t dim = 0;
    int32_t nlist = 0;
    float* rows = nullptr;         // [n][dim], cell-major
    int32_t* ids = nullptr;        // [n] row id of each position
    int64_t* cell_start = nullptr; // [nlist + 1]
    float* centroids = nullptr;    // [nlist][dim]
    std::vector<int64_t> h_cell_start;
    // search scratch
    float* q = nullptr;       size_t q_bytes = 0;
    double* sims = nullptr;   size_t sims_bytes = 0;
    int32_t* probe = nullptr; size_t probe_bytes = 0;
    int32_t* out_id = nullptr; size_t out_id_bytes = 0;
    double* out_sc = nullptr; size_t out_sc_bytes = 0;
    std::mutex mu;
};

namespace mdh {
namespace {

constexpr int kIvfF32MaxK = 16;
constexpr int kIvfF32Threads = 256;
constexpr int kIvfF32MaxDim = 4096;

// Orders (score, id): higher score first, then the lower id.
__device__ __forceinline__ bool better(double s, int32_t i, double t, int32_t j) {
    return s > t || (s == t && i < j);
}

__global__ void k_route_sims_f32(const float* __restrict__ q, int nq, int dim, const float* __restrict__ cen,
                                 int nlist, double* __restrict__ sims) {
    const int qi = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (qi >= nq || c >= nlist) return;
    const float* qr = q + (size_t)qi * dim;
    const float* cr = cen + (size_t)c * dim;
    double acc = 0.0;
    for (int j = 0; j < dim; j++) acc = __fma_rn((double)__ldg(qr + j), (double)__ldg(cr + j), acc);
    sims[(size_t)qi * nlist + c] = acc;
}

__global__ void k_route_top_f32(double* __restrict__ sims, int nq, int nlist, int nprobe, int32_t* __restrict__ probe) {
    const int qi = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (qi >= nq) return;
    double* row = sims + (size_t)qi * nlist;
    for (int p = 0; p < nprobe; p++) {
        double bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < nlist; c += 32) {
            const double v = row[c];
            if (v > bv || (v == bv && c < bi)) {
                bv = v;
                bi = c;
            }
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, m);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) probe[(size_t)qi * nprobe + p] = bi;
        __syncwarp();
        if (lane == (bi & 31) && bi < nlist) row[bi] = -INFINITY;  // taken
        __syncwarp();
    }
}

// The warp's k best of its lanes' sorted lists (list[0] best), popped in
// order; lane r returns the r-th.  A popped head is replaced by the lane's
// next entry.
__device__ void warp_pop_k(double (&s)[kIvfF32MaxK], int32_t (&id)[kIvfF32MaxK], int k, double& out_s,
                           int32_t& out_id, int lane) {
    out_s = -INFINITY;
    out_id = -1;
    for (int r = 0; r < k; r++) {
        double bs = s[0];
        int32_t bi = id[0];
        int bl = lane;
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
            const double os = __shfl_xor_sync(0xffffffffu, bs, m);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, m);
            const int ol = __shfl_xor_sync(0xffffffffu, bl, m);
            if (better(os, oi, bs, bi) || (os == bs && oi == bi && ol < bl)) {
                bs = os;
                bi = oi;
                bl = ol;
            }
        }
        if (lane == r) {
            out_s = bs;
            out_id = bi;
        }
        if (lane == bl) {
#pragma unroll
            for (int j = 0; j < kIvfF32MaxK - 1; j++) {
                s[j] = s[j + 1];
                id[j] = id[j + 1];
            }
            s[kIvfF32MaxK - 1] = -INFINITY;
            id[kIvfF32MaxK - 1] = -1;
        }
    }
}

__global__ void __launch_bounds__(kIvfF32Threads) k_ivf_f32_topk(const float* __restrict__ rows,
                                                                 const int32_t* __restrict__ ids,
                                                                 const int64_t* __restrict__ cell_start,
                                                                 const float* __restrict__ q, int dim,
                                                                 const int32_t* __restrict__ probe, int nprobe, int k,
                                                                 int32_t* __restrict__ out_id,
                                                                 double* __restrict__ out_sc) {
    extern __shared__ double smem_d[];
    double* qs = smem_d;                                           // [dim]
    double* ws = qs + dim;                                         // [warps][k] scores
    int32_t* wi = reinterpret_cast<int32_t*>(ws + (kIvfF32Threads / 32) * kIvfF32MaxK);  // [warps][k] ids
    const int qi = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = threadIdx.x; j < dim; j += blockDim.x) qs[j] = (double)q[(size_t)qi * dim + j];
    __syncthreads();
    double s[kIvfF32MaxK];
    int32_t id[kIvfF32MaxK];
#pragma unroll
    for (int j = 0; j < kIvfF32MaxK; j++) {
        s[j] = -INFINITY;
        id[j] = -1;
    }
    for (int p = 0; p < nprobe; p++) {
        const int c = probe[(size_t)qi * nprobe + p];
        const int64_t r0 = cell_start[c], r1 = cell_start[c + 1];
        for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
            const float* v = rows + (size_t)r * dim;
            double acc = 0.0;
            for (int j = 0; j < dim; j++) acc = __fma_rn((double)__ldg(v + j), qs[j], acc);
            const int32_t gid = __ldg(ids + r);
            if (!better(acc, gid, s[k - 1], id[k - 1])) continue;
            // Insert into the descending list; the k-th entry drops out.
            int pos = k - 1;
            while (pos > 0 && better(acc, gid, s[pos - 1], id[pos - 1])) {
                s[pos] = s[pos - 1];
                id[pos] = id[pos - 1];
                pos--;
            }
            s[pos] = acc;
            id[pos] = gid;
        }
    }
    double bs;
    int32_t bi;
    warp_pop_k(s, id, k, bs, bi, lane);
    if (lane < k) {
        ws[warp * kIvfF32MaxK + lane] = bs;
        wi[warp * kIvfF32MaxK + lane] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        // Lanes 0..7 hold the warps' sorted lists; merge them the same way.
#pragma unroll
        for (int j = 0; j < kIvfF32MaxK; j++) {
            const bool have = lane < (kIvfF32Threads / 32) && j < k;
            s[j] = have ? ws[lane * kIvfF32MaxK + j] : -INFINITY;
            id[j] = have ? wi[lane * kIvfF32MaxK + j] : -1;
        }
        warp_pop_k(s, id, k, bs, bi, lane);
        if (lane < k) {
            out_sc[(size_t)qi * k + lane] = bi >= 0 ? bs : -INFINITY;
            out_id[(size_t)qi * k + lane] = bi;
        }
    }
}

template <class T>
void grow_buf(T** p, size_t* have, size_t need) {
    void* v = *p;
    ensure(&v, have, need);
    *p = static_cast<T*>(v);
}

void free_ivf_f32(mdh_ivf_f32* ix) {
    if (!ix) return;
    cudaSetDevice(ix->device);
    if (ix->stream) cudaStreamSynchronize(ix->stream);
    for (void* p : {(void*)ix->rows, (void*)ix->ids, (void*)ix->cell_start, (void*)ix->centroids, (void*)ix->q,
                    (void*)ix->sims, (void*)ix->probe, (void*)ix->out_id, (void*)ix->out_sc})
        if (p) cudaFree(p);
    if (ix->stream) cudaStreamDestroy(ix->stream);
    delete ix;
}

struct CreateArgs {
    const float* rows;
    int64_t n;
    int32_t dim;
    const float* cen;
    int32_t nlist;
    const int32_t* labels;
    int32_t device;
    mdh_ivf_f32** out;
};

void create_f32(void* p) {
    const CreateArgs& a = *static_cast<const CreateArgs*>(p);
    MDH_REQUIRE(a.out, MDH_ERR_INVALID_ARG, "null output pointer");
    *a.out = nullptr;
    MDH_REQUIRE(a.rows && a.cen && a.labels, MDH_ERR_INVALID_ARG, "null rows, centroids or labels");
    MDH_REQUIRE(a.n > 0 && a.n < (int64_t(1) << 31), MDH_ERR_INVALID_ARG, "n must be in [1, 2^31)");
    MDH_REQUIRE(a.dim > 0 && a.dim <= kIvfF32MaxDim, MDH_ERR_INVALID_ARG, "dim must be in [1, 4096]");
    MDH_REQUIRE(a.nlist > 0 && a.nlist <= 65536, MDH_ERR_INVALID_ARG, "nlist must be in [1, 65536]");
    const int dev = a.device < 0 ? 0 : a.device;
    check_device_usable(dev);
    // Cell-major order (stable: row ids ascend inside a cell).
    std::vector<int64_t> start((size_t)a.nlist + 1, 0);
    for (int64_t i = 0; i < a.n; i++) {
        MDH_REQUIRE(a.labels[i] >= 0 && a.labels[i] < a.nlist, MDH_ERR_INVALID_ARG,
                    "label out of range at row " + std::to_string(i));
        start[(size_t)a.labels[i] + 1]++;
    }
    for (int c = 0; c < a.nlist; c++) start[(size_t)c + 1] += start[(size_t)c];
    std::vector<int64_t> cur(start.begin(), start.end() - 1);
    std::vector<int32_t> pos_id((size_t)a.n);
    std::vector<float> perm((size_t)a.n * a.dim);
    for (int64_t i = 0; i < a.n; i++) {
        const int64_t at = cur[(size_t)a.labels[i]]++;
        pos_id[(size_t)at] = (int32_t)i;
        std::memcpy(perm.data() + (size_t)at * a.dim, a.rows + (size_t)i * a.dim, (size_t)a.dim * sizeof(float));
    }
    auto* ix = new mdh_ivf_f32();
    try {
        ix->device = dev;
        ix->n = a.n;
        ix->dim = a.dim;
        ix->nlist = a.nlist;
        ix->h_cell_start = start;
        MDH_CUDA(cudaSetDevice(dev));
        MDH_CUDA(cudaStreamCreateWithFlags(&ix->stream, cudaStreamNonBlocking));
        MDH_CUDA(cudaMalloc(&ix->rows, perm.size() * sizeof(float)));
        MDH_CUDA(cudaMalloc(&ix->ids, (size_t)a.n * 4));
        MDH_CUDA(cudaMalloc(&ix->cell_start, start.size() * 8));
        MDH_CUDA(cudaMalloc(&ix->centroids, (size_t)a.nlist * a.dim * sizeof(float)));
        MDH_CUDA(cudaMemcpy(ix->rows, perm.data(), perm.size() * sizeof(float), cudaMemcpyHostToDevice));
        MDH_CUDA(cudaMemcpy(ix->ids, pos_id.data(), (size_t)a.n * 4, cudaMemcpyHostToDevice));
        MDH_CUDA(cudaMemcpy(ix->cell_start, start.data(), start.size() * 8, cudaMemcpyHostToDevice));
        MDH_CUDA(cudaMemcpy(ix->centroids, a.cen, (size_t)a.nlist * a.dim * sizeof(float), cudaMemcpyHostToDevice));
    } catch (...) {
        free_ivf_f32(ix);
        throw;
    }
    *a.out = ix;
}

struct SearchArgs {
    mdh_ivf_f32* ix;
    const float* q;
    int32_t nq, k, nprobe;
    int32_t* out_ids;
    double* out_scores;
    mdh_stats* stats;
};

void search_f32(void* p) {
    const SearchArgs& a = *static_cast<const SearchArgs*>(p);
    const auto t0 = std::chrono::high_resolution_clock::now();
    mdh_ivf_f32* ix = a.ix;
    MDH_REQUIRE(ix, MDH_ERR_INVALID_ARG, "null index");
    MDH_REQUIRE(a.nq >= 0, MDH_ERR_INVALID_ARG, "nq must be >= 0");
    MDH_REQUIRE(a.k >= 1 && a.k <= kIvfF32MaxK, MDH_ERR_UNSUPPORTED, "k must be in [1, 16] for a float IVF index");
    MDH_REQUIRE(a.nprobe >= 1, MDH_ERR_INVALID_ARG, "nprobe must be >= 1");
    MDH_REQUIRE(a.nq == 0 || (a.q && a.out_ids), MDH_ERR_INVALID_ARG, "null queries or output ids");
    std::lock_guard<std::mutex> lock(ix->mu);
    mdh_stats st{};
    const int nprobe = std::min(a.nprobe, ix->nlist);
    if (a.nq > 0) {
        MDH_CUDA(cudaSetDevice(ix->device));
        cudaStream_t s = ix->stream;
        const int nq = a.nq, k = a.k, dim = ix->dim, nlist = ix->nlist;
        grow_buf(&ix->q, &ix->q_bytes, (size_t)nq * dim * sizeof(float));
        grow_buf(&ix->sims, &ix->sims_bytes, (size_t)nq * nlist * sizeof(double));
        grow_buf(&ix->probe, &ix->probe_bytes, (size_t)nq * nprobe * 4);
        grow_buf(&ix->out_id, &ix->out_id_bytes, (size_t)nq * k * 4);
        grow_buf(&ix->out_sc, &ix->out_sc_bytes, (size_t)nq * k * sizeof(double));
        MDH_CUDA(cudaMemcpyAsync(ix->q, a.q, (size_t)nq * dim * sizeof(float), cudaMemcpyHostToDevice, s));
        k_route_sims_f32<<<dim3((unsigned)((nlist + 127) / 128), (unsigned)nq), 128, 0, s>>>(ix->q, nq, dim,
                                                                                           ix->centroids, nlist,
                                                                                           ix->sims);
        MDH_CUDA(cudaGetLastError());
        k_route_top_f32<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(ix->sims, nq, nlist, nprobe, ix->probe);
        MDH_CUDA(cudaGetLastError());
        const size_t smem = (size_t)dim * sizeof(double) + (kIvfF32Threads / 32) * kIvfF32MaxK * (8 + 4);
        MDH_REQUIRE(smem <= 48 * 1024 || cudaFuncSetAttribute(k_ivf_f32_topk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                              (int)smem) == cudaSuccess,
                    MDH_ERR_UNSUPPORTED, "dimension too large for the float IVF scan");
        k_ivf_f32_topk<<<(unsigned)nq, kIvfF32Threads, smem, s>>>(ix->rows, ix->ids, ix->cell_start, ix->q, dim,
                                                                 ix->probe, nprobe, k, ix->out_id, ix->out_sc);
        MDH_CUDA(cudaGetLastError());
        std::vector<int32_t> probe((size_t)nq * nprobe);
        MDH_CUDA(cudaMemcpyAsync(a.out_ids, ix->out_id, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, s));
        if (a.out_scores)
            MDH_CUDA(cudaMemcpyAsync(a.out_scores, ix->out_sc, (size_t)nq * k * sizeof(double), cudaMemcpyDeviceToHost,
                                     s));
        MDH_CUDA(cudaMemcpyAsync(probe.data(), ix->probe, probe.size() * 4, cudaMemcpyDeviceToHost, s));
        MDH_CUDA(cudaStreamSynchronize(s));
        // Pairs scored: the rows of every probed cell.
        for (size_t i = 0; i < probe.size(); i++) {
            const int c = probe[i];
            if (c >= 0 && c < nlist) st.pairs_scored += ix->h_cell_start[(size_t)c + 1] - ix->h_cell_start[(size_t)c];
        }
        st.full_scan_pairs = st.pairs_scored;
        st.kernel_launches = 3;
        st.levels = 1;
    }
    st.latency_ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t0).count();
    if (a.stats) *a.stats = st;
}

}  // namespace
}  // namespace mdh

using namespace mdh;

extern "C" {

mdh_status mdh_ivf_create_f32(const float* host_rows, int64_t n, int32_t dim, const float* centroids, int32_t nlist,
                              const int32_t* labels, int32_t device, mdh_ivf_f32** out) {
    CreateArgs a{host_rows, n, dim, centroids, nlist, labels, device, out};
    return run_guarded(create_f32, &a);
}

mdh_status mdh_ivf_search_f32(mdh_ivf_f32* index, const float* host_queries, int32_t nq, int32_t k, int32_t nprobe,
                              int32_t* out_ids, double* out_scores, mdh_stats* stats) {
    SearchArgs a{index, host_queries, nq, k, nprobe, out_ids, out_scores, stats};
    return run_guarded(search_f32, &a);
}

mdh_status mdh_ivf_destroy_f32(mdh_ivf_f32* index) {
    return run_guarded([](void* p) { free_ivf_f32(static_cast<mdh_ivf_f32*>(p)); }, index);
}

}  // extern "C"
