// Clustered (IVF) exact L2 search over a u8 corpus: the GPU form of
// MadHybrid's uint8 path (python/winnex_madhava/__init__.py:547-654).
//
// Semantics: a query is routed to the nprobe cells whose centroids have the
// largest inner product with it (the reference's `centroids @ q`,
// __init__.py:631-632; here in fp64 with a fixed multiply-add order and ties
// to the lower cell id), and the result is the exact top-k over the union of
// those cells' rows, ranked by (squared L2 distance, row id).
//
// Layout: rows are grouped by cell (cell-major), sorted by (|v|^2, id)
// inside a cell, and every cell starts on a 256-row boundary (pad rows: zero
// bytes, norm 2^30, id -1).  So a cell is a run of whole corpus tiles and
// every 32-row chunk of it starts with its smallest norm, which the tensor
// scan's chunk bound needs.
//
// Search, per batch of queries:
//   1. route (k_route_sims, k_route_select): fp64 dot products with every
//      centroid, top nprobe;
//   2. pass 0: each query against a coarse sample of its cells (rows whose
//      id hashes below 1/256, and the 2 lowest-norm rows of each cell) with
//      an infinite threshold; the k-th smallest (key, id) is a valid
//      threshold for the union (the sample is part of it);
//   3. pass 1: each query against a finer sample (1/32, and the 8
//      lowest-norm rows of each cell) with that threshold; its k-th smallest
//      candidate tightens the threshold so that about 32 k of the union's
//      rows lie at or below it;
//   4. pass 2: each query against all its cells with that threshold; the
//      candidates' first k are exact.  Overflowed lists rerun with their
//      k-th stored entry, strictly tighter, until they fit.
// Every pass runs the tcgen05 scan (scan_tc.cu) over a unit table: a unit
// is one cell (or a run of at most 64 of its tiles) against up to 128 of the
// queries that probe it, gathered into one query matrix.  The coarse pass
// keeps the first sample pass from handling every sampled pair as a
// candidate.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <chrono>
#include <cstring>
#include <string>
#include <vector>

#include "internal.h"

namespace mdh {
// Device buffers of one IVF pass: gathered query matrix, its norms, its map
// to batch queries, and the unit table.
struct IvfPassBufs {
    uint8_t* g = nullptr;      size_t g_bytes = 0;
    int32_t* gqn = nullptr;    size_t gqn_bytes = 0;
    int32_t* gmap = nullptr;   size_t gmap_bytes = 0;
    ScanUnit* units = nullptr; size_t units_bytes = 0;
    void free_all() {
        for (void* p : {(void*)g, (void*)gqn, (void*)gmap, (void*)units})
            if (p) cudaFree(p);
        *this = IvfPassBufs();
    }
};
}  // namespace mdh

struct mdh_ivf {
    int device = 0;
    cudaStream_t stream = nullptr;
    int64_t n = 0;
    int32_t dim = 0;
    int32_t dpad = 0;
    int32_t nlist = 0;
    int32_t metric = MDH_METRIC_L2;      // L2, or COSINE: rank by the inner product q.v
    mdh::Level rows;                     // all cells, padded
    std::vector<int64_t> cell_start;     // first row of cell c
    std::vector<int64_t> cell_count;     // real rows of cell c
    mdh::Level sample;                   // per-cell samples (1/32), same layout
    std::vector<int64_t> sample_start;
    std::vector<int64_t> sample_count;
    mdh::Level coarse;                   // per-cell coarse samples (1/256), same layout
    std::vector<int64_t> coarse_start;
    std::vector<int64_t> coarse_count;
    float* centroids = nullptr;          // [nlist][dim]
    mdh::Workspace ws;
    mdh::IvfPassBufs pass[3];            // coarse samples, samples, whole cells (pass[2] holds the query matrix)
    // Device-side planning: per cell and pass {first tile, tiles, row end} of
    // the pass's layout; the cells in planning order (most tiles first);
    // scratch for the plan (query counts, fill cursors, query offsets, unit
    // offsets of each pass, table lengths) and pair counts.
    int32_t* plan_info = nullptr;        // [nlist][3 passes][3]
    int32_t* plan_order = nullptr;       // [nlist]
    int32_t* plan_scratch = nullptr;     // [6 * nlist + 3 + 1]
    unsigned long long* plan_pairs = nullptr;  // [3]
    int64_t unit_max_runs[3] = {0, 0, 0};  // per pass: max over cells of ceil(tiles / 64)
    int64_t unit_sum_runs[3] = {0, 0, 0};  // per pass: sum over cells of ceil(tiles / 64)
    // Passing chunks of the deferred scans (mdh::ChunkOut): 32 dot products
    // and a header per entry.
    uint4* chunk_x = nullptr;  size_t chunk_x_bytes = 0;
    int4* chunk_hdr = nullptr; size_t chunk_hdr_bytes = 0;
    std::mutex mu;
};

namespace mdh {

namespace {

constexpr int kIvfTileRows = 256;     // tile of the tensor scan (CfgNarrow::BN)
constexpr int kIvfMaxTilesPerUnit = 64;
constexpr int kIvfMaxNlist = 8192;
constexpr int kIvfMaxProbe = 1024;
constexpr int kIvfPasses = 3;         // coarse samples, samples, whole cells
constexpr int kIvfCap0 = 4096;        // coarse-sample pass candidate lists
constexpr int kIvfCap1 = 16384;       // sample pass candidate lists
constexpr uint32_t kIvfSampleThresh = 0x08000000u;  // id hash below this: in the sample (1/32)
constexpr int kIvfSampleHead = 8;     // lowest-norm rows of every cell always in the sample
constexpr uint32_t kIvfCoarseThresh = 0x01000000u;  // ... in the coarse sample (1/256)
constexpr int kIvfCoarseHead = 2;
constexpr int kIvfCap2 = 16384;       // pass 2 candidate lists
// Chunk-buffer entries per query of a deferred pass, plus two partly used
// 64-entry blocks per epilogue warp.  Config-5 queries (10M rows, nlist 1024,
// nprobe 16) leave about 300 chunks each to pass 2.  A pass that needs more
// reruns pass 2 with keys formed in the scan.
constexpr int kIvfChunksPerQuery = 512;
// Inner-product ranking (metric COSINE) runs the L2 scan with every row norm
// set to 0 and every query norm to this offset: the key offset - 2 q.v is then
// positive (2 q.v <= 2 * 128 * 255^2 < 2^24 for dim <= 128) and ascends as
// q.v descends; the chunk bound (first norm 0) stays exact.
constexpr int32_t kIvfIpOffset = 1 << 24;

template <class T>
T* dalloc(size_t count) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, count * sizeof(T) + 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw Error(MDH_ERR_OOM, std::string("device allocation failed: ") + cudaGetErrorString(e));
    }
    return static_cast<T*>(p);
}

// key = label << 32 | |v|^2 for row r (8 lanes per row); value = r.
__global__ void k_ivf_keys(const uint8_t* __restrict__ rows, const int32_t* __restrict__ labels, int64_t n, int dpad,
                           unsigned long long* __restrict__ keys, int32_t* __restrict__ vals) {
    const int lane = threadIdx.x & 31;
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l8 = lane & 7;
    uint32_t s = 0;
    if (r < n) {
        const uint8_t* row = rows + (size_t)r * dpad;
        for (int off = l8 * 16; off < dpad; off += 128) {
            uint4 v = *reinterpret_cast<const uint4*>(row + off);
            s = __dp4a(v.x, v.x, s);
            s = __dp4a(v.y, v.y, s);
            s = __dp4a(v.z, v.z, s);
            s = __dp4a(v.w, v.w, s);
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (r < n && l8 == 0) {
        keys[r] = ((unsigned long long)(uint32_t)labels[r] << 32) | (unsigned long long)s;
        vals[r] = (int32_t)r;
    }
}

// Sorted position p (cell l = key >> 32) goes to row cell_start[l] + p - cell_first[l].
__global__ void k_ivf_gather(const uint8_t* __restrict__ src, const unsigned long long* __restrict__ keys,
                             const int32_t* __restrict__ vals, int64_t n, int dpad,
                             const int64_t* __restrict__ cell_start, const int64_t* __restrict__ cell_first,
                             uint8_t* __restrict__ rows, int32_t* __restrict__ norms, int32_t* __restrict__ ids,
                             int zero_norms) {
    const int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l8 = threadIdx.x & 7;
    if (p >= n) return;
    const unsigned long long key = keys[p];
    const int l = (int)(key >> 32);
    const int64_t dst = cell_start[l] + (p - cell_first[l]);
    const int64_t s = vals[p];
    for (int off = l8 * 16; off < dpad; off += 128)
        *reinterpret_cast<uint4*>(rows + (size_t)dst * dpad + off) =
            *reinterpret_cast<const uint4*>(src + (size_t)s * dpad + off);
    if (l8 == 0) {
        norms[dst] = zero_norms ? 0 : (int32_t)(key & 0xffffffffull);
        ids[dst] = (int32_t)s;
    }
}

// Sample row p copies main row pos[p] (pos -1: a pad row).
__global__ void k_ivf_gather_rows(const int32_t* __restrict__ pos, int64_t m, int dpad,
                                  const uint8_t* __restrict__ src_rows, const int32_t* __restrict__ src_norms,
                                  const int32_t* __restrict__ src_ids, uint8_t* __restrict__ rows,
                                  int32_t* __restrict__ norms, int32_t* __restrict__ ids) {
    const int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l8 = threadIdx.x & 7;
    if (p >= m) return;
    const int32_t s = pos[p];
    for (int off = l8 * 16; off < dpad; off += 128)
        *reinterpret_cast<uint4*>(rows + (size_t)p * dpad + off) =
            s >= 0 ? *reinterpret_cast<const uint4*>(src_rows + (size_t)s * dpad + off) : make_uint4(0, 0, 0, 0);
    if (l8 == 0) {
        norms[p] = s >= 0 ? src_norms[s] : kNormPad;
        ids[p] = s >= 0 ? src_ids[s] : -1;
    }
}

uint32_t sample_hash_host(int32_t id) {
    uint64_t z = (uint64_t)(uint32_t)id + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (uint32_t)(z >> 32);
}

__global__ void k_ivf_fill(int32_t* __restrict__ p, int64_t n, int32_t v) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// Routing, step 1: sims[q][c] = sum_j q[j] * centroid[c][j] in fp64, one
// fused multiply-add per j in dimension order from 0.0 (deterministic, so the
// cell order is reproducible).  Block tile: 64 queries x 64 centroids in
// shared memory, stored by dimension (row j holds the tile's 64 values of
// dimension j): the queries converted to fp64 once, the centroids kept in
// fp32 and widened as they are read (exact either way).  Each thread forms
// the 4 x 4 dot products of 4 consecutive queries and 4 consecutive
// centroids, so a step of j is three vector loads (two double2, one float4)
// for 16 multiply-adds.  The kernel is bound by the latency of its shared
// loads: the fp32 centroid tile lets two blocks share an SM (with fp64 tiles
// and one block per SM it ran 1.65x longer), and the vector loads took it
// from 181 to 162 us against 8 scalar loads per step.  Rows of the tiles are
// 66 doubles and 68 floats long, multiples of 16 bytes.
constexpr int kRouteQ = 64, kRouteC = 64, kRouteDim = 128;
constexpr int kRouteQS = kRouteQ + 2, kRouteCS = kRouteC + 4;
constexpr size_t kRouteSmem = (size_t)kRouteDim * kRouteQS * sizeof(double) +
                              (size_t)kRouteDim * kRouteCS * sizeof(float);
__global__ void __launch_bounds__(256) k_route_sims(const uint8_t* __restrict__ q, int nq, int dpad, int dim,
                                                    const float* __restrict__ centroids, int nlist,
                                                    double* __restrict__ sims) {
    extern __shared__ __align__(16) double route_smem[];
    double* qs = route_smem;                                                // [dim][kRouteQS]
    float* cs = reinterpret_cast<float*>(route_smem + kRouteDim * kRouteQS);  // [dim][kRouteCS]
    const int q0 = blockIdx.y * kRouteQ, c0 = blockIdx.x * kRouteC;
    // A warp per row, lanes along the row (coalesced, no index division).
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    for (int c = warp; c < kRouteC; c += nwarps) {
        const bool have = c0 + c < nlist;
        const float* src = centroids + (size_t)(c0 + c) * dim;
        for (int j = lane; j < dim; j += 32) cs[j * kRouteCS + c] = have ? __ldg(src + j) : 0.0f;
    }
    for (int r = warp; r < kRouteQ; r += nwarps) {
        const bool have = q0 + r < nq;
        const uint8_t* src = q + (size_t)(q0 + r) * dpad;
        for (int j = lane; j < dim; j += 32) qs[j * kRouteQS + r] = have ? (double)__ldg(src + j) : 0.0;
    }
    __syncthreads();
    // Thread: queries 4 rp + a and centroids 4 cq + b (a, b < 4).  A warp
    // reads 16 consecutive float4 of the centroid row and broadcasts two
    // query double2 pairs.
    const int cq = threadIdx.x & 15, rp = threadIdx.x >> 4;
    double acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) acc[a][b] = 0.0;
    for (int j = 0; j < dim; j++) {
        const double2 qa = *reinterpret_cast<const double2*>(qs + j * kRouteQS + 4 * rp);
        const double2 qb = *reinterpret_cast<const double2*>(qs + j * kRouteQS + 4 * rp + 2);
        const float4 cf = *reinterpret_cast<const float4*>(cs + j * kRouteCS + 4 * cq);
        const double qv[4] = {qa.x, qa.y, qb.x, qb.y};
        const double cv[4] = {(double)cf.x, (double)cf.y, (double)cf.z, (double)cf.w};
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
            for (int b = 0; b < 4; b++) acc[a][b] = __fma_rn(qv[a], cv[b], acc[a][b]);
    }
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 4; b++) {
            const int qi = q0 + 4 * rp + a, c = c0 + 4 * cq + b;
            if (qi < nq && c < nlist) sims[(size_t)qi * nlist + c] = acc[a][b];
        }
}

// Routing, step 2: one warp per query takes the nprobe largest similarities,
// ties to the lower cell id, best first.
__global__ void __launch_bounds__(256) k_route_select(double* __restrict__ sims, int nq, int nlist, int nprobe,
                                                      int32_t* __restrict__ probe) {
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
        if (lane == (bi & 31)) row[bi] = -INFINITY;  // taken
        __syncwarp();
    }
}

// (x, c) ranks before (y, d): larger similarity, then the lower cell id.
__device__ __forceinline__ bool route_before(double x, int c, double y, int d) { return x > y || (x == y && c < d); }

// Lane l's kRouteList best cells (of l, l + 32, ...) ranked after (av, ac),
// best first; empty slots hold (-inf, INT_MAX).  Each cell is inserted by
// the full (similarity, id) order: an entry it displaces can tie with a later
// one of higher id and must still move ahead of it.
constexpr int kRouteList = 4;
template <int PER>
__device__ __forceinline__ void route_lane_list(const double (&v)[PER], int lane, int nlist, double av, int ac,
                                                double (&hv)[kRouteList], int (&hc)[kRouteList]) {
#pragma unroll
    for (int s = 0; s < kRouteList; s++) {
        hv[s] = -INFINITY;
        hc[s] = 0x7fffffff;
    }
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int c = lane + 32 * i;
        if (c >= nlist || !route_before(av, ac, v[i], c)) continue;
        double tv = v[i];
        int tc = c;
#pragma unroll
        for (int s = 0; s < kRouteList; s++) {
            if (route_before(tv, tc, hv[s], hc[s])) {
                const double xv = hv[s];
                const int xc = hc[s];
                hv[s] = tv;
                hc[s] = tc;
                tv = xv;
                tc = xc;
            }
        }
    }
}

// The same selection with the row held in registers (nlist <= 32 * PER):
// lane l holds cells l, l + 32, ..., and keeps a sorted list of its best
// kRouteList.  Each round the warp takes the best of the lists' heads
// (largest similarity, lower id on ties) and its lane pops it; a lane whose
// list runs out rebuilds it from the cells ranked after its last pop.  A
// round is one warp argmax, not a pass over every lane's PER values.
template <int PER>
__global__ void __launch_bounds__(256) k_route_select_reg(const double* __restrict__ sims, int nq, int nlist,
                                                          int nprobe, int32_t* __restrict__ probe) {
    const int qi = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (qi >= nq) return;
    const double* row = sims + (size_t)qi * nlist;
    double v[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) {
        const int c = lane + 32 * i;
        v[i] = c < nlist ? row[c] : -INFINITY;
    }
    double hv[kRouteList];
    int hc[kRouteList];
    route_lane_list(v, lane, nlist, INFINITY, -1, hv, hc);
    for (int p = 0; p < nprobe; p++) {
        double bv = hv[0];
        int bi = hc[0];
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, m);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
            if (route_before(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) probe[(size_t)qi * nprobe + p] = bi;
        if (bi == hc[0] && bi < nlist) {  // this lane's head was taken
            const double lv = hv[0];
#pragma unroll
            for (int s = 0; s + 1 < kRouteList; s++) {
                hv[s] = hv[s + 1];
                hc[s] = hc[s + 1];
            }
            hv[kRouteList - 1] = -INFINITY;
            hc[kRouteList - 1] = 0x7fffffff;
            if (hc[0] == 0x7fffffff) route_lane_list(v, lane, nlist, lv, bi, hv, hc);
        }
    }
}

void launch_route(const uint8_t* q, int nq, int dpad, int dim, const float* centroids, int nlist, int nprobe,
                  double* sims, int32_t* probe, cudaStream_t st) {
    if (nq <= 0) return;
    MDH_REQUIRE(dim <= kRouteDim, MDH_ERR_INTERNAL, "routing supports dim <= 128");
    dim3 grid((unsigned)((nlist + kRouteC - 1) / kRouteC), (unsigned)((nq + kRouteQ - 1) / kRouteQ));
    // A function attribute belongs to the current device: set it on every launch.
    MDH_CUDA(cudaFuncSetAttribute(k_route_sims, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRouteSmem));
    k_route_sims<<<grid, 256, kRouteSmem, st>>>(q, nq, dpad, dim, centroids, nlist, sims);
    MDH_CUDA(cudaGetLastError());
    if (nlist <= 32 * 32)
        k_route_select_reg<32><<<(unsigned)((nq * 32 + 255) / 256), 256, 0, st>>>(sims, nq, nlist, nprobe, probe);
    else
        k_route_select<<<(unsigned)((nq * 32 + 255) / 256), 256, 0, st>>>(sims, nq, nlist, nprobe, probe);
    MDH_CUDA(cudaGetLastError());
}

template <class T>
void grow_dev(T** p, size_t* have, size_t bytes) {
    void* v = *p;
    ensure(&v, have, bytes);
    *p = static_cast<T*>(v);
}

// ---------------------------------------------------------------- planning
// All passes probe the same cells, so they share one grouped query matrix
// (queries listed cell by cell) and differ in their unit tables.  The plan
// is built on the device from the routing output, so routing, planning and
// the passes run back to back on one stream.  The order of queries inside a
// cell's list depends on atomics; results do not (candidates are selected by
// (key, id)).  Pass p uses layout p: coarse samples, samples, whole cells.

constexpr int kPlanThreads = 1024;
constexpr int kPlanItems = kIvfMaxNlist / kPlanThreads;  // cells per thread in k_plan_scan
constexpr int kPlanCounters = 1 + kIvfPasses;            // queries, then units of each pass
static_assert(kPlanItems * kPlanThreads == kIvfMaxNlist, "plan scan covers every cell");

__global__ void k_plan_count(const int32_t* __restrict__ probe, int total, int32_t* __restrict__ cnt) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < total) atomicAdd(cnt + probe[i], 1);
}

// Block-wide exclusive scan of kPlanCounters counters (one block of kPlanThreads).
__device__ __forceinline__ void block_scan(int (&v)[kPlanCounters], int (&total)[kPlanCounters]) {
    __shared__ int wsum[kPlanCounters][kPlanThreads / 32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int incl[kPlanCounters];
#pragma unroll
    for (int j = 0; j < kPlanCounters; j++) {
        incl[j] = v[j];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl[j], o);
            if (lane >= o) incl[j] += t;
        }
        if (lane == 31) wsum[j][wid] = incl[j];
    }
    __syncthreads();
    if (wid == 0) {
#pragma unroll
        for (int j = 0; j < kPlanCounters; j++) {
            int x = wsum[j][lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += t;
            }
            wsum[j][lane] = x;  // inclusive over warps
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kPlanCounters; j++) {
        total[j] = wsum[j][kPlanThreads / 32 - 1];
        v[j] = incl[j] - v[j] + (wid > 0 ? wsum[j][wid - 1] : 0);
    }
}

// One block.  For every cell, taken in planning order: the offset of its
// query list in the grouped matrix (qstart) and of its first unit in each
// pass's table (ustart[pass][cell]); the tables' lengths (nunits[pass]) and
// the (query, row) pairs each pass scans (pairs[pass], zeroed by the caller).
// info[cell][pass] = {first tile, tiles, row end} of the pass's layout.
__global__ void __launch_bounds__(kPlanThreads)
    k_plan_scan(const int32_t* __restrict__ cnt, const int32_t* __restrict__ order, const int32_t* __restrict__ info,
                int nlist, int32_t* __restrict__ qstart, int32_t* __restrict__ ustart, int32_t* __restrict__ nunits,
                unsigned long long* __restrict__ pairs) {
    int item[kPlanItems][kPlanCounters];
    int sum[kPlanCounters] = {};
    unsigned long long pr[kIvfPasses] = {};
#pragma unroll
    for (int j = 0; j < kPlanItems; j++) {
        const int pos = threadIdx.x * kPlanItems + j;
        int x[kPlanCounters] = {};
        if (pos < nlist) {
            const int c = order[pos];
            const int qn = cnt[c];
            x[0] = qn;
            if (qn > 0) {
#pragma unroll
                for (int p = 0; p < kIvfPasses; p++) {
                    const int32_t* g = info + 9 * c + 3 * p;
                    if (g[1] > 0) {
                        x[1 + p] = (qn + 127) / 128 * ((g[1] + kIvfMaxTilesPerUnit - 1) / kIvfMaxTilesPerUnit);
                        pr[p] += (unsigned long long)qn * (unsigned long long)(g[2] - g[0] * kIvfTileRows);
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kPlanCounters; q++) {
            item[j][q] = x[q];
            sum[q] += x[q];
        }
    }
    int total[kPlanCounters];
    block_scan(sum, total);
#pragma unroll
    for (int j = 0; j < kPlanItems; j++) {
        const int pos = threadIdx.x * kPlanItems + j;
        if (pos < nlist) {
            const int c = order[pos];
            qstart[c] = sum[0];
#pragma unroll
            for (int p = 0; p < kIvfPasses; p++) ustart[p * nlist + c] = sum[1 + p];
        }
#pragma unroll
        for (int q = 0; q < kPlanCounters; q++) sum[q] += item[j][q];
    }
    if (threadIdx.x == 0)
#pragma unroll
        for (int p = 0; p < kIvfPasses; p++) nunits[p] = total[1 + p];
#pragma unroll
    for (int p = 0; p < kIvfPasses; p++) {
        unsigned long long x = pr[p];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if ((threadIdx.x & 31) == 0 && x) atomicAdd(pairs + p, x);
    }
}

// probe[i] = the j-th cell of query i / nprobe: list the query in its cell.
__global__ void k_plan_fill(const int32_t* __restrict__ probe, int total, int nprobe,
                            const int32_t* __restrict__ qstart, int32_t* __restrict__ fill,
                            int32_t* __restrict__ gmap) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int c = probe[i];
    gmap[qstart[c] + atomicAdd(fill + c, 1)] = i / nprobe;
}

struct PassUnits {
    ScanUnit* u[kIvfPasses];
};

// One thread per (cell, pass): the cell's units, runs of at most 64 tiles
// against at most 128 of its queries.
__global__ void k_plan_units(const int32_t* __restrict__ cnt, const int32_t* __restrict__ info,
                             const int32_t* __restrict__ qstart, const int32_t* __restrict__ ustart, int nlist,
                             PassUnits tables) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    const int p = blockIdx.y;
    if (c >= nlist) return;
    const int qn = cnt[c];
    const int32_t* g = info + 9 * c + 3 * p;
    const int tf = g[0], tiles = g[1], rend = g[2];
    if (qn == 0 || tiles == 0) return;
    ScanUnit* out = tables.u[p] + ustart[p * nlist + c];
    int k = 0;
    for (int q0 = 0; q0 < qn; q0 += 128)
        for (int t0 = 0; t0 < tiles; t0 += kIvfMaxTilesPerUnit) {
            ScanUnit u;
            u.q_row = qstart[c] + q0;
            u.q_count = min(128, qn - q0);
            u.t0 = tf + t0;
            u.t1 = tf + min(tiles, t0 + kIvfMaxTilesPerUnit);
            u.row_end = rend;
            u.pad = 0;
            out[k++] = u;
        }
}

// Per-cell planning facts, uploaded once per index.
void build_ivf_plan_info(mdh_ivf* ix, cudaStream_t st) {
    const int nl = ix->nlist;
    std::vector<int32_t> info((size_t)nl * 9);
    std::vector<int32_t> order((size_t)nl);
    const std::vector<int64_t>* starts[kIvfPasses] = {&ix->coarse_start, &ix->sample_start, &ix->cell_start};
    const std::vector<int64_t>* counts[kIvfPasses] = {&ix->coarse_count, &ix->sample_count, &ix->cell_count};
    for (int c = 0; c < nl; c++) {
        for (int p = 0; p < kIvfPasses; p++) {
            const int64_t s0 = (*starts[p])[(size_t)c], cn = (*counts[p])[(size_t)c];
            int32_t* f = info.data() + 9 * (size_t)c + 3 * p;
            f[0] = (int32_t)(s0 / kIvfTileRows);
            f[1] = (int32_t)((cn + kIvfTileRows - 1) / kIvfTileRows);
            f[2] = (int32_t)(s0 + cn);
            const int64_t runs = (f[1] + kIvfMaxTilesPerUnit - 1) / kIvfMaxTilesPerUnit;
            ix->unit_max_runs[p] = std::max(ix->unit_max_runs[p], runs);
            ix->unit_sum_runs[p] += runs;
        }
        order[(size_t)c] = c;
    }
    // Most tiles first, so the persistent grid's tail is short.
    std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
        return info[9 * (size_t)a + 3 * (kIvfPasses - 1) + 1] > info[9 * (size_t)b + 3 * (kIvfPasses - 1) + 1];
    });
    ix->plan_info = dalloc<int32_t>(info.size());
    ix->plan_order = dalloc<int32_t>(order.size());
    ix->plan_scratch = dalloc<int32_t>((size_t)6 * nl + kIvfPasses + 1);  // + the scans' unit counter
    ix->plan_pairs = dalloc<unsigned long long>(kIvfPasses);
    MDH_CUDA(cudaMemcpyAsync(ix->plan_info, info.data(), info.size() * 4, cudaMemcpyHostToDevice, st));
    MDH_CUDA(cudaMemcpyAsync(ix->plan_order, order.data(), order.size() * 4, cudaMemcpyHostToDevice, st));
    MDH_CUDA(cudaStreamSynchronize(st));
}

// Plans every pass for `total` = m * nprobe probes in ws.flags: the grouped
// query matrix in pass[kIvfPasses - 1] (g, gqn, gmap) and the unit tables,
// whose lengths land in nunits[pass] on the device.  Returns per-pass upper
// bounds of the table lengths (they size the buffers and the grids).
void plan_passes(mdh_ivf* ix, int m, int nprobe, cudaStream_t st, int64_t bound[kIvfPasses], int32_t** nunits) {
    const int nl = ix->nlist;
    const int total = m * nprobe;
    Workspace& w = ix->ws;
    int32_t* cnt = ix->plan_scratch;
    int32_t* fill = cnt + nl;
    int32_t* qstart = fill + nl;
    int32_t* ustart = qstart + nl;  // [kIvfPasses][nlist]
    *nunits = ustart + kIvfPasses * nl;
    MDH_CUDA(cudaMemsetAsync(cnt, 0, (size_t)2 * nl * 4, st));
    MDH_CUDA(cudaMemsetAsync(ix->plan_pairs, 0, kIvfPasses * sizeof(unsigned long long), st));
    k_plan_count<<<(total + 255) / 256, 256, 0, st>>>(w.flags, total, cnt);
    k_plan_scan<<<1, kPlanThreads, 0, st>>>(cnt, ix->plan_order, ix->plan_info, nl, qstart, ustart, *nunits,
                                            ix->plan_pairs);
    IvfPassBufs& g = ix->pass[kIvfPasses - 1];
    grow_dev(&g.g, &g.g_bytes, (size_t)total * ix->dpad);
    grow_dev(&g.gqn, &g.gqn_bytes, (size_t)total * 4);
    grow_dev(&g.gmap, &g.gmap_bytes, (size_t)total * 4);
    k_plan_fill<<<(total + 255) / 256, 256, 0, st>>>(w.flags, total, nprobe, qstart, fill, g.gmap);
    launch_gather_queries_u8(w.q_u8, w.qn, g.gmap, total, ix->dpad, g.g, g.gqn, st);
    // sum_c ceil(q_c / 128) * runs_c <= sum_c (q_c / 128 + 1) * runs_c <= total * max_runs / 128 + sum_runs.
    PassUnits tables;
    for (int p = 0; p < kIvfPasses; p++) {
        bound[p] = std::max<int64_t>(1, ((int64_t)total * ix->unit_max_runs[p] + 127) / 128 + ix->unit_sum_runs[p]);
        MDH_REQUIRE(bound[p] < (int64_t(1) << 31), MDH_ERR_UNSUPPORTED, "IVF unit table too large");
        grow_dev(&ix->pass[p].units, &ix->pass[p].units_bytes, (size_t)bound[p] * sizeof(ScanUnit));
        tables.u[p] = ix->pass[p].units;
    }
    k_plan_units<<<dim3((unsigned)((nl + 255) / 256), kIvfPasses), 256, 0, st>>>(cnt, ix->plan_info, qstart, ustart,
                                                                                 nl, tables);
    MDH_CUDA(cudaGetLastError());
}

void check_ivf_device(int dev) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        throw Error(MDH_ERR_CUDA, "no CUDA device is available (this library has no CPU fallback)");
    }
    MDH_REQUIRE(dev >= 0 && dev < count, MDH_ERR_INVALID_ARG, "device ordinal out of range");
    cudaDeviceProp p;
    MDH_CUDA(cudaGetDeviceProperties(&p, dev));
    MDH_REQUIRE(p.major == 10 && p.minor == 0, MDH_ERR_CUDA, "this library is built for sm_100a (B200)");
}

// Per-cell samples in the main layout: rows whose id hashes below `thresh`
// plus the first `head` rows of each cell, in the cell's norm order, each
// cell padded to whole tiles.
void build_ivf_sample(mdh_ivf* ix, const std::vector<int32_t>& ids, uint32_t thresh, int head, Level& sv,
                      std::vector<int64_t>& start, std::vector<int64_t>& count, cudaStream_t st) {
    const Level& lv = ix->rows;
    const int nl = ix->nlist;
    start.assign((size_t)nl, 0);
    count.assign((size_t)nl, 0);
    std::vector<int32_t> pos;
    for (int c = 0; c < nl; c++) {
        start[(size_t)c] = (int64_t)pos.size();
        const int64_t s0 = ix->cell_start[(size_t)c], cnt = ix->cell_count[(size_t)c];
        for (int64_t r = s0; r < s0 + cnt; r++)
            if (r - s0 < head || sample_hash_host(ids[(size_t)r]) < thresh) pos.push_back((int32_t)r);
        count[(size_t)c] = (int64_t)pos.size() - start[(size_t)c];
        while (pos.size() % kIvfTileRows) pos.push_back(-1);
    }
    if (pos.empty())
        for (int i = 0; i < kIvfTileRows; i++) pos.push_back(-1);
    const int64_t m = (int64_t)pos.size();
    sv.n = m;
    sv.n_pad = m;
    sv.rows = dalloc<uint8_t>((size_t)m * ix->dpad);
    sv.norms = dalloc<int32_t>(m);
    sv.ids = dalloc<int32_t>(m);
    int32_t* dpos = dalloc<int32_t>(m);
    MDH_CUDA(cudaMemcpyAsync(dpos, pos.data(), (size_t)m * 4, cudaMemcpyHostToDevice, st));
    k_ivf_gather_rows<<<(unsigned)((m * 8 + 255) / 256), 256, 0, st>>>(dpos, m, ix->dpad, lv.rows, lv.norms, lv.ids,
                                                                        sv.rows, sv.norms, sv.ids);
    cudaError_t e = cudaGetLastError();
    cudaError_t e2 = cudaStreamSynchronize(st);
    cudaFree(dpos);
    MDH_CUDA(e);
    MDH_CUDA(e2);
    make_tmap_rows(sv, ix->dpad);
}

void build_ivf_samples(mdh_ivf* ix, cudaStream_t st) {
    const Level& lv = ix->rows;
    std::vector<int32_t> ids((size_t)lv.n_pad);
    MDH_CUDA(cudaMemcpyAsync(ids.data(), lv.ids, ids.size() * 4, cudaMemcpyDeviceToHost, st));
    MDH_CUDA(cudaStreamSynchronize(st));
    build_ivf_sample(ix, ids, kIvfSampleThresh, kIvfSampleHead, ix->sample, ix->sample_start, ix->sample_count, st);
    build_ivf_sample(ix, ids, kIvfCoarseThresh, kIvfCoarseHead, ix->coarse, ix->coarse_start, ix->coarse_count, st);
}

void ivf_create(const uint8_t* host, int64_t n, int32_t dim, const float* centroids, int32_t nlist,
                const int32_t* labels, int32_t metric, int32_t device, mdh_ivf** out) {
    MDH_REQUIRE(out, MDH_ERR_INVALID_ARG, "null output pointer");
    *out = nullptr;
    MDH_REQUIRE(n >= 1 && host && labels && centroids, MDH_ERR_INVALID_ARG, "null or empty corpus");
    MDH_REQUIRE(n <= 0x7FFFFFFF - 256 * (int64_t)kIvfMaxNlist, MDH_ERR_INVALID_ARG, "too many rows");
    MDH_REQUIRE(dim >= 1 && dim <= 128, MDH_ERR_UNSUPPORTED, "the IVF scan supports dim <= 128");
    MDH_REQUIRE(nlist >= 1 && nlist <= kIvfMaxNlist, MDH_ERR_UNSUPPORTED, "nlist must be in [1, 8192]");
    MDH_REQUIRE(metric == MDH_METRIC_L2 || metric == MDH_METRIC_COSINE, MDH_ERR_INVALID_ARG, "metric must be 0 or 1");
    int dev = device;
    if (dev < 0) {
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            throw Error(MDH_ERR_CUDA, "no CUDA device is available (this library has no CPU fallback)");
        }
    }
    check_ivf_device(dev);
    for (int64_t i = 0; i < (int64_t)nlist * dim; i++)
        MDH_REQUIRE(std::isfinite(centroids[i]), MDH_ERR_INVALID_ARG, "centroids must be finite");
    std::vector<int64_t> count((size_t)nlist, 0);
    for (int64_t i = 0; i < n; i++) {
        const int32_t l = labels[i];
        MDH_REQUIRE(l >= 0 && l < nlist, MDH_ERR_INVALID_ARG, "label out of range [0, nlist)");
        count[(size_t)l]++;
    }
    std::unique_ptr<mdh_ivf> ix(new mdh_ivf());
    ix->device = dev;
    ix->n = n;
    ix->dim = dim;
    ix->dpad = 128;
    ix->metric = metric;
    ix->nlist = nlist;
    ix->cell_count = count;
    ix->cell_start.resize((size_t)nlist);
    std::vector<int64_t> first((size_t)nlist);
    int64_t off = 0, pos = 0;
    for (int c = 0; c < nlist; c++) {
        ix->cell_start[(size_t)c] = off;
        first[(size_t)c] = pos;
        off += (count[(size_t)c] + kIvfTileRows - 1) / kIvfTileRows * kIvfTileRows;
        pos += count[(size_t)c];
    }
    const int64_t total = std::max<int64_t>(off, kIvfTileRows);
    MDH_CUDA(cudaSetDevice(dev));
    MDH_CUDA(cudaStreamCreateWithFlags(&ix->stream, cudaStreamNonBlocking));
    cudaStream_t st = ix->stream;
    const int dpad = ix->dpad;
    uint8_t* stage = nullptr;
    int32_t* dlabels = nullptr;
    unsigned long long *keys = nullptr, *keys2 = nullptr;
    int32_t *vals = nullptr, *vals2 = nullptr;
    int64_t *dstart = nullptr, *dfirst = nullptr;
    void* tmp = nullptr;
    auto release_tmp = [&]() {
        for (void* p : {(void*)stage, (void*)dlabels, (void*)keys, (void*)keys2, (void*)vals, (void*)vals2,
                        (void*)dstart, (void*)dfirst, tmp})
            if (p) cudaFree(p);
    };
    try {
        stage = dalloc<uint8_t>((size_t)n * dpad);
        MDH_CUDA(cudaMemsetAsync(stage, 0, (size_t)n * dpad, st));
        MDH_CUDA(cudaMemcpy2DAsync(stage, dpad, host, dim, dim, n, cudaMemcpyHostToDevice, st));
        dlabels = dalloc<int32_t>(n);
        MDH_CUDA(cudaMemcpyAsync(dlabels, labels, (size_t)n * 4, cudaMemcpyHostToDevice, st));
        keys = dalloc<unsigned long long>(n);
        keys2 = dalloc<unsigned long long>(n);
        vals = dalloc<int32_t>(n);
        vals2 = dalloc<int32_t>(n);
        k_ivf_keys<<<(unsigned)((n * 8 + 255) / 256), 256, 0, st>>>(stage, dlabels, n, dpad, keys, vals);
        MDH_CUDA(cudaGetLastError());
        size_t tmp_bytes = 0;
        MDH_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, keys, keys2, vals, vals2, (int)n, 0, 64, st));
        tmp = dalloc<uint8_t>(tmp_bytes);
        MDH_CUDA(cub::DeviceRadixSort::SortPairs(tmp, tmp_bytes, keys, keys2, vals, vals2, (int)n, 0, 64, st));
        Level& lv = ix->rows;
        lv.n = total;
        lv.n_pad = total;
        lv.rows = dalloc<uint8_t>((size_t)total * dpad);
        lv.norms = dalloc<int32_t>(total);
        lv.ids = dalloc<int32_t>(total);
        MDH_CUDA(cudaMemsetAsync(lv.rows, 0, (size_t)total * dpad, st));
        k_ivf_fill<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(lv.norms, total, kNormPad);
        k_ivf_fill<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(lv.ids, total, -1);
        dstart = dalloc<int64_t>(nlist);
        dfirst = dalloc<int64_t>(nlist);
        MDH_CUDA(cudaMemcpyAsync(dstart, ix->cell_start.data(), (size_t)nlist * 8, cudaMemcpyHostToDevice, st));
        MDH_CUDA(cudaMemcpyAsync(dfirst, first.data(), (size_t)nlist * 8, cudaMemcpyHostToDevice, st));
        k_ivf_gather<<<(unsigned)((n * 8 + 255) / 256), 256, 0, st>>>(stage, keys2, vals2, n, dpad, dstart, dfirst,
                                                                       lv.rows, lv.norms, lv.ids,
                                                                       metric == MDH_METRIC_COSINE ? 1 : 0);
        MDH_CUDA(cudaGetLastError());
        ix->centroids = dalloc<float>((size_t)nlist * dim);
        MDH_CUDA(cudaMemcpyAsync(ix->centroids, centroids, (size_t)nlist * dim * 4, cudaMemcpyHostToDevice, st));
        MDH_CUDA(cudaStreamSynchronize(st));
        make_tmap_rows(lv, dpad);
        build_ivf_samples(ix.get(), st);
        build_ivf_plan_info(ix.get(), st);
    } catch (...) {
        cudaStreamSynchronize(st);
        release_tmp();
        free_level_buffers(ix->rows);
        free_level_buffers(ix->sample);
        free_level_buffers(ix->coarse);
        if (ix->centroids) cudaFree(ix->centroids);
        for (void* p : {(void*)ix->plan_info, (void*)ix->plan_order, (void*)ix->plan_scratch, (void*)ix->plan_pairs,
                        (void*)ix->chunk_x, (void*)ix->chunk_hdr})
            if (p) cudaFree(p);
        cudaStreamDestroy(ix->stream);
        throw;
    }
    release_tmp();
    *out = ix.release();
}

// Routes nq host queries: staged u8 queries in ws.q_u8, norms in ws.qn, the
// probe matrix [nq][nprobe] in ws.flags; copied to `probe` when it is given.
void ivf_route_impl(mdh_ivf* ix, const uint8_t* host_q, int nq, int nprobe, std::vector<int32_t>* probe) {
    Workspace& w = ix->ws;
    cudaStream_t st = ix->stream;
    grow_dev(&w.q_u8, &w.q_u8_bytes, (size_t)nq * ix->dpad);
    grow_dev(&w.qn, &w.qn_bytes, (size_t)nq * 4);
    grow_dev(&w.flags, &w.flags_bytes, (size_t)nq * nprobe * 4);  // probe matrix
    MDH_CUDA(cudaMemsetAsync(w.q_u8, 0, (size_t)nq * ix->dpad, st));
    MDH_CUDA(cudaMemcpy2DAsync(w.q_u8, ix->dpad, host_q, ix->dim, ix->dim, nq, cudaMemcpyHostToDevice, st));
    if (ix->metric == MDH_METRIC_COSINE)
        launch_fill_u32(reinterpret_cast<uint32_t*>(w.qn), nq, (uint32_t)kIvfIpOffset, st);
    else
        launch_query_norms_u8(w.q_u8, nq, ix->dpad, w.qn, st);
    grow_dev(&w.tmp, &w.tmp_bytes, (size_t)nq * ix->nlist * sizeof(double));  // similarities
    launch_route(w.q_u8, nq, ix->dpad, ix->dim, ix->centroids, ix->nlist, nprobe, static_cast<double*>(w.tmp), w.flags,
                 st);
    if (probe) {
        probe->resize((size_t)nq * nprobe);
        MDH_CUDA(cudaMemcpyAsync(probe->data(), w.flags, probe->size() * 4, cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaStreamSynchronize(st));
    }
}

void ivf_search_impl(mdh_ivf* ix, const uint8_t* host_q, int nq, int k, int nprobe, int32_t* out_ids,
                     int32_t* out_dist, mdh_stats* stats) {
    auto t_start = std::chrono::high_resolution_clock::now();
    MDH_REQUIRE(ix, MDH_ERR_INVALID_ARG, "null index");
    MDH_REQUIRE(nq >= 0 && k >= 0, MDH_ERR_INVALID_ARG, "nq and k must be >= 0");
    MDH_REQUIRE(nq == 0 || k == 0 || (host_q && out_ids), MDH_ERR_INVALID_ARG, "null buffer");
    MDH_REQUIRE(nprobe >= 1, MDH_ERR_INVALID_ARG, "nprobe must be >= 1");
    MDH_REQUIRE(k <= 4096, MDH_ERR_UNSUPPORTED, "the IVF search supports k <= 4096");
    nprobe = std::min(nprobe, ix->nlist);
    MDH_REQUIRE(nprobe <= kIvfMaxProbe, MDH_ERR_UNSUPPORTED, "nprobe must be <= 1024");
    std::lock_guard<std::mutex> lock(ix->mu);
    MDH_CUDA(cudaSetDevice(ix->device));
    mdh_stats s{};
    for (size_t i = 0; i < (size_t)nq * k; i++) out_ids[i] = -1;
    if (out_dist)
        for (size_t i = 0; i < (size_t)nq * k; i++) out_dist[i] = -1;
    if (nq == 0 || k == 0) {
        if (stats) *stats = s;
        return;
    }
    cudaStream_t st = ix->stream;
    Workspace& w = ix->ws;
    const Level& lv = ix->rows;
    const int chunk = (int)std::max<int64_t>(1, std::min<int64_t>(nq, (int64_t(2) << 30) / ((int64_t)kIvfCap2 * 8)));
    std::vector<uint32_t> hkey;
    std::vector<int32_t> hid;
    if (!w.ev_prep)
        for (cudaEvent_t* e : {&w.ev0, &w.ev1, &w.ev_start, &w.ev_sel, &w.ev_prep})
            if (!*e) MDH_CUDA(cudaEventCreate(e));
    for (int c0 = 0; c0 < nq; c0 += chunk) {
        const int m = std::min(chunk, nq - c0);
        MDH_CUDA(cudaEventRecord(w.ev_prep, st));
        ivf_route_impl(ix, host_q + (size_t)c0 * ix->dim, m, nprobe, nullptr);
        s.kernel_launches += 3;
        int64_t bound[kIvfPasses];
        int32_t* nunits = nullptr;
        plan_passes(ix, m, nprobe, st, bound, &nunits);
        int32_t* ucounter = nunits + kIvfPasses;  // the scans hand out units at run time, longest cells first
        const int total = m * nprobe;
        s.kernel_launches += 5;
        const IvfPassBufs& qm = ix->pass[kIvfPasses - 1];  // the grouped query matrix
        grow_dev(&w.thr_key, &w.thr_key_bytes, (size_t)m * 4);
        grow_dev(&w.thr_id, &w.thr_id_bytes, (size_t)m * 4);
        grow_dev(&w.counts, &w.counts_bytes, (size_t)m * 4);
        grow_dev(&w.cand, &w.cand_bytes, (size_t)m * std::max(kIvfCap1, kIvfCap2) * sizeof(uint2));
        grow_dev(&w.out_key, &w.out_key_bytes, (size_t)m * k * 4);
        grow_dev(&w.out_id, &w.out_id_bytes, (size_t)m * k * 4);
        grow_dev(&w.qlist, &w.qlist_bytes, (size_t)m * 4);  // overflow flags
        ChunkOut defer;
        {
            int sms = 0;
            MDH_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ix->device));
            const uint64_t cap = (uint64_t)m * kIvfChunksPerQuery + (uint64_t)sms * 16 * 2 * kChunkBlock;
            uint64_t cap64 = std::min<uint64_t>((cap + kChunkBlock - 1) / kChunkBlock * kChunkBlock,
                                                (uint64_t)1 << 30);
            if (take_fault(kFaultIvfChunks)) cap64 = kChunkBlock;
            grow_dev(&ix->chunk_x, &ix->chunk_x_bytes, (size_t)cap64 * 128);
            grow_dev(&ix->chunk_hdr, &ix->chunk_hdr_bytes, (size_t)cap64 * 16);
            defer.x = ix->chunk_x;
            defer.hdr = ix->chunk_hdr;
            defer.capacity = (uint32_t)cap64;
            defer.nq = m;
        }
        if (!w.status) {
            MDH_CUDA(cudaMalloc(&w.status, kStatusWords * sizeof(int32_t)));
            MDH_CUDA(cudaHostAlloc(&w.h_status, kStatusWords * sizeof(int32_t), cudaHostAllocDefault));
        }
        MDH_CUDA(cudaMemsetAsync(w.status, 0, (kStatusChunkOverflow + 1) * sizeof(int32_t), st));
        defer.counter = reinterpret_cast<uint32_t*>(w.status + kStatusChunkCounter);
        unsigned long long* n_cand = reinterpret_cast<unsigned long long*>(w.status + 2);
        unsigned long long* bstats = reinterpret_cast<unsigned long long*>(w.status + kStatusBlockStats);
        // Pass 0: coarse samples of the probed cells, infinite thresholds; the
        // k-th (key, id) is a threshold for the union (the sample is part of it).
        MDH_CUDA(cudaEventRecord(w.ev_start, st));
        launch_fill_threshold(w.thr_key, w.thr_id, m, kKeyInf, kIdInf, st);
        MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)m * 4, st));
        launch_filter_tc_u8_l2_units(ix->coarse, ix->dpad, qm.g, total, qm.gmap, w.qn, ix->pass[0].units,
                                     (int)bound[0], nunits, ucounter, w.thr_key, w.thr_id, w.counts, w.cand, kIvfCap0,
                                     w.status, bstats, &defer, st);
        launch_select(w.counts, w.cand, kIvfCap0, ix->coarse.ids, m, k, 0, w.thr_key, w.thr_id, w.out_key, w.out_id,
                      w.qlist, w.status + 1, nullptr, nullptr, st);
        // Pass 1: the samples with that threshold tighten it (a list that
        // overflows keeps the k-th of what it stored: still a valid bound).
        MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)m * 4, st));
        launch_filter_tc_u8_l2_units(ix->sample, ix->dpad, qm.g, total, qm.gmap, w.qn, ix->pass[1].units,
                                     (int)bound[1], nunits + 1, ucounter, w.thr_key, w.thr_id, w.counts, w.cand, kIvfCap1,
                                     w.status, bstats, &defer, st);
        launch_select(w.counts, w.cand, kIvfCap1, ix->sample.ids, m, k, 0, w.thr_key, w.thr_id, w.out_key, w.out_id,
                      w.qlist, w.status + 1, nullptr, nullptr, st);
        s.kernel_launches += 6;
        // Pass 2: every probed cell with that threshold.  A chunk buffer that
        // overflowed in passes 0 and 1 only left their thresholds looser (a
        // k-th over part of a sample still bounds the union); in pass 2 it
        // means a rerun, so its flag starts clear.
        MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)m * 4, st));
        MDH_CUDA(cudaMemsetAsync(w.status + kStatusChunkOverflow, 0, sizeof(int32_t), st));
        MDH_CUDA(cudaEventRecord(w.ev0, st));
        launch_filter_tc_u8_l2_units(lv, ix->dpad, qm.g, total, qm.gmap, w.qn, ix->pass[2].units, (int)bound[2],
                                     nunits + 2, ucounter, w.thr_key, w.thr_id, w.counts, w.cand, kIvfCap2,
                                     w.status, bstats, &defer, st);
        MDH_CUDA(cudaEventRecord(w.ev1, st));
        launch_select(w.counts, w.cand, kIvfCap2, lv.ids, m, k, 1, w.thr_key, w.thr_id, w.out_key, w.out_id, w.qlist,
                      w.status + 1, nullptr, n_cand, st);
        MDH_CUDA(cudaEventRecord(w.ev_sel, st));
        s.kernel_launches += 5;  // three re-key passes, the selection and the pass-2 scan
        // Status, pair counts and the results come back with one synchronization
        // (the results are copied again after an overflow round).
        hkey.resize((size_t)m * k);
        hid.resize((size_t)m * k);
        unsigned long long pairs[kIvfPasses] = {};
        MDH_CUDA(cudaMemcpyAsync(w.h_status, w.status, kStatusWords * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaMemcpyAsync(pairs, ix->plan_pairs, sizeof(pairs), cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaMemcpyAsync(hkey.data(), w.out_key, (size_t)m * k * 4, cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaMemcpyAsync(hid.data(), w.out_id, (size_t)m * k * 4, cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaStreamSynchronize(st));
        int64_t chunk_pairs = (int64_t)(pairs[0] + pairs[1] + pairs[2]);
        s.pairs_scored += chunk_pairs;
        s.full_scan_pairs += (int64_t)pairs[2];
        if (w.h_status[0] != kDevOk)
            throw Error(MDH_ERR_TIMEOUT, "IVF scan reported device status " + std::to_string(w.h_status[0]));
        {
            // Stages of this chunk: routing and planning (with the query
            // upload), passes 0 and 1 with their re-key passes and
            // selections, pass 2 with its re-key pass, the final selection.
            auto ms = [](cudaEvent_t a, cudaEvent_t b) {
                float v = 0.0f;
                MDH_CUDA(cudaEventElapsedTime(&v, a, b));
                return (double)v;
            };
            s.prep_ms += ms(w.ev_prep, w.ev_start);
            s.sample_ms += ms(w.ev_start, w.ev0);
            s.full_scan_ms += ms(w.ev0, w.ev1);
            s.select_ms += ms(w.ev1, w.ev_sel);
        }
        int rounds = 0;
        while (w.h_status[1] > 0 || w.h_status[kStatusChunkOverflow] != 0) {
            // Overflowed lists got a strictly tighter threshold; the others keep
            // theirs and reproduce their result.  After a chunk-buffer overflow
            // every list reruns: its threshold is still a valid bound.  Reruns
            // form keys in the scan (no chunk buffer).
            MDH_REQUIRE(++rounds < 64, MDH_ERR_INTERNAL, "candidate overflow did not converge");
            w.h_status[kStatusChunkOverflow] = 0;
            MDH_CUDA(cudaMemsetAsync(w.counts, 0, (size_t)m * 4, st));
            MDH_CUDA(cudaMemsetAsync(w.status + 1, 0, sizeof(int32_t), st));
            launch_filter_tc_u8_l2_units(lv, ix->dpad, qm.g, total, qm.gmap, w.qn, ix->pass[2].units,
                                         (int)bound[2], nunits + 2, ucounter, w.thr_key, w.thr_id, w.counts, w.cand, kIvfCap2,
                                         w.status, bstats, nullptr, st);
            launch_select(w.counts, w.cand, kIvfCap2, lv.ids, m, k, 1, w.thr_key, w.thr_id, w.out_key, w.out_id,
                          w.qlist, w.status + 1, nullptr, n_cand, st);
            s.kernel_launches += 2;
            s.pairs_scored += (int64_t)pairs[2];
            chunk_pairs += (int64_t)pairs[2];
            MDH_CUDA(cudaMemcpyAsync(w.h_status, w.status, kStatusChunkOverflow * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
            MDH_CUDA(cudaMemcpyAsync(hkey.data(), w.out_key, (size_t)m * k * 4, cudaMemcpyDeviceToHost, st));
            MDH_CUDA(cudaMemcpyAsync(hid.data(), w.out_id, (size_t)m * k * 4, cudaMemcpyDeviceToHost, st));
            MDH_CUDA(cudaStreamSynchronize(st));
            if (w.h_status[0] != kDevOk)
                throw Error(MDH_ERR_TIMEOUT, "IVF scan reported device status " + std::to_string(w.h_status[0]));
        }
        {
            unsigned long long cand_n = 0, bs[3] = {};
            std::memcpy(&cand_n, w.h_status + 2, 8);
            std::memcpy(bs, w.h_status + kStatusBlockStats, sizeof(bs));
            s.candidates += (int64_t)cand_n;
            // Every pass and rerun ran the unit-table scan: each pair of a
            // probed cell was either settled by its chunk's bound or formed.
            s.blocks_tested += (int64_t)bs[0];
            s.blocks_passed += (int64_t)bs[1];
            s.pairs_pruned_by_bound += chunk_pairs - (int64_t)bs[2];
        }
        for (size_t i = 0; i < (size_t)m * k; i++) {
            out_ids[(size_t)c0 * k + i] = hid[i];
            if (out_dist)
                out_dist[(size_t)c0 * k + i] = hid[i] < 0                        ? -1
                                               : ix->metric == MDH_METRIC_COSINE ? (kIvfIpOffset - (int32_t)hkey[i]) / 2
                                                                                 : (int32_t)hkey[i];
        }
    }
    s.levels = kIvfPasses;
    s.tensor_core_path = 1;
    s.latency_ms = std::chrono::duration<double, std::milli>(std::chrono::high_resolution_clock::now() - t_start).count();
    if (stats) *stats = s;
}

}  // namespace

}  // namespace mdh

using namespace mdh;

extern "C" {

mdh_status mdh_ivf_create_u8_metric(const uint8_t* host_corpus, int64_t n, int32_t dim, const float* centroids,
                                    int32_t nlist, const int32_t* labels, int32_t metric, int32_t device,
                                    mdh_ivf** out) {
    struct A {
        const uint8_t* c; int64_t n; int32_t dim; const float* cen; int32_t nl; const int32_t* lab; int32_t metric;
        int32_t dev; mdh_ivf** out;
    } a{host_corpus, n, dim, centroids, nlist, labels, metric, device, out};
    return run_guarded([](void* p) {
        A& x = *static_cast<A*>(p);
        ivf_create(x.c, x.n, x.dim, x.cen, x.nl, x.lab, x.metric, x.dev, x.out);
    }, &a);
}

mdh_status mdh_ivf_create_u8(const uint8_t* host_corpus, int64_t n, int32_t dim, const float* centroids,
                             int32_t nlist, const int32_t* labels, int32_t device, mdh_ivf** out) {
    return mdh_ivf_create_u8_metric(host_corpus, n, dim, centroids, nlist, labels, MDH_METRIC_L2, device, out);
}

mdh_status mdh_ivf_route_u8(mdh_ivf* index, const uint8_t* host_queries, int32_t nq, int32_t nprobe,
                            int32_t* out_cells) {
    struct A {
        mdh_ivf* ix; const uint8_t* q; int32_t nq, np; int32_t* out;
    } a{index, host_queries, nq, nprobe, out_cells};
    return run_guarded([](void* p) {
        A& x = *static_cast<A*>(p);
        MDH_REQUIRE(x.ix, MDH_ERR_INVALID_ARG, "null index");
        MDH_REQUIRE(x.nq >= 0 && (x.nq == 0 || (x.q && x.out)), MDH_ERR_INVALID_ARG, "null buffer");
        MDH_REQUIRE(x.np >= 1 && x.np <= x.ix->nlist && x.np <= kIvfMaxProbe, MDH_ERR_INVALID_ARG,
                    "nprobe must be in [1, min(nlist, 1024)]");
        if (x.nq == 0) return;
        std::lock_guard<std::mutex> lock(x.ix->mu);
        MDH_CUDA(cudaSetDevice(x.ix->device));
        std::vector<int32_t> probe;
        ivf_route_impl(x.ix, x.q, x.nq, x.np, &probe);
        std::memcpy(x.out, probe.data(), probe.size() * 4);
    }, &a);
}

mdh_status mdh_ivf_search_u8(mdh_ivf* index, const uint8_t* host_queries, int32_t nq, int32_t k, int32_t nprobe,
                             int32_t* out_ids, int32_t* out_dist, mdh_stats* stats) {
    struct A {
        mdh_ivf* ix; const uint8_t* q; int32_t nq, k, np; int32_t *ids, *dist; mdh_stats* st;
    } a{index, host_queries, nq, k, nprobe, out_ids, out_dist, stats};
    return run_guarded([](void* p) {
        A& x = *static_cast<A*>(p);
        ivf_search_impl(x.ix, x.q, x.nq, x.k, x.np, x.ids, x.dist, x.st);
    }, &a);
}

mdh_status mdh_ivf_info(const mdh_ivf* index, int64_t* n, int32_t* dim, int32_t* nlist, int64_t* cell_rows) {
    struct A {
        const mdh_ivf* ix; int64_t* n; int32_t *dim, *nlist; int64_t* cells;
    } a{index, n, dim, nlist, cell_rows};
    return run_guarded([](void* p) {
        A& x = *static_cast<A*>(p);
        MDH_REQUIRE(x.ix, MDH_ERR_INVALID_ARG, "null index");
        if (x.n) *x.n = x.ix->n;
        if (x.dim) *x.dim = x.ix->dim;
        if (x.nlist) *x.nlist = x.ix->nlist;
        if (x.cells) std::memcpy(x.cells, x.ix->cell_count.data(), x.ix->cell_count.size() * 8);
    }, &a);
}

mdh_status mdh_ivf_destroy(mdh_ivf* index) {
    return run_guarded([](void* p) {
        mdh_ivf* ix = static_cast<mdh_ivf*>(p);
        if (!ix) return;
        cudaSetDevice(ix->device);
        if (ix->stream) cudaStreamSynchronize(ix->stream);
        ix->pass[0].free_all();
        ix->pass[1].free_all();
        ix->pass[2].free_all();
        free_level_buffers(ix->rows);
        free_level_buffers(ix->sample);
        free_level_buffers(ix->coarse);
        if (ix->centroids) cudaFree(ix->centroids);
        for (void* p : {(void*)ix->plan_info, (void*)ix->plan_order, (void*)ix->plan_scratch, (void*)ix->plan_pairs,
                        (void*)ix->chunk_x, (void*)ix->chunk_hdr})
            if (p) cudaFree(p);
        free_workspace(ix->ws);
        if (ix->stream) cudaStreamDestroy(ix->stream);
        delete ix;
    }, index);
}

}  // extern "C"
