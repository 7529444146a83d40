// Index build: one device shard of the corpus.
//
// Replaces the reference's construction step (SpeedEngine::SpeedEngine,
// src/speed_cpu.cpp:81-144, and the norm part of MadhavaL2::build,
// src/winnex_madhava.cpp:150-179).  Instead of a float copy (4x memory) the
// shard keeps:
//   * u8 rows sorted ascending by (|v|^2, row id), row stride dpad bytes
//     (dpad = dim rounded up to 128, zero padded), rows padded to 256;
//   * int32 |v|^2 per row (exact: dim * 255^2 < 2^31);
//   * int32 global row id per sorted position;
//   * nested random samples of the rows (same layout) used to find each
//     query's distance threshold before the full scan.
// Sorting by norm makes every 32-row chunk's minimum norm its first entry,
// which the tensor-core scan uses for its Cauchy-Schwarz chunk filter.
#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_select.cuh>
#include <thrust/iterator/counting_iterator.h>

#include <algorithm>

#include "internal.h"

namespace mdh {

namespace {

// 8 lanes per row, 16 bytes per lane per step.
__global__ void k_row_norms_u8(const uint8_t* __restrict__ rows, int64_t n, int dpad,
                               unsigned long long* __restrict__ keys) {
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
    if (r < n && l8 == 0) keys[r] = ((unsigned long long)s << 32) | (unsigned long long)(uint32_t)r;
}

// Sorted position p takes source row (key & 0xffffffff).
__global__ void k_gather_sorted(const uint8_t* __restrict__ src, const unsigned long long* __restrict__ keys,
                                int64_t n, int dpad, int64_t id_base, uint8_t* __restrict__ rows,
                                int32_t* __restrict__ norms, int32_t* __restrict__ ids) {
    const int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l8 = threadIdx.x & 7;
    if (p >= n) return;
    const unsigned long long key = keys[p];
    const int64_t s = (int64_t)(key & 0xffffffffull);
    for (int off = l8 * 16; off < dpad; off += 128)
        *reinterpret_cast<uint4*>(rows + (size_t)p * dpad + off) =
            *reinterpret_cast<const uint4*>(src + (size_t)s * dpad + off);
    if (l8 == 0) {
        norms[p] = (int32_t)(key >> 32);
        ids[p] = (int32_t)(id_base + s);
    }
}

// Gather a subset (positions list) of an existing level.
__global__ void k_gather_subset(const uint8_t* __restrict__ src_rows, const int32_t* __restrict__ src_norms,
                                const int32_t* __restrict__ src_ids, const float* __restrict__ src_f32,
                                const float* __restrict__ src_nf, const int32_t* __restrict__ pos, int64_t m,
                                int dpad, int dim, uint8_t* __restrict__ rows, int32_t* __restrict__ norms,
                                int32_t* __restrict__ ids, float* __restrict__ rows_f32, float* __restrict__ nf) {
    const int64_t p = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l8 = threadIdx.x & 7;
    if (p >= m) return;
    const int64_t s = pos[p];
    if (src_rows)
        for (int off = l8 * 16; off < dpad; off += 128)
            *reinterpret_cast<uint4*>(rows + (size_t)p * dpad + off) =
                *reinterpret_cast<const uint4*>(src_rows + (size_t)s * dpad + off);
    if (src_f32)
        for (int j = l8; j < dim; j += 8) rows_f32[(size_t)p * dim + j] = src_f32[(size_t)s * dim + j];
    if (l8 == 0) {
        if (src_norms) norms[p] = src_norms[s];
        ids[p] = src_ids[s];
        if (src_nf) nf[p] = src_nf[s];
    }
}

__global__ void k_fill_i32(int32_t* p, int64_t n, int32_t v) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

__device__ __forceinline__ uint32_t sample_hash(int32_t id) {
    // splitmix64 finalizer of the global row id; the high half decides
    // membership, so samples are nested by construction.
    unsigned long long z = (unsigned long long)(uint32_t)id + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (uint32_t)(z >> 32);
}

__global__ void k_sample_flags(const int32_t* __restrict__ ids, int64_t n, uint32_t thresh, uint8_t* __restrict__ flags) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) flags[i] = sample_hash(ids[i]) < thresh ? 1 : 0;
}

// SpeedEngine float rows (src/speed_cpu.cpp:81-144): cosine rows are scaled
// by 1/sqrt(sum v^2) (sequential FMA chain), L2 rows keep v and |v|^2.
__global__ void k_prepare_f32(const float* __restrict__ src_f32, const uint8_t* __restrict__ src_u8, int64_t n,
                              int dim, int dpad, int cosine, float* __restrict__ dst, float* __restrict__ nf) {
    int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    float norm = 0.0f;
    float* d = dst + (size_t)r * dim;
    for (int j = 0; j < dim; j++) {
        float v = src_f32 ? src_f32[(size_t)r * dim + j] : (float)src_u8[(size_t)r * dpad + j];
        d[j] = v;
        norm = __fmaf_rn(v, v, norm);
    }
    if (cosine) {
        norm = __fsqrt_rn(norm);
        if (norm > 1e-12f) {
            float inv = __fdiv_rn(1.0f, norm);
            for (int j = 0; j < dim; j++) d[j] = __fmul_rn(d[j], inv);
        }
        nf[r] = 1.0f;
    } else {
        nf[r] = norm;
    }
}

template <class T>
T* dalloc(size_t count) {
    void* p = nullptr;
    if (count == 0) count = 1;
    cudaError_t e = cudaMalloc(&p, count * sizeof(T));
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw Error(MDH_ERR_OOM, std::string("device allocation failed: ") + cudaGetErrorString(e));
    }
    return static_cast<T*>(p);
}

}  // namespace

int g_sample_top_ratio = kSampleTopRatioDefault;

// Nested sample sizes for a shard of n rows: 1024 * 4^j up to n / R
// (R = g_sample_top_ratio, 8 by default).  A search picks its chain of levels
// from this ladder by cost (capi.cu, plan_levels): the best largest sample
// is about sqrt(4,500 k n) rows (scan cost against candidate cost), which the
// ladder brackets within a factor of 2 for every k up to 128 and n above
// ~1M.  The samples hold at most n/6 rows (0.056 n at 100M rows).  Shards
// under 8,192 rows get no sample.
std::vector<int64_t> plan_samples(int64_t n) {
    std::vector<int64_t> s;
    if (n < 8 * 1024) return s;
    const int64_t top = std::max<int64_t>(1024, n / std::max(2, g_sample_top_ratio));
    for (int64_t m = 1024; m <= top; m *= 4) s.push_back(m);
    // A search for k rows starts from a level of at least k rows whose dense
    // list fits the selector (16,384 entries).  Shards above that size whose
    // ladder stops short of it get a 16,384-row level too, so any k up to it
    // has a first level; the planner skips it where it does not pay.
    constexpr int64_t kSelectorRows = 16384;
    if (n > kSelectorRows && s.back() < kSelectorRows) s.push_back(kSelectorRows);
    return s;
}

namespace {

void build_samples(mdh_index* ix, Shard& sh, bool u8, bool f32) {
    cudaStream_t st = sh.stream;
    Level full = sh.levels.back();
    const int64_t n = full.n;
    std::vector<int64_t> sizes = plan_samples(n);
    if (sizes.empty()) return;
    uint8_t* flags = dalloc<uint8_t>(n);
    int32_t* pos = dalloc<int32_t>(n);
    int32_t* nsel = dalloc<int32_t>(1);
    size_t tmp_bytes = 0;
    thrust::counting_iterator<int32_t> it(0);
    cub::DeviceSelect::Flagged(nullptr, tmp_bytes, it, flags, pos, nsel, (int)n, st);
    void* tmp = dalloc<uint8_t>(tmp_bytes);
    std::vector<Level> samples;
    for (int64_t want : sizes) {
        double frac = (double)want / (double)n;
        uint32_t thresh = (uint32_t)std::min(4294967295.0, frac * 4294967296.0);
        k_sample_flags<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(full.ids, n, thresh, flags);
        MDH_CUDA(cudaGetLastError());
        MDH_CUDA(cub::DeviceSelect::Flagged(tmp, tmp_bytes, it, flags, pos, nsel, (int)n, st));
        int32_t m = 0;
        MDH_CUDA(cudaMemcpyAsync(&m, nsel, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        MDH_CUDA(cudaStreamSynchronize(st));
        if (m < 64) continue;
        Level lv;
        alloc_level(lv, m, ix->dpad, ix->dim, u8, f32, st);
        k_gather_subset<<<(unsigned)((m * 8 + 255) / 256), 256, 0, st>>>(
            u8 ? full.rows : nullptr, u8 ? full.norms : nullptr, full.ids, f32 ? full.rows_f32 : nullptr,
            f32 ? full.norms_f32 : nullptr, pos, m, ix->dpad, ix->dim, lv.rows, lv.norms, lv.ids, lv.rows_f32,
            lv.norms_f32);
        MDH_CUDA(cudaGetLastError());
        samples.push_back(lv);
    }
    MDH_CUDA(cudaStreamSynchronize(st));
    cudaFree(tmp);
    cudaFree(flags);
    cudaFree(pos);
    cudaFree(nsel);
    samples.push_back(full);
    sh.levels = samples;
}

}  // namespace

void alloc_level(Level& lv, int64_t n, int dpad, int dim, bool u8, bool f32, cudaStream_t st) {
    lv.n = n;
    lv.n_pad = round_up(n > 0 ? n : 1, kTileRows);
    lv.ids = dalloc<int32_t>(lv.n_pad);
    if (u8) {
        lv.rows = dalloc<uint8_t>((size_t)lv.n_pad * dpad);
        lv.norms = dalloc<int32_t>(lv.n_pad);
        if (lv.n_pad > n) {
            MDH_CUDA(cudaMemsetAsync(lv.rows + (size_t)n * dpad, 0, (size_t)(lv.n_pad - n) * dpad, st));
            k_fill_i32<<<(unsigned)((lv.n_pad - n + 255) / 256), 256, 0, st>>>(lv.norms + n, lv.n_pad - n, kNormPad);
        }
    }
    if (f32) {
        lv.rows_f32 = dalloc<float>((size_t)lv.n_pad * dim);
        lv.norms_f32 = dalloc<float>(lv.n_pad);
    }
    if (lv.n_pad > n)
        k_fill_i32<<<(unsigned)((lv.n_pad - n + 255) / 256), 256, 0, st>>>(lv.ids + n, lv.n_pad - n, -1);
    MDH_CUDA(cudaGetLastError());
}

void finish_shard(mdh_index* ix, Shard& sh, bool u8, bool f32) {
    build_samples(ix, sh, u8, f32);
    if (u8)
        for (Level& lv : sh.levels) {
            if (tc_supported(ix, lv)) make_tmap_rows(lv, ix->dpad);
            if (tc2_supported(ix, lv)) make_tmap_rows_pair(lv, ix->dpad);
        }
    MDH_CUDA(cudaStreamSynchronize(sh.stream));
}

void build_shard_u8(mdh_index* ix, Shard& sh, const uint8_t* host_rows, int64_t n) {
    MDH_CUDA(cudaSetDevice(sh.device));
    cudaStream_t st = sh.stream;
    const int dpad = ix->dpad, dim = ix->dim;
    sh.n = n;
    Level full;
    alloc_level(full, n, dpad, dim, true, false, st);
    if (n > 0) {
        // Stage rows with the padded stride, then sort by (norm, row).
        uint8_t* stage = dalloc<uint8_t>((size_t)n * dpad);
        if (dpad != dim) MDH_CUDA(cudaMemsetAsync(stage, 0, (size_t)n * dpad, st));
        // cudaMemcpyDefault: the source may be host memory or (device build) memory of this device.
        MDH_CUDA(cudaMemcpy2DAsync(stage, dpad, host_rows, dim, dim, n, cudaMemcpyDefault, st));
        unsigned long long* keys = dalloc<unsigned long long>(n);
        unsigned long long* keys2 = dalloc<unsigned long long>(n);
        k_row_norms_u8<<<(unsigned)((n * 8 + 255) / 256), 256, 0, st>>>(stage, n, dpad, keys);
        MDH_CUDA(cudaGetLastError());
        size_t tmp_bytes = 0;
        cub::DeviceRadixSort::SortKeys(nullptr, tmp_bytes, keys, keys2, (int)n, 0, 64, st);
        void* tmp = dalloc<uint8_t>(tmp_bytes);
        MDH_CUDA(cub::DeviceRadixSort::SortKeys(tmp, tmp_bytes, keys, keys2, (int)n, 0, 64, st));
        k_gather_sorted<<<(unsigned)((n * 8 + 255) / 256), 256, 0, st>>>(stage, keys2, n, dpad, sh.id_base, full.rows,
                                                                        full.norms, full.ids);
        MDH_CUDA(cudaGetLastError());
        MDH_CUDA(cudaStreamSynchronize(st));
        cudaFree(tmp);
        cudaFree(keys);
        cudaFree(keys2);
        cudaFree(stage);
    }
    sh.levels.clear();
    sh.levels.push_back(full);
    finish_shard(ix, sh, true, false);
}

void build_shard_f32(mdh_index* ix, Shard& sh, const float* host_rows, int64_t n) {
    MDH_CUDA(cudaSetDevice(sh.device));
    cudaStream_t st = sh.stream;
    const int dim = ix->dim;
    sh.n = n;
    Level full;
    alloc_level(full, n, ix->dpad, dim, false, true, st);
    if (n > 0) {
        float* stage = dalloc<float>((size_t)n * dim);
        MDH_CUDA(cudaMemcpyAsync(stage, host_rows, (size_t)n * dim * sizeof(float), cudaMemcpyHostToDevice, st));
        k_prepare_f32<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(stage, nullptr, n, dim, ix->dpad,
                                                                  ix->metric == MDH_METRIC_COSINE, full.rows_f32,
                                                                  full.norms_f32);
        MDH_CUDA(cudaGetLastError());
        // Float corpora keep id order.
        std::vector<int32_t> hid((size_t)n);
        for (int64_t i = 0; i < n; i++) hid[(size_t)i] = (int32_t)(sh.id_base + i);
        MDH_CUDA(cudaMemcpyAsync(full.ids, hid.data(), (size_t)n * sizeof(int32_t), cudaMemcpyHostToDevice, st));
        MDH_CUDA(cudaStreamSynchronize(st));
        cudaFree(stage);
    }
    sh.levels.clear();
    sh.levels.push_back(full);
    finish_shard(ix, sh, false, true);
}

// Float rows for SpeedEngine cosine over a u8 corpus (normalized copy),
// built on first use.
void ensure_speed_rows_u8(mdh_index* ix, Shard& sh) {
    MDH_CUDA(cudaSetDevice(sh.device));
    for (Level& lv : sh.levels) {
        if (lv.rows_f32) continue;
        lv.rows_f32 = dalloc<float>((size_t)lv.n_pad * ix->dim);
        lv.norms_f32 = dalloc<float>(lv.n_pad);
        if (lv.n > 0) {
            k_prepare_f32<<<(unsigned)((lv.n + 127) / 128), 128, 0, sh.stream>>>(
                nullptr, lv.rows, lv.n, ix->dim, ix->dpad, ix->metric == MDH_METRIC_COSINE, lv.rows_f32, lv.norms_f32);
            MDH_CUDA(cudaGetLastError());
        }
    }
    MDH_CUDA(cudaStreamSynchronize(sh.stream));
}

void free_level_buffers(Level& lv) {
    if (lv.owns) {
        cudaFree(lv.rows_bf16);
        cudaFree(lv.rows);
        cudaFree(lv.norms);
        cudaFree(lv.ids);
        cudaFree(lv.rows_f32);
        cudaFree(lv.norms_f32);
    }
    lv = Level();
}

void free_workspace(Workspace& w) {
    void* ptrs[] = {w.q_u8, w.q_f32, w.q_bf16, w.qn, w.thr_key, w.thr_id, w.counts, w.cand, w.out_key, w.out_id, w.flags,
                    w.qlist, w.status, w.tmp};
    for (void* p : ptrs) cudaFree(p);
    if (w.h_status) cudaFreeHost(w.h_status);
    for (cudaEvent_t e : {w.ev0, w.ev1, w.ev_start, w.ev_sel, w.ev_rescore, w.ev_prep})
        if (e) cudaEventDestroy(e);
    w = Workspace();
}

void free_shard(Shard& sh) {
    cudaSetDevice(sh.device);
    for (Level& lv : sh.levels) free_level_buffers(lv);
    sh.levels.clear();
    free_workspace(sh.ws);
    if (sh.stream) cudaStreamDestroy(sh.stream);
    sh.stream = nullptr;
}

}  // namespace mdh
