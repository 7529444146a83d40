// CUDA-core scan kernels.
//
// Contract shared by every filter kernel (CUDA-core here, tensor-core in
// scan_tc.cu): for each query q and each real row r of a Level, compute the
// rank key of (q, r); when (key, id[r]) <= (thr_key[q], thr_id[q]) append
// {key, r} to query q's candidate list (slot = atomicAdd(counts[q]), stored
// only while slot < cap).  On a dense level (infinite thresholds, cap >= rows)
// row r goes to slot r with no atomics.  The selection step (select.cu) maps
// row positions to ids and turns candidate lists into thresholds or final
// top-k lists.
//
// Integer u8 kernels: 8 lanes cover one 128-byte row segment (16 bytes per
// lane, 128-bit loads, a warp reads 512 contiguous bytes), __dp4a forms the
// partial dot products and an 8-lane butterfly reduce-scatter leaves lane j
// of the group holding the full dot product of the row with query j, so one
// load of a row serves QG queries.
//
// Float kernels reproduce the reference's float evaluation order exactly
// (8 FMA lanes, left-to-right lane sum, scalar tail) with explicit
// round-to-nearest intrinsics so nvcc cannot contract or reorder them:
//   l2_sq_avx           src/winnex_madhava.cpp:119-146
//   exact_score cosine  src/winnex_madhava.cpp:714-763
//   dot_f32             src/speed_cpu.cpp:60-76 (scores :336-337, :386)
#include "internal.h"
#include "scan_common.cuh"

namespace mdh {

namespace {

// ---------------------------------------------------------------------------
// Query norms |q|^2 (int32) for u8 queries [nq][dpad].
__global__ void k_query_norms_u8(const uint8_t* __restrict__ q, int nq, int dpad, int32_t* __restrict__ qn) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= nq) return;
    const uint8_t* row = q + (size_t)warp * dpad;
    uint32_t s = 0;
    for (int off = lane * 16; off < dpad; off += 512) {
        uint4 v = *reinterpret_cast<const uint4*>(row + off);
        s = __dp4a(v.x, v.x, s);
        s = __dp4a(v.y, v.y, s);
        s = __dp4a(v.z, v.z, s);
        s = __dp4a(v.w, v.w, s);
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
    if (lane == 0) qn[warp] = (int32_t)s;
}

// MODE 0: L2 (key = |q|^2 + |v|^2 - 2 q.v, exact integer)
// MODE 1: cosine over u8 (key = descending order of dot / sqrt(|v|^2 |q|^2),
//         float arithmetic as exact_score, src/winnex_madhava.cpp:759-762)
template <int QG, int SEGS, int MODE>
__global__ void __launch_bounds__(256) k_filter_u8(
    const uint8_t* __restrict__ rows, const int32_t* __restrict__ norms, const int32_t* __restrict__ ids,
    int64_t n, int64_t n_pad, int dpad, const uint8_t* __restrict__ q, const int32_t* __restrict__ qn, int nq,
    const uint32_t* __restrict__ thr_key, const int32_t* __restrict__ thr_id, uint32_t* __restrict__ counts,
    uint2* __restrict__ cand, int cap, int dense) {
    const int lane = threadIdx.x & 31;
    const int l8 = lane & 7;
    const int grp = lane >> 3;
    const int64_t warp = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int q0 = blockIdx.y * QG;

    uint4 qv[QG][SEGS];
#pragma unroll
    for (int j = 0; j < QG; j++) {
#pragma unroll
        for (int s = 0; s < SEGS; s++) {
            if (q0 + j < nq)
                qv[j][s] = *reinterpret_cast<const uint4*>(q + (size_t)(q0 + j) * dpad + s * 128 + l8 * 16);
            else
                qv[j][s] = make_uint4(0, 0, 0, 0);
        }
    }
    // Per-lane view of its (row, query) pair after the reduce-scatter.
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
    float qn_f = (float)my_qn;

    constexpr int UNR = 4;
    for (int64_t base = warp * 4; base < n_pad; base += nwarps * 4 * UNR) {
        uint4 x[UNR][SEGS];
        int64_t r[UNR];
#pragma unroll
        for (int u = 0; u < UNR; u++) {
            r[u] = base + (int64_t)u * nwarps * 4 + grp;
#pragma unroll
            for (int s = 0; s < SEGS; s++) {
                if (r[u] < n_pad)
                    x[u][s] = __ldg(reinterpret_cast<const uint4*>(rows + (size_t)r[u] * dpad + s * 128 + l8 * 16));
                else
                    x[u][s] = make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int u = 0; u < UNR; u++) {
            uint32_t acc[QG];
#pragma unroll
            for (int j = 0; j < QG; j++) {
                uint32_t a = 0;
#pragma unroll
                for (int s = 0; s < SEGS; s++) {
                    a = __dp4a(x[u][s].x, qv[j][s].x, a);
                    a = __dp4a(x[u][s].y, qv[j][s].y, a);
                    a = __dp4a(x[u][s].z, qv[j][s].z, a);
                    a = __dp4a(x[u][s].w, qv[j][s].w, a);
                }
                acc[j] = a;
            }
            int qs2;
            bool act2;
            reduce_scatter8<QG>(acc, l8, qs2, act2);
            if (qvalid && r[u] < n) {
                const uint32_t dot = acc[0];
                const int32_t nv = __ldg(norms + r[u]);
                uint32_t key;
                if (MODE == 0) {
                    key = (uint32_t)(my_qn + nv - 2 * (int32_t)dot);
                } else {
                    float denom = __fsqrt_rn(__fmul_rn((float)nv, qn_f));
                    float sc = denom > 1e-10f ? __fdiv_rn((float)dot, denom) : 0.0f;
                    key = ordered_key_desc(sc);
                }
                offer_candidate(counts, cand, cap, dense, qi, key, r[u], ids, tkey, tid);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Float replica kernels: one thread per row, QG queries per block (staged in
// shared memory), all QG accumulator sets advance while the row streams once.
template <int KIND, int QG>
__global__ void __launch_bounds__(128) k_filter_f32(
    const uint8_t* __restrict__ rows_u8, const float* __restrict__ rows_f32, const int32_t* __restrict__ norms_i,
    const float* __restrict__ norms_f, const int32_t* __restrict__ ids, int64_t n, int dim, int dpad,
    const float* __restrict__ q, const float* __restrict__ qaux, int nq, const uint32_t* __restrict__ thr_key,
    const int32_t* __restrict__ thr_id, uint32_t* __restrict__ counts, uint2* __restrict__ cand, int cap, int dense) {
    extern __shared__ float sq[];  // [QG][dim]
    const int q0 = blockIdx.y * QG;
    for (int i = threadIdx.x; i < QG * dim; i += blockDim.x) {
        int j = i / dim;
        sq[i] = (q0 + j < nq) ? q[(size_t)(q0 + j) * dim + (i - j * dim)] : 0.0f;
    }
    __syncthreads();
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;

    float acc[QG][8];
    float acc2[QG][8];  // |v|^2 lanes for the cosine-over-u8 score
#pragma unroll
    for (int j = 0; j < QG; j++)
#pragma unroll
        for (int l = 0; l < 8; l++) { acc[j][l] = 0.0f; acc2[j][l] = 0.0f; }

    int jt = 0;  // start of the scalar tail
    if (KIND == kScoreL2SqU8 || KIND == kScoreCosU8) {
        const uint8_t* row = rows_u8 + (size_t)r * dpad;
        for (; jt + 16 <= dim; jt += 16) {
            uint4 w = *reinterpret_cast<const uint4*>(row + jt);
            const uint8_t* b = reinterpret_cast<const uint8_t*>(&w);
#pragma unroll
            for (int j = 0; j < QG; j++) {
                const float* qq = sq + j * dim + jt;
                if (KIND == kScoreL2SqU8) {
#pragma unroll
                    for (int l = 0; l < 8; l++) {
                        float d = __fsub_rn((float)b[l], qq[l]);
                        acc[j][l] = __fmaf_rn(d, d, acc[j][l]);
                    }
#pragma unroll
                    for (int l = 0; l < 8; l++) {
                        float d = __fsub_rn((float)b[8 + l], qq[8 + l]);
                        acc[j][l] = __fmaf_rn(d, d, acc[j][l]);
                    }
                } else {
#pragma unroll
                    for (int l = 0; l < 8; l++) acc[j][l] = __fmaf_rn((float)b[l], qq[l], acc[j][l]);
#pragma unroll
                    for (int l = 0; l < 8; l++) acc[j][l] = __fmaf_rn((float)b[8 + l], qq[8 + l], acc[j][l]);
                    if (j == 0) {
#pragma unroll
                        for (int l = 0; l < 8; l++) acc2[0][l] = __fmaf_rn((float)b[l], (float)b[l], acc2[0][l]);
#pragma unroll
                        for (int l = 0; l < 8; l++)
                            acc2[0][l] = __fmaf_rn((float)b[8 + l], (float)b[8 + l], acc2[0][l]);
                    }
                }
            }
        }
    } else {
        // SpeedEngine over a u8 corpus keeps (float)v rows (src/speed_cpu.cpp:124-127):
        // read the u8 row and convert, which is exact.
        const bool from_u8 = rows_f32 == nullptr;
        const float* row = from_u8 ? nullptr : rows_f32 + (size_t)r * dim;
        const uint8_t* row8 = rows_u8 + (size_t)r * dpad;
        if (KIND == kScoreExactCosF32) {
            jt = 0;  // scalar loop, handled below
        } else {
            for (; jt + 8 <= dim; jt += 8) {
                float v[8];
#pragma unroll
                for (int l = 0; l < 8; l++) v[l] = from_u8 ? (float)row8[jt + l] : __ldg(row + jt + l);
#pragma unroll
                for (int j = 0; j < QG; j++) {
                    const float* qq = sq + j * dim + jt;
#pragma unroll
                    for (int l = 0; l < 8; l++) acc[j][l] = __fmaf_rn(v[l], qq[l], acc[j][l]);
                }
            }
        }
    }

#pragma unroll
    for (int j = 0; j < QG; j++) {
        const int qi = q0 + j;
        if (qi >= nq) break;
        float s = 0.0f;
        uint32_t key;
        if (KIND == kScoreL2SqU8) {
            s = acc[j][0];
#pragma unroll
            for (int l = 1; l < 8; l++) s = __fadd_rn(s, acc[j][l]);
            const uint8_t* row = rows_u8 + (size_t)r * dpad;
            for (int t = jt; t < dim; t++) {
                float d = __fsub_rn((float)row[t], sq[j * dim + t]);
                s = __fmaf_rn(d, d, s);
            }
            key = ordered_key_asc(s);
        } else if (KIND == kScoreCosU8) {
            float dot = 0.0f, vn2 = 0.0f;
#pragma unroll
            for (int l = 0; l < 8; l++) { dot = __fadd_rn(dot, acc[j][l]); vn2 = __fadd_rn(vn2, acc2[0][l]); }
            const uint8_t* row = rows_u8 + (size_t)r * dpad;
            for (int t = jt; t < dim; t++) {
                float f = (float)row[t];
                dot = __fmaf_rn(f, sq[j * dim + t], dot);
                vn2 = __fmaf_rn(f, f, vn2);
            }
            float denom = __fsqrt_rn(__fmul_rn(vn2, qaux[qi]));
            float sc = denom > 1e-10f ? __fdiv_rn(dot, denom) : 0.0f;
            key = ordered_key_desc(sc);
        } else if (KIND == kScoreExactCosF32) {
            const float* row = rows_f32 + (size_t)r * dim;
            float dot = 0.0f, vn2 = 0.0f;
            for (int t = 0; t < dim; t++) {
                float vf = __ldg(row + t);
                dot = __fmaf_rn(vf, sq[j * dim + t], dot);
                vn2 = __fmaf_rn(vf, vf, vn2);
            }
            float denom = __fsqrt_rn(__fmul_rn(vn2, qaux[qi]));
            float sc = denom > 1e-10f ? __fdiv_rn(dot, denom) : 0.0f;
            key = ordered_key_desc(sc);
        } else {
            s = acc[j][0];
#pragma unroll
            for (int l = 1; l < 8; l++) s = __fadd_rn(s, acc[j][l]);
            if (rows_f32 == nullptr) {
                const uint8_t* row8 = rows_u8 + (size_t)r * dpad;
                for (int t = jt; t < dim; t++) s = __fmaf_rn((float)row8[t], sq[j * dim + t], s);
            } else {
                const float* row = rows_f32 + (size_t)r * dim;
                for (int t = jt; t < dim; t++) s = __fmaf_rn(__ldg(row + t), sq[j * dim + t], s);
            }
            if (KIND == kScoreSpeedL2) {
                // 2*ip - |v|^2 rounded once (src/speed_cpu.cpp:336-337, :386).
                const float nv = norms_f ? __ldg(norms_f + r) : (float)__ldg(norms_i + r);
                s = __fmaf_rn(2.0f, s, -nv);
            }
            key = ordered_key_desc(s);
        }
        offer_candidate(counts, cand, cap, dense, qi, key, r, ids, thr_key[qi], thr_id[qi]);
    }
}

template <int QG, int SEGS, int MODE>
void launch_u8_t(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq, const uint32_t* tk,
                 const int32_t* ti, uint32_t* counts, uint2* cand, int cap, int dense, cudaStream_t st) {
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    const int groups = (nq + QG - 1) / QG;
    // Enough CTAs to fill the GPU several times over; each warp covers
    // 4 rows per step, so cap the row blocks by the rows available.
    int64_t want = (int64_t)sms * 16 / groups;
    int64_t max_blocks = (lv.n_pad + 8 * 4 * 4 - 1) / (8 * 4 * 4);
    int64_t bx = want < 1 ? 1 : want;
    if (bx > max_blocks) bx = max_blocks;
    if (bx < 1) bx = 1;
    MDH_REQUIRE(groups <= 65535, MDH_ERR_INTERNAL, "too many query groups for one launch");
    dim3 grid((unsigned)bx, (unsigned)groups);
    k_filter_u8<QG, SEGS, MODE><<<grid, 256, 0, st>>>(lv.rows, lv.norms, lv.ids, lv.n, lv.n_pad, dpad, q, qn, nq, tk,
                                                      ti, counts, cand, cap, dense);
    MDH_CUDA(cudaGetLastError());
}

template <int MODE>
void launch_u8_dispatch(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq, const uint32_t* tk,
                        const int32_t* ti, uint32_t* counts, uint2* cand, int cap, int dense, cudaStream_t st) {
    const int segs = dpad / 128;
    if (segs == 1) {
        if (nq >= 8)
            launch_u8_t<8, 1, MODE>(lv, dpad, q, qn, nq, tk, ti, counts, cand, cap, dense, st);
        else if (nq >= 4)
            launch_u8_t<4, 1, MODE>(lv, dpad, q, qn, nq, tk, ti, counts, cand, cap, dense, st);
        else if (nq >= 2)
            launch_u8_t<2, 1, MODE>(lv, dpad, q, qn, nq, tk, ti, counts, cand, cap, dense, st);
        else
            launch_u8_t<1, 1, MODE>(lv, dpad, q, qn, nq, tk, ti, counts, cand, cap, dense, st);
    } else if (segs == 2) {
        if (nq >= 4)
            launch_u8_t<4, 2, MODE>(lv, dpad, q, qn, nq, tk, ti, counts, cand, cap, dense, st);
        else
            launch_u8_t<1, 2, MODE>(lv, dpad, q, qn, nq, tk, ti, counts, cand, cap, dense, st);
    } else {
        throw Error(MDH_ERR_INTERNAL, "integer u8 scan supports dim <= 256");
    }
}

template <int KIND>
void launch_f32_t(const Level& lv, int dim, int dpad, const float* q, const float* qaux, int nq, const uint32_t* tk,
                  const int32_t* ti, uint32_t* counts, uint2* cand, int cap, int dense, cudaStream_t st) {
    constexpr int QG = 4;
    const int groups = (nq + QG - 1) / QG;
    MDH_REQUIRE(groups <= 65535, MDH_ERR_INTERNAL, "too many query groups for one launch");
    size_t smem = (size_t)QG * dim * sizeof(float);
    MDH_REQUIRE(smem <= 200 * 1024, MDH_ERR_UNSUPPORTED, "dimension too large for the float scan");
    if (smem > 48 * 1024)
        MDH_CUDA(cudaFuncSetAttribute(k_filter_f32<KIND, QG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)((lv.n + 127) / 128), (unsigned)groups);
    if (lv.n == 0) return;
    k_filter_f32<KIND, QG><<<grid, 128, smem, st>>>(lv.rows, lv.rows_f32, lv.norms, lv.norms_f32, lv.ids, lv.n, dim,
                                                    dpad, q, qaux, nq, tk, ti, counts, cand, cap, dense);
    MDH_CUDA(cudaGetLastError());
}

}  // namespace

void launch_query_norms_u8(const uint8_t* q, int nq, int dpad, int32_t* qn, cudaStream_t st) {
    if (nq <= 0) return;
    int threads = 256;
    int blocks = (nq * 32 + threads - 1) / threads;
    k_query_norms_u8<<<blocks, threads, 0, st>>>(q, nq, dpad, qn);
    MDH_CUDA(cudaGetLastError());
}

void launch_filter_simt_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                              const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand,
                              int cap, int dense, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    launch_u8_dispatch<0>(lv, dpad, q, qn, nq, thr_key, thr_id, counts, cand, cap, dense, st);
}

void launch_filter_simt_u8_cos(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                               const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand,
                               int cap, int dense, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    launch_u8_dispatch<1>(lv, dpad, q, qn, nq, thr_key, thr_id, counts, cand, cap, dense, st);
}

void launch_filter_f32(const Level& lv, int dim, int dpad, int score_kind, const float* q, int nq,
                       const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap,
                       int dense, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    // qaux (per-query |q|^2 for the cosine scores) is stored right after the
    // nq x dim query block by the caller.
    const float* qaux = q + (size_t)nq * dim;
    switch (score_kind) {
        case kScoreL2SqU8: launch_f32_t<kScoreL2SqU8>(lv, dim, dpad, q, qaux, nq, thr_key, thr_id, counts, cand, cap, dense, st); break;
        case kScoreCosU8: launch_f32_t<kScoreCosU8>(lv, dim, dpad, q, qaux, nq, thr_key, thr_id, counts, cand, cap, dense, st); break;
        case kScoreSpeedL2: launch_f32_t<kScoreSpeedL2>(lv, dim, dpad, q, qaux, nq, thr_key, thr_id, counts, cand, cap, dense, st); break;
        case kScoreSpeedCos: launch_f32_t<kScoreSpeedCos>(lv, dim, dpad, q, qaux, nq, thr_key, thr_id, counts, cand, cap, dense, st); break;
        case kScoreExactCosF32: launch_f32_t<kScoreExactCosF32>(lv, dim, dpad, q, qaux, nq, thr_key, thr_id, counts, cand, cap, dense, st); break;
        default: throw Error(MDH_ERR_INTERNAL, "unknown score kind");
    }
}

}  // namespace mdh
