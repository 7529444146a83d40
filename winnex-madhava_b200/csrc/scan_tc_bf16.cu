// Approximate bf16 tensor-core scan for float cosine scores (SpeedEngine
// cosine, src/speed_cpu.cpp:88-101 and :271-398), sm_100a.
//
// The reference scores a normalized float row v against a normalized float
// query q by an fp32 dot product.  This scan forms the same dot product from
// bf16 copies of v and q on tcgen05 (kind::f16, fp32 accumulators in tensor
// memory) and keeps every pair whose bf16 score is >= T - eps, T the query's
// threshold score.  With unit roundoff u = 2^-8 of bf16, |bf16 score - exact
// dot| <= (2u + u^2) sum_j |q_j v_j| <= (2u + u^2) |q| |v|, so for unit
// vectors the bf16 score is within 2^-7 + 2^-16 of the true dot product, and
// the fp32 accumulations (here and in the reference) add at most dim * 2^-24
// each; the caller passes eps covering the sum.  No pair with exact score
// >= T is dropped.  launch_rescore_speed_cos then recomputes every kept
// pair's score with the reference's fp32 arithmetic (8 lanes of fused
// multiply-adds, a left-to-right lane sum, then the scalar tail), so ranking
// and returned scores are the reference's own.
//
// Tile: 128 queries x 256 rows; the dimension is streamed in blocks of 64
// bf16 (one 128-byte swizzle row): each stage holds the query block (16 KB)
// and the row block (32 KB), 4 stages.  Warp roles as in scan_tc.cu: 16
// epilogue warps (TMEM lane quarter w % 4, 64 columns of the 256), a TMA
// producer and a single-thread MMA issuer.  Every mbarrier wait is bounded.
#include <cuda_bf16.h>

#include <algorithm>

#include "internal.h"
#include "tc_ptx.cuh"

namespace mdh {

namespace {

using namespace tc;

constexpr int BM = 128, BN = 256;
constexpr int KB = 64;                     // bf16 elements per dimension block (128 bytes)
constexpr int STAGES = 4;
constexpr int ACC_STAGES = 2;
constexpr int TMEM_COLS = 512;
constexpr int EPI_WARPS = 16;
constexpr int COLS_PER_WARP = 64;
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int PRODUCER_WARP = EPI_WARPS;
constexpr int MMA_WARP = EPI_WARPS + 1;
constexpr int NUM_THREADS = 32 * (EPI_WARPS + 2);
constexpr int BUFN = 4;
constexpr int MAX_KBLOCKS = 16;            // dim <= 1024
constexpr uint32_t A_BYTES = BM * 128;
constexpr uint32_t B_BYTES = BN * 128;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t OFF_BUF = STAGES * STAGE_BYTES;
constexpr uint32_t OFF_BAR = OFF_BUF + BUFN * EPI_THREADS * 8;
constexpr uint32_t BAR_FULL = 0, BAR_EMPTY = STAGES, BAR_ACC_FULL = 2 * STAGES, BAR_ACC_EMPTY = 2 * STAGES + ACC_STAGES,
                   BAR_DRAIN = 2 * STAGES + 2 * ACC_STAGES, NUM_BARS = BAR_DRAIN + 1;
constexpr uint32_t OFF_TMEM_SLOT = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t OFF_ABORT = OFF_TMEM_SLOT + 4;
constexpr uint32_t SMEM_BYTES = OFF_ABORT + 4 + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
static_assert(A_BYTES % 1024 == 0 && STAGE_BYTES % 1024 == 0, "swizzle alignment");
// kind::f16 instruction descriptor: D f32 (1 << 4), A and B bf16, both K-major.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

struct SchedB {
    int n_groups, n_tiles, n_chunks, nkb;
    long long n_units;
};

__device__ __forceinline__ void unit_coords(const SchedB& s, long long u, int& g, int& t0, int& t1) {
    const int c = (int)(u / s.n_groups);
    g = (int)(u - (long long)c * s.n_groups);
    t0 = (int)((long long)c * s.n_tiles / s.n_chunks);
    t1 = (int)((long long)(c + 1) * s.n_tiles / s.n_chunks);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ float fmax32f(const uint32_t (&v)[32]) {
    float t[11];
#pragma unroll
    for (int i = 0; i < 10; i++)
        t[i] = fmax3(__uint_as_float(v[3 * i]), __uint_as_float(v[3 * i + 1]), __uint_as_float(v[3 * i + 2]));
    t[10] = fmaxf(__uint_as_float(v[30]), __uint_as_float(v[31]));
    const float u0 = fmax3(t[0], t[1], t[2]), u1 = fmax3(t[3], t[4], t[5]), u2 = fmax3(t[6], t[7], t[8]);
    return fmaxf(fmax3(u0, u1, u2), fmaxf(t[9], t[10]));
}

__device__ __forceinline__ uint32_t pass_mask32f(const uint32_t (&v)[32], float need) {
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < 32; j++) m |= (__uint_as_float(v[j]) >= need ? 1u : 0u) << j;
    return m;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_filter_tc_bf16_cos(const __grid_constant__ CUtensorMap tmap_rows, const __grid_constant__ CUtensorMap tmap_q,
                         int32_t n_rows, int nq, const uint32_t* __restrict__ thr_key, uint32_t* __restrict__ counts,
                         uint2* __restrict__ cand, int cap, int dense, float eps, SchedB sched,
                         int32_t* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + OFF_BAR;
    volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + OFF_ABORT);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM_SLOT);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nkb = sched.nkb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bars + 8 * (BAR_FULL + s), 1);
            mbar_init(bars + 8 * (BAR_EMPTY + s), 1);
        }
        for (int s = 0; s < ACC_STAGES; s++) {
            mbar_init(bars + 8 * (BAR_ACC_FULL + s), 1);
            mbar_init(bars + 8 * (BAR_ACC_EMPTY + s), EPI_WARPS);
        }
        mbar_init(bars + 8 * BAR_DRAIN, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == MMA_WARP) tmem_alloc<1>(smem_u32(tmem_slot), TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == PRODUCER_WARP) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_rows) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_parity = 0;
            bool ok = true;
            for (long long u = blockIdx.x; u < sched.n_units && ok; u += gridDim.x) {
                int g, t0, t1;
                unit_coords(sched, u, g, t0, t1);
                for (int t = t0; t < t1 && ok; t++) {
                    for (int kb = 0; kb < nkb; kb++) {
                        ok = mbar_wait<false>(bars + 8 * (BAR_EMPTY + stage), phase ^ 1, abort_flag, status);
                        if (!ok) break;
                        const uint32_t full = bars + 8 * (BAR_FULL + stage);
                        mbar_expect_tx(full, STAGE_BYTES);
                        tma_load_2d(sbase + stage * STAGE_BYTES, &tmap_q, full, kb * KB, g * BM);
                        tma_load_2d(sbase + stage * STAGE_BYTES + A_BYTES, &tmap_rows, full, kb * KB, t * BN);
                        tma_load_2d(sbase + stage * STAGE_BYTES + A_BYTES + B_BYTES / 2, &tmap_rows, full, kb * KB,
                                    t * BN + BN / 2);
                        issued_mask |= 1u << stage;
                        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                        if (++stage == STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            if (!ok)
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s))
                        mbar_drain_wait<false>(bars + 8 * (BAR_FULL + s), (last_parity >> s) & 1);
        }
    } else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        // The next dimension block's stage is probed between this block's
        // MMAs (a blocking wait would leave the tensor pipe idle).
        if (lane == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true, issued = false, full_ready = false;
            for (long long u = blockIdx.x; u < sched.n_units && ok; u += gridDim.x) {
                int g, t0, t1;
                unit_coords(sched, u, g, t0, t1);
                for (int t = t0; t < t1 && ok; t++) {
                    ok = mbar_wait_inl<false>(bars + 8 * (BAR_ACC_EMPTY + acc), acc_phase ^ 1, abort_flag, status);
                    if (!ok) break;
                    const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                    for (int kb = 0; kb < nkb; kb++) {
                        if (!full_ready) {
                            ok = mbar_wait_inl<false>(bars + 8 * (BAR_FULL + stage), phase, abort_flag, status);
                            if (!ok) break;
                        }
                        tc_fence_after();
                        const int nstage = stage + 1 == STAGES ? 0 : stage + 1;
                        const uint32_t nphase = stage + 1 == STAGES ? phase ^ 1 : phase;
                        const uint64_t adesc = sw128_desc(sbase + stage * STAGE_BYTES);
                        const uint64_t bdesc = sw128_desc(sbase + stage * STAGE_BYTES + A_BYTES);
                        bool pf = false;
#pragma unroll
                        for (int kk = 0; kk < KB / 16; kk++) {
                            umma_bf16(d, adesc + (uint64_t)((kk * 32) >> 4), bdesc + (uint64_t)((kk * 32) >> 4),
                                      (kb > 0 || kk > 0) ? 1u : 0u);
                            if (kk == 1) pf = mbar_test_wait(bars + 8 * (BAR_FULL + nstage), nphase);
                        }
                        issued = true;
                        umma_commit(bars + 8 * (BAR_EMPTY + stage));
                        full_ready = pf;
                        stage = nstage;
                        phase = nphase;
                    }
                    if (!ok) break;
                    umma_commit(bars + 8 * (BAR_ACC_FULL + acc));
                    if (++acc == ACC_STAGES) {
                        acc = 0;
                        acc_phase ^= 1;
                    }
                }
            }
            if (!ok && issued) {
                umma_commit(bars + 8 * BAR_DRAIN);
                mbar_drain_wait<false>(bars + 8 * BAR_DRAIN, 0);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 0-15)
        const int quarter = warp & 3, part = warp >> 2;
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        CandBuf<EPI_THREADS, BUFN> buf;
        buf.base = reinterpret_cast<uint2*>(smem + OFF_BUF) + threadIdx.x;
        buf.n = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (long long u = blockIdx.x; u < sched.n_units && ok; u += gridDim.x) {
            int g, t0, t1;
            unit_coords(sched, u, g, t0, t1);
            const int qi = g * BM + quarter * 32 + lane;
            const bool qvalid = qi < nq;
            // need = T - eps; an infinite threshold keeps every row, an invalid
            // query none.
            float need = INFINITY;
            if (qvalid) {
                const uint32_t tk = thr_key[qi];
                need = tk == kKeyInf ? -INFINITY : key_to_float_asc(~tk) - eps;
            }
            for (int t = t0; t < t1; t++) {
                ok = mbar_wait_inl<false>(bars + 8 * (BAR_ACC_FULL + acc), acc_phase, abort_flag, status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tcol = tmem_base + lane_base + (uint32_t)(acc * BN + part * COLS_PER_WARP);
                uint32_t v[2][32];
                __syncwarp();
                tmem_ld32_issue(tcol, v[0]);
                tmem_ld32_issue(tcol + 32, v[1]);
                tmem_ld_wait(v[0]);
                tmem_ld_wait(v[1]);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bars + 8 * (BAR_ACC_EMPTY + acc));
                if (++acc == ACC_STAGES) {
                    acc = 0;
                    acc_phase ^= 1;
                }
                if (fmax32f(v[0]) < need && fmax32f(v[1]) < need) continue;
                const int32_t row0 = t * BN + part * COLS_PER_WARP;
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    uint32_t mask = pass_mask32f(v[c], need);
                    while (mask) {
                        const int j = __ffs(mask) - 1;
                        mask &= mask - 1;
                        const int32_t r = row0 + 32 * c + j;
                        if (r >= n_rows) break;  // pad rows trail the level
                        const uint32_t key = ordered_key_desc(__uint_as_float(pick32(v[c], j)));
                        if (dense)
                            cand[(size_t)qi * cap + r] = make_uint2(key, (uint32_t)r);
                        else
                            buf.push(key, (uint32_t)r, counts, cand, cap, qi);
                    }
                }
            }
            if (qvalid) buf.flush(counts, cand, cap, qi);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, TMEM_COLS);
    }
}

__global__ void k_convert_bf16(const float* __restrict__ src, int64_t count, __nv_bfloat16* __restrict__ dst) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) dst[i] = __float2bfloat16_rn(src[i]);
}

// The reference's SpeedEngine score of a normalized float row against a
// normalized float query (dot_f32, src/speed_cpu.cpp:60-76): lane l of 8
// accumulates fused multiply-adds of elements l, l + 8, l + 16, ...; the 8
// lanes are summed left to right, then the scalar tail -- the operations and
// order of k_filter_f32 (scan_simt.cu).  A warp rescores 4 candidates at a
// time: threads 8c .. 8c + 7 run the 8 lane chains of candidate c.  The rows
// are read in 128-float segments, one coalesced 512-byte float4 load per
// candidate and thread, staged in the warp's shared buffer; each thread then
// folds its chain's 16 elements of the segment in order.  One block per
// query; the query row sits in shared memory.
constexpr int RESCORE_WARPS = 8;
constexpr int RESCORE_SEG = 128;  // floats per staged segment

__global__ void __launch_bounds__(RESCORE_WARPS * 32) k_rescore_speed_cos(const uint32_t* __restrict__ counts,
                                                                          uint2* __restrict__ cand, int cap,
                                                                          const float* __restrict__ rows, int dim,
                                                                          const float* __restrict__ q, int nq) {
    extern __shared__ float4 smem4[];
    float* sq = reinterpret_cast<float*>(smem4);                        // [dim rounded up to 4]
    const int qi = blockIdx.x;
    if (qi >= nq) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4* wbuf = smem4 + (dim + 3) / 4 + warp * (4 * RESCORE_SEG / 4);  // [4][128] floats of this warp
    const float* wf = reinterpret_cast<const float*>(wbuf);
    for (int j = threadIdx.x; j < dim; j += blockDim.x) sq[j] = q[(size_t)qi * dim + j];
    __syncthreads();
    const uint32_t c_all = counts[qi];
    const int c = (int)(c_all < (uint32_t)cap ? c_all : (uint32_t)cap);
    uint2* lst = cand + (size_t)qi * cap;
    const int g = lane >> 3, l = lane & 7;  // this thread: chain l of candidate g
    const int jt_end = dim & ~7;
    const bool vec = (dim & 3) == 0;         // rows are 16-byte aligned for float4 reads
    for (int i0 = warp * 4; i0 < c; i0 += RESCORE_WARPS * 4) {
        uint32_t r4[4];
#pragma unroll
        for (int h = 0; h < 4; h++) r4[h] = i0 + h < c ? lst[i0 + h].y : 0xffffffffu;
        float acc = 0.0f;
        for (int s0 = 0; s0 < jt_end; s0 += RESCORE_SEG) {
            float4 x[4];
#pragma unroll
            for (int h = 0; h < 4; h++) {
                const int e = s0 + 4 * lane;
                x[h] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (r4[h] != 0xffffffffu && e < dim) {
                    const float* src = rows + (size_t)r4[h] * dim + e;
                    if (vec && e + 3 < dim) {
                        x[h] = __ldg(reinterpret_cast<const float4*>(src));
                    } else {
                        x[h].x = __ldg(src);
                        if (e + 1 < dim) x[h].y = __ldg(src + 1);
                        if (e + 2 < dim) x[h].z = __ldg(src + 2);
                        if (e + 3 < dim) x[h].w = __ldg(src + 3);
                    }
                }
            }
            __syncwarp();  // the previous segment's folds are done with the buffer
#pragma unroll
            for (int h = 0; h < 4; h++) wbuf[h * (RESCORE_SEG / 4) + lane] = x[h];
            __syncwarp();
            const float* seg = wf + g * RESCORE_SEG;
#pragma unroll
            for (int m = 0; m < RESCORE_SEG / 8; m++) {
                const int jt = s0 + 8 * m;
                if (jt < jt_end) acc = __fmaf_rn(seg[8 * m + l], sq[jt + l], acc);
            }
        }
        const int gbase = g * 8;
        float sum = __shfl_sync(0xffffffffu, acc, gbase);
#pragma unroll
        for (int mm = 1; mm < 8; mm++) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, acc, gbase + mm));
        if (l == 0 && r4[g] != 0xffffffffu) {
            const float* row = rows + (size_t)r4[g] * dim;
            for (int t = jt_end; t < dim; t++) sum = __fmaf_rn(__ldg(row + t), sq[t], sum);
            lst[i0 + g].x = ordered_key_desc(sum);
        }
    }
}

}  // namespace

// A dense level's lists hold every row with its bf16 score.  Only rows whose
// bf16 score is within 2 eps of the list's k-th bf16 score s' can be in its
// exact top k: k rows score >= s' in bf16, so >= s' - eps exactly, so the
// exact k-th score is >= s' - eps and every row of the exact top k has a
// bf16 score >= s' - 2 eps.  thr_key holds s' (k-th key, from a selection);
// each list is compacted in place, in order, to those rows (one block per
// query, chunk by chunk: a chunk is read before any of its slots is
// written).  A list with fewer than k rows (infinite threshold) is kept.
__global__ void __launch_bounds__(256) k_compact_bf16_band(uint32_t* __restrict__ counts, uint2* __restrict__ cand,
                                                           int cap, const uint32_t* __restrict__ thr_key,
                                                           float two_eps) {
    __shared__ uint32_t warp_n[8];
    __shared__ uint32_t base_s;
    const int qi = blockIdx.x;
    const uint32_t tk = thr_key[qi];
    if (tk == kKeyInf) return;
    const uint32_t c_all = counts[qi];
    const int c = (int)(c_all < (uint32_t)cap ? c_all : (uint32_t)cap);
    uint2* lst = cand + (size_t)qi * cap;
    const float lo = __fsub_rd(key_to_float_asc(~tk), two_eps);
    const uint32_t bound = ordered_key_desc(lo);  // key <= bound  <=>  bf16 score >= lo
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) base_s = 0;
    __syncthreads();
    for (int i0 = 0; i0 < c; i0 += blockDim.x) {
        const int i = i0 + threadIdx.x;
        const uint2 e = i < c ? lst[i] : make_uint2(0xffffffffu, 0u);
        const bool keep = i < c && e.x <= bound;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) warp_n[warp] = __popc(bal);
        __syncthreads();  // every entry of this chunk is read
        uint32_t before = base_s;
        for (int w = 0; w < warp; w++) before += warp_n[w];
        if (keep) lst[before + __popc(bal & ((1u << lane) - 1u))] = e;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t t = base_s;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += warp_n[w];
            base_s = t;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) counts[qi] = base_s;
}

bool tc_bf16_supported(const mdh_index* ix, const Level& lv) {
    return ix && ix->dim % 8 == 0 && ix->dim <= KB * MAX_KBLOCKS && lv.rows_f32 && lv.n_pad % BN == 0 &&
           lv.n_pad < (int64_t(1) << 31);
}

void ensure_bf16_rows(mdh_index* ix, Shard& sh) {
    MDH_CUDA(cudaSetDevice(sh.device));
    for (Level& lv : sh.levels) {
        if (lv.rows_bf16 || !lv.rows_f32 || !tc_bf16_supported(ix, lv)) continue;
        const int64_t count = lv.n_pad * (int64_t)ix->dim;
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, (size_t)count * 2);
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw Error(MDH_ERR_OOM, std::string("device allocation failed: ") + cudaGetErrorString(e));
        }
        lv.rows_bf16 = static_cast<uint16_t*>(p);
        k_convert_bf16<<<(unsigned)((count + 255) / 256), 256, 0, sh.stream>>>(
            lv.rows_f32, count, reinterpret_cast<__nv_bfloat16*>(lv.rows_bf16));
        MDH_CUDA(cudaGetLastError());
        encode_tmap_2d_sw128(&lv.tmap_bf16, 1, lv.rows_bf16, (uint64_t)ix->dim, (uint64_t)lv.n_pad,
                             (uint64_t)ix->dim * 2, KB, BN / 2);
        lv.has_tmap_bf16 = true;
    }
    MDH_CUDA(cudaStreamSynchronize(sh.stream));
}

void launch_convert_bf16(const float* src, int64_t count, uint16_t* dst, cudaStream_t st) {
    if (count <= 0) return;
    k_convert_bf16<<<(unsigned)((count + 255) / 256), 256, 0, st>>>(src, count, reinterpret_cast<__nv_bfloat16*>(dst));
    MDH_CUDA(cudaGetLastError());
}

void launch_filter_tc_bf16_cos(const Level& lv, int dim, const uint16_t* q_bf16, int nq, const uint32_t* thr_key,
                               uint32_t* counts, uint2* cand, int cap, int dense, float eps, int32_t* status,
                               cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    MDH_REQUIRE(lv.has_tmap_bf16, MDH_ERR_INTERNAL, "bf16 scan needs the bf16 rows");
    MDH_REQUIRE(!dense || cap >= lv.n, MDH_ERR_INTERNAL, "dense scan needs cap >= rows");
    MDH_REQUIRE((reinterpret_cast<uintptr_t>(q_bf16) & 15) == 0 && (dim * 2) % 16 == 0, MDH_ERR_INTERNAL,
                "bf16 queries must be 16-byte aligned rows");
    CUtensorMap tq;
    encode_tmap_2d_sw128(&tq, 1, q_bf16, (uint64_t)dim, (uint64_t)nq, (uint64_t)dim * 2, KB, BM);
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    SchedB s;
    s.n_groups = (nq + BM - 1) / BM;
    s.n_tiles = (int)(lv.n_pad / BN);
    s.nkb = (dim + KB - 1) / KB;
    int ctas = sms;
    s.n_chunks = choose_scan_chunks(s.n_groups, s.n_tiles, ctas, 16);  // a tile streams 12 dimension blocks
    s.n_units = (long long)s.n_groups * s.n_chunks;
    if (s.n_units < ctas) ctas = (int)s.n_units;
    MDH_CUDA(cudaFuncSetAttribute(k_filter_tc_bf16_cos, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
    k_filter_tc_bf16_cos<<<ctas, NUM_THREADS, SMEM_BYTES, st>>>(lv.tmap_bf16, tq, (int32_t)lv.n, nq, thr_key, counts,
                                                                cand, cap, dense, eps, s, status);
    MDH_CUDA(cudaGetLastError());
}

namespace {

// SpeedEngine query normalization (src/speed_cpu.cpp:278-287 single query,
// :365-372 batch) on the device, in the reference's fp32 order: |q|^2 by a
// sequential FMA chain, then the scale 1/sqrt, then one multiply per element.
// One warp per query: lane 0 runs the chain, the warp scales and writes the
// fp32 row in place and its bf16 copy (bf16 may be null).
__global__ void k_normalize_speed_cos(float* __restrict__ q, int nq, int dim, int batch_guard,
                                      __nv_bfloat16* __restrict__ q_bf16) {
    const int qi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (qi >= nq) return;
    float* row = q + (size_t)qi * dim;
    float inv = 0.0f;
    if (lane == 0) {
        float qn = 0.0f;
        for (int j = 0; j < dim; j++) qn = __fmaf_rn(row[j], row[j], qn);
        if (batch_guard) {
            inv = qn > 1e-12f ? __fdiv_rn(1.0f, __fsqrt_rn(qn)) : 0.0f;
        } else {
            const float s = __fsqrt_rn(qn);
            inv = s > 1e-12f ? __fdiv_rn(1.0f, s) : 0.0f;
        }
    }
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int j = lane; j < dim; j += 32) {
        const float x = __fmul_rn(row[j], inv);
        row[j] = x;
        if (q_bf16) q_bf16[(size_t)qi * dim + j] = __float2bfloat16_rn(x);
    }
}

}  // namespace

void launch_normalize_speed_cos(float* q, int nq, int dim, int batch_guard, uint16_t* q_bf16, cudaStream_t st) {
    if (nq <= 0) return;
    k_normalize_speed_cos<<<(nq + 7) / 8, 256, 0, st>>>(q, nq, dim, batch_guard,
                                                        reinterpret_cast<__nv_bfloat16*>(q_bf16));
    MDH_CUDA(cudaGetLastError());
}

void launch_compact_bf16_band(uint32_t* counts, uint2* cand, int cap, const uint32_t* thr_key, float two_eps, int nq,
                              cudaStream_t st) {
    if (nq <= 0) return;
    k_compact_bf16_band<<<nq, 256, 0, st>>>(counts, cand, cap, thr_key, two_eps);
    MDH_CUDA(cudaGetLastError());
}

void launch_rescore_speed_cos(const uint32_t* counts, uint2* cand, int cap, const float* rows_f32, int dim,
                              const float* q_f32, int nq, cudaStream_t st) {
    if (nq <= 0) return;
    const size_t smem = (size_t)(dim + 3) / 4 * 16 + (size_t)RESCORE_WARPS * 4 * RESCORE_SEG * sizeof(float);
    MDH_REQUIRE(smem <= 48 * 1024, MDH_ERR_UNSUPPORTED, "dimension too large for the rescore kernel");
    k_rescore_speed_cos<<<nq, RESCORE_WARPS * 32, smem, st>>>(counts, cand, cap, rows_f32, dim, q_f32, nq);
    MDH_CUDA(cudaGetLastError());
}

}  // namespace mdh
