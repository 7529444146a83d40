// Tensor-core (tcgen05) u8 L2 scan for sm_100a.
//
// Same contract as the CUDA-core filter (scan_simt.cu): for each query q and
// real row r of a Level, key = |q|^2 + |v|^2 - 2 q.v; pairs with
// (key, id) <= (thr_key[q], thr_id[q]) are appended to q's candidate list.
//
// Tile: 128 queries (TMEM lanes, the MMA's M) x 256 corpus rows (the MMA's N)
// x 128 bytes (K: four kind::i8 MMAs of K = 32).  u8 x u8 products
// accumulate exactly in s32 in tensor memory.  Operands are staged by TMA
// with the 128-byte swizzle (one 128-byte row per vector = one swizzle row).
//
// Warp roles (192 threads, one CTA per SM, persistent):
//   warps 0-3  epilogue: tcgen05.ld 32 columns per thread per step (thread =
//              one query), per-chunk Cauchy-Schwarz filter, rare appends;
//   warp 4     TMA producer (query tile once per work unit, corpus tiles
//              through a STAGES-deep ring);
//   warp 5     TMEM allocator + single-thread MMA issuer.
// Two accumulator stages (2 x 256 of the 512 TMEM columns) let the MMA of
// tile t+1 run while the epilogue drains tile t.
//
// Epilogue filter: rows are sorted by |v|^2, so the first row of each
// 32-row chunk has the chunk's smallest norm n_min.  With m = max q.v over
// the chunk, every key in the chunk is >= |q|^2 + n_min - 2m; when that
// exceeds the query's threshold the whole chunk is skipped after one max
// reduction.  The dot products are below 2^23 (128 * 255^2 < 2^23), so their
// s32 bit patterns order like positive subnormal floats and the 3-input
// max.f32 of sm_100 reduces them directly.
//
// Work units: (query tile, corpus chunk), ordered chunk-major so the CTAs
// running at the same time share corpus chunks through L2; each CTA takes
// units blockIdx.x, blockIdx.x + gridDim.x, ...
//
// Every mbarrier wait is bounded (clock64 budget).  On expiry the kernel
// writes kDevTimeout to *status, raises a shared abort flag so every role
// leaves its loop, drains its own outstanding TMA loads and MMAs with bounded
// waits, frees its tensor memory and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "internal.h"

namespace mdh {

namespace {

constexpr int BM = 128;           // queries per tile (TMEM lanes)
constexpr int BN = 256;           // corpus rows per tile
constexpr int BK = 128;           // bytes per row (K)
constexpr int STAGES = 4;         // corpus tile ring depth
constexpr int ACC_STAGES = 2;
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 192;
constexpr uint32_t A_BYTES = BM * BK;
constexpr uint32_t B_BYTES = BN * BK;
constexpr long long kWaitBudget = 4000000000ll;  // cycles (~2 s)

// Shared memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_B = OFF_A + A_BYTES;
constexpr uint32_t OFF_BAR = OFF_B + STAGES * B_BYTES;
constexpr uint32_t BAR_FULL = 0, BAR_EMPTY = STAGES, BAR_ACC_FULL = 2 * STAGES,
                   BAR_ACC_EMPTY = 2 * STAGES + ACC_STAGES, BAR_A_FULL = 2 * STAGES + 2 * ACC_STAGES,
                   BAR_A_EMPTY = BAR_A_FULL + 1, BAR_DRAIN = BAR_A_FULL + 2, NUM_BARS = BAR_A_FULL + 3;
constexpr uint32_t OFF_TMEM_SLOT = OFF_BAR + NUM_BARS * 8;
constexpr uint32_t OFF_ABORT = OFF_TMEM_SLOT + 4;
constexpr uint32_t SMEM_USED = OFF_ABORT + 4;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;  // alignment slack

// Instruction descriptor: D s32, A/B u8, both K-major, N = 256, M = 128.
constexpr uint32_t IDESC = (2u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false when the CTA is aborting (this wait timed out, or another role's did).
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int32_t* abort_flag, int32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitBudget) {
            *abort_flag = 1;
            atomicExch(status, (int32_t)kDevTimeout);
            return false;
        }
    }
}

// Bounded wait used while draining after an abort (ignores the abort flag).
__device__ __noinline__ void mbar_drain_wait(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitBudget) return;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    // Shared-memory matrix descriptor, K-major, 128-byte swizzle:
    // start >> 4 | LBO 16 B (unused for swizzled K-major) | SBO 1024 B
    // (8 rows x 128 B) | version 1 | layout SWIZZLE_128B (2).
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Load 32 consecutive TMEM columns of this thread's lane and wait for them
// in one statement, so no use of the registers can precede the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// Max of 32 non-negative s32 values below 2^23 (ordered as subnormal floats).
__device__ __forceinline__ int32_t max32(const uint32_t (&v)[32]) {
    float t[11];
#pragma unroll
    for (int i = 0; i < 10; i++)
        t[i] = fmax3(__uint_as_float(v[3 * i]), __uint_as_float(v[3 * i + 1]), __uint_as_float(v[3 * i + 2]));
    t[10] = fmaxf(__uint_as_float(v[30]), __uint_as_float(v[31]));
    float u0 = fmax3(t[0], t[1], t[2]), u1 = fmax3(t[3], t[4], t[5]), u2 = fmax3(t[6], t[7], t[8]);
    float u3 = fmaxf(t[9], t[10]);
    return (int32_t)__float_as_uint(fmaxf(fmax3(u0, u1, u2), u3));
}

struct Sched {
    int n_qtiles;     // G
    int n_tiles;      // corpus tiles of BN rows
    int n_chunks;     // corpus chunks per query tile
    long long n_units;
};

__device__ __forceinline__ void unit_coords(const Sched& s, long long u, int& g, int& t0, int& t1) {
    const int c = (int)(u / s.n_qtiles);
    g = (int)(u - (long long)c * s.n_qtiles);
    t0 = (int)((long long)c * s.n_tiles / s.n_chunks);
    t1 = (int)((long long)(c + 1) * s.n_tiles / s.n_chunks);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_filter_tc_u8_l2(const __grid_constant__ CUtensorMap tmap_rows, const __grid_constant__ CUtensorMap tmap_q,
                      const int32_t* __restrict__ norms, const int32_t* __restrict__ ids, int64_t n_rows,
                      const int32_t* __restrict__ qn, int nq, const uint32_t* __restrict__ thr_key,
                      const int32_t* __restrict__ thr_id, uint32_t* __restrict__ counts, uint2* __restrict__ cand,
                      int cap, Sched sched, int32_t* __restrict__ status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + OFF_BAR;
    volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + OFF_ABORT);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + OFF_TMEM_SLOT);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bars + 8 * (BAR_FULL + s), 1);
            mbar_init(bars + 8 * (BAR_EMPTY + s), 1);
        }
        for (int s = 0; s < ACC_STAGES; s++) {
            mbar_init(bars + 8 * (BAR_ACC_FULL + s), 1);
            mbar_init(bars + 8 * (BAR_ACC_EMPTY + s), 4);
        }
        mbar_init(bars + 8 * BAR_A_FULL, 1);
        mbar_init(bars + 8 * BAR_A_EMPTY, 1);
        mbar_init(bars + 8 * BAR_DRAIN, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 5) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_rows) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
            int stage = 0;
            uint32_t phase = 0, a_iter = 0;
            uint32_t issued_mask = 0, last_parity = 0;
            bool a_issued = false;
            bool ok = true;
            for (long long u = blockIdx.x; u < sched.n_units && ok; u += gridDim.x) {
                int g, t0, t1;
                unit_coords(sched, u, g, t0, t1);
                ok = mbar_wait(bars + 8 * BAR_A_EMPTY, (a_iter & 1) ^ 1, abort_flag, status);
                if (!ok) break;
                mbar_expect_tx(bars + 8 * BAR_A_FULL, A_BYTES);
                tma_load_2d(sbase + OFF_A, &tmap_q, bars + 8 * BAR_A_FULL, 0, g * BM);
                a_issued = true;
                a_iter++;
                for (int t = t0; t < t1; t++) {
                    ok = mbar_wait(bars + 8 * (BAR_EMPTY + stage), phase ^ 1, abort_flag, status);
                    if (!ok) break;
                    mbar_expect_tx(bars + 8 * (BAR_FULL + stage), B_BYTES);
                    tma_load_2d(sbase + OFF_B + stage * B_BYTES, &tmap_rows, bars + 8 * (BAR_FULL + stage), 0,
                                t * BN);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                // Drain: every issued load completes its full barrier phase.
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s)) mbar_drain_wait(bars + 8 * (BAR_FULL + s), (last_parity >> s) & 1);
                if (a_issued) mbar_drain_wait(bars + 8 * BAR_A_FULL, (a_iter - 1) & 1);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0, a_iter = 0;
            bool ok = true, issued = false;
            for (long long u = blockIdx.x; u < sched.n_units && ok; u += gridDim.x) {
                int g, t0, t1;
                unit_coords(sched, u, g, t0, t1);
                ok = mbar_wait(bars + 8 * BAR_A_FULL, a_iter & 1, abort_flag, status);
                if (!ok) break;
                a_iter++;
                tc_fence_after();
                const uint64_t adesc = sw128_desc(sbase + OFF_A);
                for (int t = t0; t < t1; t++) {
                    ok = mbar_wait(bars + 8 * (BAR_ACC_EMPTY + acc), acc_phase ^ 1, abort_flag, status);
                    if (!ok) break;
                    ok = mbar_wait(bars + 8 * (BAR_FULL + stage), phase, abort_flag, status);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t bdesc = sw128_desc(sbase + OFF_B + stage * B_BYTES);
                    const uint32_t d = tmem_base + (uint32_t)(acc * BN);
#pragma unroll
                    for (int kk = 0; kk < BK / 32; kk++)
                        umma_i8(d, adesc + (uint64_t)((kk * 32) >> 4), bdesc + (uint64_t)((kk * 32) >> 4),
                                kk > 0 ? 1u : 0u);
                    issued = true;
                    umma_commit(bars + 8 * (BAR_EMPTY + stage));
                    umma_commit(bars + 8 * (BAR_ACC_FULL + acc));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                    if (++acc == ACC_STAGES) {
                        acc = 0;
                        acc_phase ^= 1;
                    }
                }
                if (!ok) break;
                umma_commit(bars + 8 * BAR_A_EMPTY);
            }
            if (!ok && issued) {
                umma_commit(bars + 8 * BAR_DRAIN);
                mbar_drain_wait(bars + 8 * BAR_DRAIN, 0);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 0-3)
        const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        for (long long u = blockIdx.x; u < sched.n_units && ok; u += gridDim.x) {
            int g, t0, t1;
            unit_coords(sched, u, g, t0, t1);
            const int qi = g * BM + warp * 32 + lane;
            const bool qvalid = qi < nq;
            uint32_t tkey = 0;
            int32_t tid = 0, qnv = 0;
            if (qvalid) {
                tkey = thr_key[qi];
                tid = thr_id[qi];
                qnv = qn[qi];
            }
            // Chunk passes when qn + n_min - 2m <= tkey  <=>  2m >= n_min + (qn - tkey).
            const long long bias = qvalid ? (long long)qnv - (long long)tkey : (1ll << 40);
            for (int t = t0; t < t1; t++) {
                const int64_t row0 = (int64_t)t * BN;
                // Lane l holds n_min of chunk l & 7 (first row of the chunk, rows are norm-sorted).
                const int32_t nmin_l = __ldg(norms + row0 + (lane & 7) * 32);
                ok = mbar_wait(bars + 8 * (BAR_ACC_FULL + acc), acc_phase, abort_flag, status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tcol = tmem_base + lane_base + (uint32_t)(acc * BN);
#pragma unroll 1
                for (int c = 0; c < BN / 32; c++) {
                    uint32_t v[32];
                    __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the slow path
                    tmem_ld32(tcol + (uint32_t)(c * 32), v);
                    const int32_t nmin = __shfl_sync(0xffffffffu, nmin_l, c);
                    const int32_t m = max32(v);
                    if (2ll * m + 0 >= (long long)nmin + bias) {
                        // Slow path: exact key for each of the 32 rows.
                        const int64_t rbase = row0 + c * 32;
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            const int64_t r = rbase + j;
                            if (r < n_rows) {
                                const uint32_t key = (uint32_t)(qnv + __ldg(norms + r) - 2 * (int32_t)v[j]);
                                if (key <= tkey) {
                                    const int32_t id = __ldg(ids + r);
                                    if (key < tkey || id <= tid) {
                                        const uint32_t slot = atomicAdd(counts + qi, 1u);
                                        if (slot < (uint32_t)cap) cand[(size_t)qi * cap + slot] = make_uint2(key, (uint32_t)id);
                                    }
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bars + 8 * (BAR_ACC_EMPTY + acc));
                if (++acc == ACC_STAGES) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                     : "memory");
    }
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        MDH_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        MDH_REQUIRE(q == cudaDriverEntryPointSuccess && p, MDH_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

void encode_u8_rows(CUtensorMap* map, const void* base, int64_t rows, int dpad, int box_rows) {
    MDH_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, MDH_ERR_INTERNAL, "TMA base must be 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)dpad, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)dpad};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MDH_REQUIRE(r == CUDA_SUCCESS, MDH_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

int choose_chunks(int g, int n_tiles, int ctas) {
    // Smallest chunk count that makes the unit count a multiple of the CTA
    // count (no tail round), scaled up while chunks keep >= 64 tiles.
    int a = g, b = ctas;
    while (b) {
        int t = a % b;
        a = b;
        b = t;
    }
    const int base = ctas / a;
    if (base > n_tiles) return n_tiles;
    int mult = 1;
    while ((long long)base * (mult + 1) * 64 <= n_tiles && mult < 8) mult++;
    return base * mult;
}

}  // namespace

bool tc_supported(const mdh_index* ix, const Level& lv) {
    return ix && !ix->is_f32 && ix->dpad == BK && ix->dim <= BK && lv.rows && lv.n_pad % BN == 0;
}

void make_tmap_rows(Level& lv, int dpad) {
    if (dpad != BK || !lv.rows) return;
    encode_u8_rows(&lv.tmap_rows, lv.rows, lv.n_pad, dpad, BN);
    lv.has_tmap = true;
}

void launch_filter_tc_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                            const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap,
                            int32_t* status, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    MDH_REQUIRE(dpad == BK && lv.has_tmap, MDH_ERR_INTERNAL, "tensor-core scan needs 128-byte rows and a TMA map");
    CUtensorMap tq;
    encode_u8_rows(&tq, q, nq, dpad, BM);
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    Sched s;
    s.n_qtiles = (nq + BM - 1) / BM;
    s.n_tiles = (int)(lv.n_pad / BN);
    int ctas = sms;
    s.n_chunks = choose_chunks(s.n_qtiles, s.n_tiles, ctas);
    s.n_units = (long long)s.n_qtiles * s.n_chunks;
    if (s.n_units < ctas) ctas = (int)s.n_units;
    static bool attr_set = false;
    if (!attr_set) {
        MDH_CUDA(cudaFuncSetAttribute(k_filter_tc_u8_l2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES));
        attr_set = true;
    }
    k_filter_tc_u8_l2<<<ctas, NUM_THREADS, SMEM_BYTES, st>>>(lv.tmap_rows, tq, lv.norms, lv.ids, lv.n, qn, nq, thr_key,
                                                            thr_id, counts, cand, cap, s, status);
    MDH_CUDA(cudaGetLastError());
}

}  // namespace mdh
