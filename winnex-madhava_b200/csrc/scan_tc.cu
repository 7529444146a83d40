// Tensor-core (tcgen05) u8 L2 scan on single SMs, sm_100a.
//
// Same contract as the CUDA-core filter (scan_simt.cu): for each query q and
// real row r of a Level, key = |q|^2 + |v|^2 - 2 q.v; pairs with
// (key, id) <= (thr_key[q], thr_id[q]) are appended to q's candidate list as
// {key, r}; on a dense level (infinite thresholds) row r goes to slot r.
//
// Tile: 128 queries (TMEM lanes, the MMA's M) x 256 corpus rows (the MMA's
// N) x 128 bytes (K: four kind::i8 MMAs of K = 32).  u8 x u8 products
// accumulate exactly in s32 in tensor memory.  Operands are staged by TMA
// with the 128-byte swizzle (one 128-byte row per vector = one swizzle row).
// An accumulator stage holds 256 columns; the 512 TMEM columns form two
// stages, so the MMA of tile t+1 overlaps the epilogue of tile t.  (The
// template keeps QT query tiles per stage as a parameter; only QT = 1 is
// built: with QT = 2, BN = 128 every MMA re-reads its A tile and the shared
// memory port, not the tensor pipe, set the pace.)
//
// Warp roles (576 threads, one CTA per SM, persistent):
//   warps 0-15 epilogue: warp w reads TMEM lanes 32*(w%4).. (thread = one
//              query) and the 64 columns [64*(w/4), +64) of each
//              accumulator stage; both 32-column chunks are copied to
//              registers and the stage released before the Cauchy-Schwarz
//              filter runs; passing rows are buffered per thread in shared
//              memory, one atomic per flush;
//   warp 16    TMA producer (the QT query tiles once per work unit, corpus
//              tiles through a STAGES-deep ring);
//   warp 17    TMEM allocator + single-thread MMA issuer.
//
// Epilogue filter: rows are sorted by |v|^2, so a row block's first row has
// its smallest norm n_min.  With m = max q.v over the block, every key in it
// is >= |q|^2 + n_min - 2m; when that exceeds the query's threshold the whole
// block is skipped after one max reduction (tc_ptx.cuh: max32).  The
// schedule form bounds each warp's 64 columns with the tile's first norm
// (neighbouring rows of a sorted level have nearly equal norms); the unit
// table form (IVF cells, whose tiles span a wider norm range) bounds each
// 32-row chunk with its own first norm.  Blocks that pass are expanded per
// lane: each passing lane walks its own passing columns.  In the unit table
// form the whole warp runs that walk and takes each row's norm by shuffle
// from the lane that loaded it (lane l holds rows l and 32 + l of the warp's
// columns).
//
// Work units: (query group, corpus chunk), ordered chunk-major so the CTAs
// running at the same time share corpus chunks through L2; each CTA takes
// units blockIdx.x, blockIdx.x + gridDim.x, ...  Unit tables (IVF) have
// units of unequal length; given a counter, their units are handed out at
// run time instead (feed_publish).
//
// Every mbarrier wait is bounded.  On expiry the kernel writes kDevTimeout to
// *status, raises a shared abort flag so every role leaves its loop, drains
// its own outstanding copies and MMAs with bounded waits, frees its tensor
// memory and returns.
#include <algorithm>
#include <type_traits>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "internal.h"
#include "tc_ptx.cuh"

namespace mdh {

namespace {

using namespace tc;

constexpr int BM = 128;           // queries per query tile (TMEM lanes)
constexpr int BK = 128;           // bytes per row (K)
constexpr int BOX_ROWS = 256;     // corpus rows per TMA box (BN / BOX_ROWS boxes per stage; 256 is the box limit)
constexpr int TMEM_COLS = 512;
constexpr int EPI_WARPS = 16;     // 4 per TMEM lane quarter
constexpr int COLS_PER_WARP = 64; // two 32-column chunks
constexpr int EPI_THREADS = 32 * EPI_WARPS;
constexpr int PRODUCER_WARP = EPI_WARPS;
constexpr int MMA_WARP = EPI_WARPS + 1;
constexpr int NUM_THREADS = 32 * (EPI_WARPS + 2);
constexpr int BUFN = 8;           // buffered candidates per epilogue thread
constexpr int BUF_FLUSH_AT = 4;   // a warp flushes together once a lane holds this many
constexpr uint32_t A_TILE_BYTES = BM * BK;

template <int BN_, int QT_>
struct TcCfg {
    static constexpr int BN = BN_;
    static constexpr int QT = QT_;
    static constexpr int QGROUP = QT * BM;             // queries per work unit
    static constexpr int ACC_COLS = QT * BN;           // TMEM columns per accumulator stage
    static constexpr int ACC_STAGES = TMEM_COLS / ACC_COLS;
    static constexpr int STAGES = 10 * 128 / BN;       // corpus tile ring: 160 KB
    static constexpr uint32_t A_BYTES = QT * A_TILE_BYTES;
    static constexpr uint32_t B_BYTES = BN * BK;
    static constexpr uint32_t IDESC = idesc_u8(BM, BN);
    // Shared memory map (offsets from a 1024-byte aligned base).
    // Two query-tile slots: the producer loads the next unit's queries while
    // the current unit's MMAs still read the other slot.
    static constexpr int A_SLOTS = 2;
    static constexpr uint32_t OFF_A = 0;
    static constexpr uint32_t OFF_B = OFF_A + A_SLOTS * A_BYTES;
    static constexpr uint32_t OFF_BUF = OFF_B + STAGES * B_BYTES;
    static constexpr uint32_t OFF_BAR = OFF_BUF + BUFN * EPI_THREADS * 8;
    static constexpr uint32_t BAR_FULL = 0, BAR_EMPTY = STAGES, BAR_ACC_FULL = 2 * STAGES,
                              BAR_ACC_EMPTY = 2 * STAGES + ACC_STAGES, BAR_A_FULL = 2 * STAGES + 2 * ACC_STAGES,
                              BAR_A_EMPTY = BAR_A_FULL + A_SLOTS, BAR_DRAIN = BAR_A_EMPTY + A_SLOTS,
                              BAR_UNIT_FULL = BAR_DRAIN + 1, BAR_UNIT_EMPTY = BAR_UNIT_FULL + 2,
                              NUM_BARS = BAR_UNIT_EMPTY + 2;
    static constexpr uint32_t OFF_USLOT = OFF_BAR + NUM_BARS * 8;  // two unit indices handed out at run time
    static constexpr uint32_t OFF_TMEM_SLOT = OFF_USLOT + 8;
    static constexpr uint32_t OFF_ABORT = OFF_TMEM_SLOT + 4;
    static constexpr uint32_t OFF_STATS = OFF_ABORT + 4;        // u32 block-bound counts: tests, unsettled, rows
    static constexpr uint32_t SMEM_BYTES = OFF_STATS + 12 + 1024;  // + alignment slack
    static_assert(ACC_COLS == 4 * COLS_PER_WARP && ACC_STAGES >= 2, "four 64-column parts per accumulator stage");
    static_assert(BN % BOX_ROWS == 0 && BN <= 256 && (COLS_PER_WARP % BN == 0 || BN % COLS_PER_WARP == 0),
                  "tile shape");
    static_assert(STAGES <= 32, "issued-stage mask is 32 bits");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
    static_assert(A_TILE_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzle alignment");
};

struct Sched {
    int n_groups;     // query groups of QT x BM
    int n_tiles;      // corpus tiles of BN rows
    int n_chunks;     // corpus chunks per query group
    long long n_units;
};

__device__ __forceinline__ void unit_coords(const Sched& s, long long u, int& g, int& t0, int& t1) {
    const int c = (int)(u / s.n_groups);
    g = (int)(u - (long long)c * s.n_groups);
    t0 = (int)((long long)c * s.n_tiles / s.n_chunks);
    t1 = (int)((long long)(c + 1) * s.n_tiles / s.n_chunks);
}

// A work unit: query rows [q_row, q_row + q_count) of the query matrix
// (padded to the group size with rows that are masked) against corpus tiles
// [t0, t1), rows at or past row_end masked.  Without a unit table, unit u is
// (query group, corpus chunk) from the schedule; with one (the IVF scan), it
// is units[u] and query row i belongs to query qmap[i].
struct UnitView {
    int q_row, q_count, t0, t1, row_end;
};

template <class C, bool UNITS>
__device__ __forceinline__ UnitView unit_view(const Sched& s, const ScanUnit* units, long long u, int n_rows, int nq) {
    UnitView v;
    if (UNITS) {
        const ScanUnit x = units[u];
        v.q_row = x.q_row;
        v.q_count = x.q_count;
        v.t0 = x.t0;
        v.t1 = x.t1;
        v.row_end = x.row_end;
    } else {
        int g;
        unit_coords(s, u, g, v.t0, v.t1);
        v.q_row = g * C::QGROUP;
        v.q_count = nq - v.q_row < C::QGROUP ? nq - v.q_row : C::QGROUP;
        v.row_end = n_rows;
    }
    return v;
}

// The rows [row0, row0 + 32) of one 32-column chunk against this thread's
// query: v[j] = q.v of row row0 + j.  need = n_min + |q|^2 - threshold, with
// n_min no larger than any of the rows' norms, so a row can reach the
// threshold only if 2 v[j] >= need.  Every such row goes to the candidate
// list as {q.v, row}: the exact key |q|^2 + |v|^2 - 2 q.v is formed after the
// scan (k_rekey_l2), so the epilogue reads no norm and no id.  The list is a
// superset of the rows at or under the threshold, which is all the selection
// needs.  Dense levels (every row a candidate) write row r at slot r.
// exact: overflow reruns instead form each key here (the row's norm and, on
// a tie, its id) and keep only rows at or under (tkey, tid), so every rerun's
// list holds rows under its threshold alone and the next threshold is
// strictly tighter.
template <bool EXACT, bool DENSE>
__device__ __forceinline__ void chunk_emit(const uint32_t (&v)[32], int32_t need, int32_t row0, int row_end, int qi,
                                           uint32_t tkey, int32_t tid, int32_t qnv,
                                           const int32_t* __restrict__ norms, const int32_t* __restrict__ ids,
                                           CandBuf<EPI_THREADS, BUFN>& buf, uint32_t* __restrict__ counts,
                                           uint2* __restrict__ cand, int cap) {
    if constexpr (DENSE) {
        // Every row of a dense level is a candidate at slot r: the chunk's
        // 32 entries are one 256-byte run of the list (rows start at
        // multiples of 32, the capacity is even), stored two at a time.
        const int32_t valid = row_end - row0;  // pad rows trail the level
        uint2* run = cand + (size_t)qi * cap + row0;
        uint4* run4 = reinterpret_cast<uint4*>(run);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            if (j + 1 < valid)
                run4[j >> 1] = make_uint4(v[j], (uint32_t)(row0 + j), v[j + 1], (uint32_t)(row0 + j + 1));
            else if (j < valid)
                run[j] = make_uint2(v[j], (uint32_t)(row0 + j));
        }
        return;
    }
    if (2 * max32(v) < need) return;
    uint32_t mask = pass_mask32(v, need);
    const int32_t valid = row_end - row0;  // pad rows trail the level
    if (valid < 32) mask &= valid > 0 ? (1u << valid) - 1u : 0u;
    while (mask) {
        const int j = __ffs(mask) - 1;
        mask &= mask - 1;
        const uint32_t x = pick32(v, j), r = (uint32_t)(row0 + j);
        if (EXACT) {
            const uint32_t key = (uint32_t)(qnv + __ldg(norms + r) - 2 * (int32_t)x);
            if (key < tkey || (key == tkey && __ldg(ids + r) <= tid)) buf.push(key, r, counts, cand, cap, qi);
        } else {
            buf.push(x, r, counts, cand, cap, qi);
        }
    }
}

// Candidates written by the schedule-form scan hold {q.v, row}; this turns
// each into {|q|^2 + |v|^2 - 2 q.v, row}, the exact L2 key the selection
// ranks by.  One block per query; dense_rows > 0: every one of the first
// dense_rows slots is filled (dense level), else counts[q] (capped) are.
__global__ void k_rekey_l2(const uint32_t* __restrict__ counts, uint2* __restrict__ cand, int cap,
                           const int32_t* __restrict__ norms, const int32_t* __restrict__ qn, int dense_rows) {
    const int q = blockIdx.x;
    const uint32_t c_all = dense_rows > 0 ? (uint32_t)dense_rows : counts[q];
    const int c = (int)(c_all < (uint32_t)cap ? c_all : (uint32_t)cap);
    const int32_t qv = qn[q];
    uint2* list = cand + (size_t)q * cap;
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
        uint2 e = list[i];
        e.x = (uint32_t)(qv + __ldg(norms + e.y) - 2 * (int32_t)e.x);
        list[i] = e;
    }
}

// Keys of a deferred unit scan's entries (see ChunkOut), eight lanes per
// entry: lane s of the group reads 16 bytes of the entry's dot products (rows
// 4s .. 4s+3) and the same rows' norms, so each group's loads are two
// coalesced 128-byte runs (entries and chunks start at multiples of 128
// bytes).  A lane marks its rows with (key, id) <= the query's threshold --
// the epilogue's exact test, ids read only on a key tie -- the group ORs the
// lane masks, its first lane takes the list's slots with one atomic on the
// query's count, and every lane writes its own rows.  The keys and ids are
// those of the EXACT epilogue, so a list gets the same rows in another
// order.  Headers are bounds-checked, and nothing runs after a scan that did
// not finish.
__global__ void __launch_bounds__(256) k_rekey_chunks(ChunkOut out, const int32_t* __restrict__ norms,
                                                      const int32_t* __restrict__ ids, int32_t n_rows_pad,
                                                      const int32_t* __restrict__ qn, int nq,
                                                      const uint32_t* __restrict__ thr_key,
                                                      const int32_t* __restrict__ thr_id,
                                                      uint32_t* __restrict__ counts, uint2* __restrict__ cand, int cap,
                                                      const int32_t* __restrict__ status) {
    if (*reinterpret_cast<const volatile int32_t*>(status) != kDevOk) return;
    const uint32_t n = min(*out.counter, out.capacity);
    const int lane = threadIdx.x & 31, sub = lane & 7, lead = lane & 24;
    const unsigned group = 0xffu << lead;  // the entry's eight lanes
    const int r0 = 4 * sub;                 // this lane's first row in the chunk
    const uint32_t stride = gridDim.x * (blockDim.x / 8);
    for (uint32_t e = (blockIdx.x * blockDim.x + threadIdx.x) / 8; e < n; e += stride) {
        const int4 h = out.hdr[e];
        const int qi = h.x, row0 = h.y, valid = h.z;
        if (qi < 0 || qi >= nq || valid <= 0 || valid > 32 || row0 < 0 || row0 > n_rows_pad - 32 || (row0 & 31))
            continue;
        const int32_t qv = __ldg(qn + qi);
        const uint32_t tk = __ldg(thr_key + qi);
        const uint4 x = out.x[(size_t)e * 8 + sub];
        const int4 nv = __ldg(reinterpret_cast<const int4*>(norms + row0) + sub);
        const uint32_t key[4] = {(uint32_t)(qv + nv.x - 2 * (int32_t)x.x), (uint32_t)(qv + nv.y - 2 * (int32_t)x.y),
                                 (uint32_t)(qv + nv.z - 2 * (int32_t)x.z), (uint32_t)(qv + nv.w - 2 * (int32_t)x.w)};
        uint32_t mine = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            // Rows tied with the threshold key stay only up to its id.
            const bool keep = r0 + j < valid &&
                              (key[j] < tk || (key[j] == tk && __ldg(ids + row0 + r0 + j) <= __ldg(thr_id + qi)));
            mine |= (uint32_t)keep << j;
        }
        uint32_t mask = mine << r0;
        mask |= __shfl_xor_sync(group, mask, 1);
        mask |= __shfl_xor_sync(group, mask, 2);
        mask |= __shfl_xor_sync(group, mask, 4);
        if (mask == 0u) continue;
        uint32_t at = 0;
        if (sub == 0) at = atomicAdd(counts + qi, (uint32_t)__popc(mask));
        at = __shfl_sync(group, at, lead) + (uint32_t)__popc(mask & ((1u << r0) - 1u));
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (!(mine >> j & 1u)) continue;
            if (at < (uint32_t)cap) cand[(size_t)qi * cap + at] = make_uint2(key[j], (uint32_t)(row0 + r0 + j));
            at++;
        }
    }
}

// Block-bound counts live in shared memory (three u32: tests, unsettled
// blocks, real rows of those blocks) and are added on the rare unsettled path
// only, so the common path keeps no counter in registers; the CTA adds them to
// the global u64 counters once, at exit.
__device__ __forceinline__ void stat_add(uint32_t* s, uint32_t v) { atomicAdd(s, v); }

// Deferred unit scans: a warp's next 64-entry block of chunk_out (warp-wide
// call), or kNoChunkBlock past the capacity, which flags the overflow.
constexpr uint32_t kNoChunkBlock = 0xffffffffu;
__device__ __forceinline__ uint32_t chunk_block_take(const ChunkOut& out, int32_t* status, int lane) {
    uint32_t base = 0;
    if (lane == 0) base = atomicAdd(out.counter, (uint32_t)kChunkBlock);
    base = __shfl_sync(0xffffffffu, base, 0);
    if (base > out.capacity - kChunkBlock) {
        if (lane == 0) atomicExch(status + kStatusChunkOverflow, 1);
        return kNoChunkBlock;
    }
    return base;
}

// Entry `idx` (< 128) of the warp's current block, continuing into the next
// one: a lane's 32 dot products of one chunk and its header.
__device__ __forceinline__ void chunk_put(const ChunkOut& out, uint32_t cur, uint32_t nxt, int idx,
                                          const uint32_t (&v)[32], int qi, int32_t row0, int32_t valid) {
    const uint32_t base = idx < kChunkBlock ? cur : nxt;
    if (base == kNoChunkBlock) return;
    const uint32_t slot = base + (uint32_t)(idx & (kChunkBlock - 1));
    uint4* dst = out.x + (size_t)slot * 8;
#pragma unroll
    for (int i = 0; i < 8; i++) dst[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    out.hdr[slot] = make_int4(qi, row0, valid, 0);
}

// Marks the unused entries [used, 64) of a warp's block (query -1) so that
// the re-key pass skips them.
__device__ __forceinline__ void chunk_block_close(const ChunkOut& out, uint32_t base, int used, int lane) {
    if (base == kNoChunkBlock) return;
    for (int j = used + lane; j < kChunkBlock; j += 32) out.hdr[base + j] = make_int4(-1, 0, 0, 0);
}

// Run-time hand-out of a unit table (its units differ in length, so fixed
// shares leave some SMs idle at the end).  The producer takes the next index
// from a global counter and publishes it in one of two shared-memory slots
// (UNIT_FULL); the MMA issuer and the 16 epilogue warps read it and release
// the slot (UNIT_EMPTY, 17 arrivals).  An index past the table ends the CTA's
// work.  Both return 1 with a unit, 0 when there are no more, -1 on abort.
__device__ __forceinline__ int feed_publish(int32_t* counter, long long n_units, volatile int32_t* slots,
                                            uint32_t bar_full, uint32_t bar_empty, int& s, uint32_t& ph,
                                            long long& u, volatile int32_t* abort_flag, int32_t* status) {
    if (!mbar_wait<false>(bar_empty + 8 * s, ph ^ 1, abort_flag, status)) return -1;
    const int got = atomicAdd(counter, 1);
    u = got < n_units ? got : -1;
    slots[s] = (int32_t)u;
    mbar_arrive(bar_full + 8 * s);  // release: the slot is visible to the readers
    if (++s == 2) {
        s = 0;
        ph ^= 1;
    }
    return u >= 0 ? 1 : 0;
}
// whole_warp: every lane of an epilogue warp calls it; else the single
// MMA-issuing thread.
__device__ __forceinline__ int feed_take(bool whole_warp, volatile int32_t* slots, uint32_t bar_full,
                                         uint32_t bar_empty, int& s, uint32_t& ph, long long& u,
                                         volatile int32_t* abort_flag, int32_t* status) {
    if (!mbar_wait_inl<false>(bar_full + 8 * s, ph, abort_flag, status)) return -1;
    u = slots[s];
    if (whole_warp) __syncwarp();
    if (!whole_warp || (threadIdx.x & 31) == 0) mbar_arrive(bar_empty + 8 * s);
    if (++s == 2) {
        s = 0;
        ph ^= 1;
    }
    return u >= 0 ? 1 : 0;
}

// UNITS: the unit-table form.  Its query rows are different queries probing
// one cell, whose passing columns rarely coincide.  With EXACT its slow path
// walks each lane's own columns (the row norm comes by shuffle); without it
// a lane whose chunk passes writes the chunk's 32 dot products to chunk_out
// and k_rekey_chunks forms the keys after the scan.  The schedule form walks
// the columns any lane keeps, warp-uniformly, with the norms already in
// registers.
template <class C, bool UNITS, bool EXACT, bool DENSE = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_filter_tc_u8_l2(const __grid_constant__ CUtensorMap tmap_rows, const __grid_constant__ CUtensorMap tmap_q,
                      const int32_t* __restrict__ norms, const int32_t* __restrict__ ids, int32_t n_rows,
                      const int32_t* __restrict__ qn, int nq, const uint32_t* __restrict__ thr_key,
                      const int32_t* __restrict__ thr_id, uint32_t* __restrict__ counts, uint2* __restrict__ cand,
                      int cap, int dense, Sched sched, int32_t* __restrict__ status,
                      const ScanUnit* __restrict__ units, const int32_t* __restrict__ qmap,
                      const int32_t* __restrict__ n_units_dev, int32_t* __restrict__ unit_counter,
                      unsigned long long* __restrict__ block_stats, ChunkOut chunk_out) {
    constexpr int BN = C::BN, QT = C::QT, STAGES = C::STAGES, ACC_STAGES = C::ACC_STAGES;
    // A unit table built on the device carries its own length.
    const long long n_units = n_units_dev ? (long long)*n_units_dev : sched.n_units;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bars = sbase + C::OFF_BAR;
    volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + C::OFF_ABORT);
    uint32_t* stats = reinterpret_cast<uint32_t*>(smem + C::OFF_STATS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEM_SLOT);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(bars + 8 * (C::BAR_FULL + s), 1);
            mbar_init(bars + 8 * (C::BAR_EMPTY + s), 1);
        }
        for (int s = 0; s < ACC_STAGES; s++) {
            mbar_init(bars + 8 * (C::BAR_ACC_FULL + s), 1);
            mbar_init(bars + 8 * (C::BAR_ACC_EMPTY + s), EPI_WARPS);
        }
        for (int s = 0; s < C::A_SLOTS; s++) {
            mbar_init(bars + 8 * (C::BAR_A_FULL + s), 1);
            mbar_init(bars + 8 * (C::BAR_A_EMPTY + s), 1);
        }
        mbar_init(bars + 8 * C::BAR_DRAIN, 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(bars + 8 * (C::BAR_UNIT_FULL + s), 1);
            mbar_init(bars + 8 * (C::BAR_UNIT_EMPTY + s), EPI_WARPS + 1);
        }
        *abort_flag = 0;
        stats[0] = stats[1] = stats[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == MMA_WARP) tmem_alloc<1>(smem_u32(tmem_slot), TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Unit hand-out (unit tables with a counter only); see feed_publish.
    const bool dyn = UNITS && unit_counter != nullptr;
    volatile int32_t* uslots = reinterpret_cast<volatile int32_t*>(smem + C::OFF_USLOT);
    const uint32_t ubar_full = bars + 8 * C::BAR_UNIT_FULL, ubar_empty = bars + 8 * C::BAR_UNIT_EMPTY;
    int us = 0;
    uint32_t uph = 0;

    if (warp == PRODUCER_WARP) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_rows) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_q) : "memory");
            int stage = 0;
            uint32_t phase = 0, a_iter = 0;
            uint32_t issued_mask = 0, last_parity = 0;
            bool ok = true;
            for (long long u = blockIdx.x;; u += gridDim.x) {
                if (!ok) break;
                if (dyn) {
                    const int r = feed_publish(unit_counter, n_units, uslots, ubar_full, ubar_empty, us, uph, u, abort_flag, status);
                    if (r < 0) ok = false;
                    if (r <= 0) break;
                } else if (u >= n_units) {
                    break;
                }
                const UnitView uv = unit_view<C, UNITS>(sched, units, u, n_rows, nq);
                const int t0 = uv.t0, t1 = uv.t1;
                // Query slot a_iter % 2, its (a_iter / 2)-th use.
                const int as = (int)(a_iter & 1);
                ok = mbar_wait<false>(bars + 8 * (C::BAR_A_EMPTY + as), ((a_iter >> 1) & 1) ^ 1, abort_flag, status);
                if (!ok) break;
                mbar_expect_tx(bars + 8 * (C::BAR_A_FULL + as), C::A_BYTES);
#pragma unroll
                for (int qt = 0; qt < QT; qt++)
                    tma_load_2d(sbase + C::OFF_A + as * C::A_BYTES + qt * A_TILE_BYTES, &tmap_q,
                                bars + 8 * (C::BAR_A_FULL + as), 0, uv.q_row + qt * BM);
                a_iter++;
                for (int t = t0; t < t1; t++) {
                    ok = mbar_wait<false>(bars + 8 * (C::BAR_EMPTY + stage), phase ^ 1, abort_flag, status);
                    if (!ok) break;
                    mbar_expect_tx(bars + 8 * (C::BAR_FULL + stage), C::B_BYTES);
#pragma unroll
                    for (int b = 0; b < BN / BOX_ROWS; b++)
                        tma_load_2d(sbase + C::OFF_B + stage * C::B_BYTES + b * BOX_ROWS * BK, &tmap_rows,
                                    bars + 8 * (C::BAR_FULL + stage), 0, t * BN + b * BOX_ROWS);
                    issued_mask |= 1u << stage;
                    last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            if (!ok) {
                // Drain: every issued copy completes its barrier phase.
                for (int s = 0; s < STAGES; s++)
                    if (issued_mask & (1u << s))
                        mbar_drain_wait<false>(bars + 8 * (C::BAR_FULL + s), (last_parity >> s) & 1);
                // The last load of each query slot (use a_iter - 1 and a_iter - 2).
                for (uint32_t i = a_iter > 2 ? a_iter - 2 : 0; i < a_iter; i++)
                    mbar_drain_wait<false>(bars + 8 * (C::BAR_A_FULL + (i & 1)), (i >> 1) & 1);
            }
        }
    } else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        // tcgen05.mma issue blocks while the tensor pipe is busy and the pipe
        // queues little more than one MMA, so a wait between tiles leaves the
        // pipe idle.  The barriers of tile t+1 are therefore probed between
        // tile t's MMAs (test_wait does not block) and, when both are already
        // complete, tile t+1 is issued without waiting.
        if (lane == 0) {
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0, a_iter = 0;
            bool ok = true, issued = false;
            for (long long u = blockIdx.x;; u += gridDim.x) {
                if (!ok) break;
                if (dyn) {
                    const int r = feed_take(false, uslots, ubar_full, ubar_empty, us, uph, u, abort_flag, status);
                    if (r < 0) ok = false;
                    if (r <= 0) break;
                } else if (u >= n_units) {
                    break;
                }
                const UnitView uv = unit_view<C, UNITS>(sched, units, u, n_rows, nq);
                const int t0 = uv.t0, t1 = uv.t1;
                const int as = (int)(a_iter & 1);
                ok = mbar_wait<false>(bars + 8 * (C::BAR_A_FULL + as), (a_iter >> 1) & 1, abort_flag, status);
                if (!ok) break;
                a_iter++;
                tc_fence_after();
                bool ready = false;  // tile t's barriers were seen complete while issuing tile t-1
                for (int t = t0; t < t1; t++) {
                    if (!ready) {
                        ok = mbar_wait_inl<false>(bars + 8 * (C::BAR_ACC_EMPTY + acc), acc_phase ^ 1, abort_flag,
                                                  status);
                        if (!ok) break;
                        ok = mbar_wait_inl<false>(bars + 8 * (C::BAR_FULL + stage), phase, abort_flag, status);
                        if (!ok) break;
                    }
                    tc_fence_after();
                    const int nstage = stage + 1 == STAGES ? 0 : stage + 1;
                    const uint32_t nphase = stage + 1 == STAGES ? phase ^ 1 : phase;
                    const int nacc = acc + 1 == ACC_STAGES ? 0 : acc + 1;
                    const uint32_t nacc_phase = acc + 1 == ACC_STAGES ? acc_phase ^ 1 : acc_phase;
                    const bool more = t + 1 < t1;
                    bool pe = false, pf = false;
                    const uint64_t bdesc = sw128_desc(sbase + C::OFF_B + stage * C::B_BYTES);
#pragma unroll
                    for (int qt = 0; qt < QT; qt++) {
                        const uint64_t adesc = sw128_desc(sbase + C::OFF_A + as * C::A_BYTES + qt * A_TILE_BYTES);
                        const uint32_t d = tmem_base + (uint32_t)(acc * C::ACC_COLS + qt * BN);
#pragma unroll
                        for (int kk = 0; kk < BK / 32; kk++) {
                            umma_i8<1>(d, adesc + (uint64_t)((kk * 32) >> 4), bdesc + (uint64_t)((kk * 32) >> 4),
                                       C::IDESC, kk > 0 ? 1u : 0u);
                            if (more && qt == QT - 1 && kk == 1)
                                pe = mbar_test_wait(bars + 8 * (C::BAR_ACC_EMPTY + nacc), nacc_phase ^ 1);
                            if (more && qt == QT - 1 && kk == 2)
                                pf = mbar_test_wait(bars + 8 * (C::BAR_FULL + nstage), nphase);
                        }
                    }
                    issued = true;
                    umma_commit(bars + 8 * (C::BAR_EMPTY + stage));
                    umma_commit(bars + 8 * (C::BAR_ACC_FULL + acc));
                    ready = pe && pf;
                    stage = nstage;
                    phase = nphase;
                    acc = nacc;
                    acc_phase = nacc_phase;
                }
                if (!ok) break;
                umma_commit(bars + 8 * (C::BAR_A_EMPTY + as));
            }
            if (!ok && issued) {
                umma_commit(bars + 8 * C::BAR_DRAIN);
                mbar_drain_wait<false>(bars + 8 * C::BAR_DRAIN, 0);
            }
        }
    } else if constexpr (!UNITS && QT == 1 && ACC_STAGES == 2) {
        // ------------------------------------------------------------ epilogue (warps 0-15), schedule form
        // Warp w reads TMEM lanes 32*(w%4) (thread = one query) and the 64
        // columns [64*(w/4), +64) of each accumulator stage.  One bound per
        // tile: n_min is the norm of the tile's first row (rows are sorted by
        // norm), and one max reduction covers the warp's 64 columns.  The tile
        // loop is unrolled over the two accumulator stages so each stage's
        // barrier and TMEM address are constants.  This keeps the epilogue's
        // ALU work -- which competes with the MMA issuer for the issue slots
        // of its sub-partition -- near the reduction itself.
        const int quarter = warp & 3, part = warp >> 2;
        const int rowoff = part * COLS_PER_WARP;
        const uint32_t tcol0 = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)rowoff;
        CandBuf<EPI_THREADS, BUFN> buf;
        buf.base = reinterpret_cast<uint2*>(smem + C::OFF_BUF) + threadIdx.x;
        buf.n = 0;
        int acc = 0;  // accumulator stage of the CTA's next tile
        uint32_t ph0 = 0, ph1 = 0;
        bool ok = true;
        for (long long u = blockIdx.x;; u += gridDim.x) {
            if (!ok) break;
            if (dyn) {
                const int r = feed_take(true, uslots, ubar_full, ubar_empty, us, uph, u, abort_flag, status);
                if (r < 0) ok = false;
                if (r <= 0) break;
            } else if (u >= n_units) {
                break;
            }
            const UnitView uv = unit_view<C, UNITS>(sched, units, u, n_rows, nq);
            const int t0 = uv.t0, t1 = uv.t1, row_end = uv.row_end;
            const int qlocal = quarter * 32 + lane;
            const bool qvalid = qlocal < uv.q_count;
            const int qi = qvalid ? uv.q_row + qlocal : 0;
            uint32_t tkey = 0;
            int32_t tid = 0, qnv = 0;
            if (qvalid) {
                tkey = thr_key[qi];
                tid = thr_id[qi];
                qnv = qn[qi];
            }
            // A row passes when qn + n - 2v <= tkey; with n >= n_min,
            // 2v >= n_min + bias (bias = qn - tkey) is necessary.  Keys of real
            // rows are below 2^30: an infinite threshold maps to a bias that
            // always passes, an invalid query to one that never does (and
            // keeps n_min + bias below 2^31 for pad rows of norm 2^30).
            int32_t bias;
            if (!qvalid)
                bias = 1 << 29;
            else if (tkey >= (1u << 30))
                bias = -(1 << 30);
            else
                bias = qnv - (int32_t)tkey;
            int32_t nm = t0 < t1 ? __ldg(norms + (int64_t)t0 * BN) : 0;  // n_min of the next tile
            auto tile = [&](int t, auto stage_c, uint32_t ph) -> bool {
                constexpr int A = decltype(stage_c)::value;
                const int32_t need = nm + bias;
                nm = __ldg(norms + (int64_t)min(t + 1, t1 - 1) * BN);
                if (!mbar_wait_inl<false>(bars + 8 * (C::BAR_ACC_FULL + A), ph, abort_flag, status)) return false;
                tc_fence_after();
                uint32_t v[2][32];
                __syncwarp();
                tmem_ld64(tcol0 + A * C::ACC_COLS, v[0], v[1]);  // one load and one wait for both chunks
                // The chunks are in registers: hand the accumulator back to the MMA.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bars + 8 * (C::BAR_ACC_EMPTY + A));
                const int32_t m = (int32_t)__float_as_uint(
                    fmaxf(__uint_as_float((uint32_t)max32(v[0])), __uint_as_float((uint32_t)max32(v[1]))));
                const bool pass = 2 * m >= need;
                // One vote settles the tile for the whole warp (the usual case);
                // the buffer can only have grown when some lane passed.
                if (!__any_sync(0xffffffffu, pass)) return true;
                if (pass) {
                    const int32_t row0 = t * BN + rowoff;  // rows < 2^31 (ids are int32)
                    if (block_stats) {
                        stat_add(stats + 1, 1u);
                        stat_add(stats + 2, (uint32_t)min(max(row_end - row0, 0), COLS_PER_WARP));
                    }
                    chunk_emit<EXACT, DENSE>(v[0], need, row0, row_end, qi, tkey, tid, qnv, norms, ids, buf,
                                      counts, cand, cap);
                    chunk_emit<EXACT, DENSE>(v[1], need, row0 + 32, row_end, qi, tkey, tid, qnv, norms, ids, buf,
                                      counts, cand, cap);
                }
                buf.warp_flush_at(BUF_FLUSH_AT, counts, cand, cap, qi);
                return true;
            };
            using S0 = std::integral_constant<int, 0>;
            using S1 = std::integral_constant<int, 1>;
            int t = t0;
            if (acc == 1 && t < t1) {
                ok = tile(t, S1{}, ph1);
                ph1 ^= 1;
                acc = 0;
                t++;
            }
            for (; ok && t + 1 < t1; t += 2) {
                ok = tile(t, S0{}, ph0);
                ph0 ^= 1;
                if (!ok) break;
                ok = tile(t + 1, S1{}, ph1);
                ph1 ^= 1;
            }
            if (ok && t < t1) {
                ok = tile(t, S0{}, ph0);
                ph0 ^= 1;
                acc = 1;
            }
            if (qvalid) buf.flush(counts, cand, cap, qi);
        }
    } else {
        // ------------------------------------------------------------ epilogue (warps 0-15), unit tables
        const int quarter = warp & 3, part = warp >> 2;
        const int qt = part * COLS_PER_WARP / BN;              // query tile of this warp's columns
        const int rowoff = part * COLS_PER_WARP - qt * BN;     // their first row within a corpus tile
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        CandBuf<EPI_THREADS, BUFN> buf;
        buf.base = reinterpret_cast<uint2*>(smem + C::OFF_BUF) + threadIdx.x;
        buf.n = 0;
        // Deferred form: this warp's current block of chunk_out entries and
        // the next one, taken ahead so that a tile's entries always fit (a
        // tile makes at most 64) and no atomic is waited on while the
        // accumulator values are live.
        uint32_t blk_cur = 0, blk_nxt = 0;
        int blk_used = 0;
        if constexpr (!EXACT) {
            blk_cur = chunk_block_take(chunk_out, status, lane);
            blk_nxt = chunk_block_take(chunk_out, status, lane);
        }
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;
        const int32_t* nrm = norms + rowoff;
        for (long long u = blockIdx.x;; u += gridDim.x) {
            if (!ok) break;
            if (dyn) {
                const int r = feed_take(true, uslots, ubar_full, ubar_empty, us, uph, u, abort_flag, status);
                if (r < 0) ok = false;
                if (r <= 0) break;
            } else if (u >= n_units) {
                break;
            }
            const UnitView uv = unit_view<C, UNITS>(sched, units, u, n_rows, nq);
            const int t0 = uv.t0, t1 = uv.t1, row_end = uv.row_end;
            const int qlocal = qt * BM + quarter * 32 + lane;
            const bool qvalid = qlocal < uv.q_count;
            const int qi = qvalid ? (qmap ? qmap[uv.q_row + qlocal] : uv.q_row + qlocal) : 0;
            uint32_t tkey = 0;
            int32_t tid = 0, qnv = 0;
            if (qvalid) {
                tkey = thr_key[qi];
                tid = thr_id[qi];
                qnv = qn[qi];
            }
            // A row passes when qn + n - 2v <= tkey; with n >= n_min,
            // 2v >= n_min + bias (bias = qn - tkey) is necessary.  Keys of real
            // rows are below 2^30: an infinite threshold maps to a bias that
            // always passes, an invalid query to one that never does (and
            // keeps n_min + bias below 2^31 for pad rows of norm 2^30).
            int32_t bias;
            if (!qvalid)
                bias = 1 << 29;
            else if (tkey >= (1u << 30))
                bias = -(1 << 30);
            else
                bias = qnv - (int32_t)tkey;
            // Lane l holds the norms of rows l and 32 + l of this warp's two
            // chunks, loaded (coalesced) one tile ahead of their use; a chunk's
            // n_min is its lane-0 value.
            int32_t nx0 = 0, nx1 = 0;
            if (t0 < t1) {
                nx0 = __ldg(nrm + (int64_t)t0 * BN + lane);
                nx1 = __ldg(nrm + (int64_t)t0 * BN + 32 + lane);
            }
            for (int t = t0; t < t1; t++) {
                if constexpr (EXACT) buf.warp_flush_at(BUF_FLUSH_AT, counts, cand, cap, qi);
                const int32_t nr0 = nx0, nr1 = nx1;
                const int32_t need0 = __shfl_sync(0xffffffffu, nr0, 0) + bias;
                const int32_t need1 = __shfl_sync(0xffffffffu, nr1, 0) + bias;
                if (t + 1 < t1) {
                    nx0 = __ldg(nrm + (int64_t)(t + 1) * BN + lane);
                    nx1 = __ldg(nrm + (int64_t)(t + 1) * BN + 32 + lane);
                }
                ok = mbar_wait_inl<false>(bars + 8 * (C::BAR_ACC_FULL + acc), acc_phase, abort_flag, status);
                if (!ok) break;
                tc_fence_after();
                const uint32_t tcol = tmem_base + lane_base + (uint32_t)(acc * C::ACC_COLS + part * COLS_PER_WARP);
                uint32_t v[2][32];
                __syncwarp();
                tmem_ld32_issue(tcol, v[0]);
                tmem_ld32_issue(tcol + 32, v[1]);
                tmem_ld_wait(v[0]);  // waits for both loads
                tmem_ld_wait(v[1]);
                // The chunks are in registers: hand the accumulator back to the MMA.
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bars + 8 * (C::BAR_ACC_EMPTY + acc));
                if (++acc == ACC_STAGES) {
                    acc = 0;
                    acc_phase ^= 1;
                }
                const int32_t m0 = max32(v[0]), m1 = max32(v[1]);
                if constexpr (!EXACT) {
                    // Chunks wholly past the cell's last row hold pad rows only.
                    const int32_t row0 = t * BN + rowoff;  // rows < 2^31 (ids are int32)
                    const int32_t valid0 = row_end - row0, valid1 = valid0 - 32;
                    const bool pass0 = 2 * m0 >= need0 && valid0 > 0, pass1 = 2 * m1 >= need1 && valid1 > 0;
                    const uint32_t b0 = __ballot_sync(0xffffffffu, pass0), b1 = __ballot_sync(0xffffffffu, pass1);
                    if ((b0 | b1) == 0u) continue;
                    const int n0 = __popc(b0), n = n0 + __popc(b1);
                    if (block_stats && lane == 0) {
                        stat_add(stats + 1, (uint32_t)n);
                        stat_add(stats + 2, (uint32_t)(n0 * min(valid0, 32) + (n - n0) * min(max(valid1, 0), 32)));
                    }
                    const uint32_t lt = (1u << lane) - 1u;
                    if (pass0)
                        chunk_put(chunk_out, blk_cur, blk_nxt, blk_used + __popc(b0 & lt), v[0], qi, row0,
                                  min(valid0, 32));
                    if (pass1)
                        chunk_put(chunk_out, blk_cur, blk_nxt, blk_used + n0 + __popc(b1 & lt), v[1], qi, row0 + 32,
                                  min(valid1, 32));
                    blk_used += n;
                    if (blk_used >= kChunkBlock) {
                        blk_used -= kChunkBlock;
                        blk_cur = blk_nxt;
                        blk_nxt = chunk_block_take(chunk_out, status, lane);
                    }
                    continue;
                }
                const bool pass0 = 2 * m0 >= need0, pass1 = 2 * m1 >= need1;
                if (!__any_sync(0xffffffffu, pass0 || pass1)) continue;
                // The queries of a unit probe one cell but rarely keep the same
                // columns: each passing lane walks its own columns.  The whole
                // warp runs the walk (as many steps as the busiest lane needs),
                // so a column's norm comes by shuffle from the lane that holds
                // it (nr0 / nr1) instead of a dependent load per column.
                const int32_t row0 = t * BN + rowoff;  // rows < 2^31 (ids are int32)
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    uint32_t mask = (c ? pass1 : pass0) ? pass_mask32(v[c], c ? need1 : need0) : 0u;
                    const int32_t valid = row_end - (row0 + 32 * c);  // pad rows trail the cell
                    if (block_stats && (c ? pass1 : pass0)) {
                        stat_add(stats + 1, 1u);
                        stat_add(stats + 2, (uint32_t)min(max(valid, 0), 32));
                    }
                    if (valid < 32) mask &= valid > 0 ? (1u << valid) - 1u : 0u;
                    const int32_t nrc = c ? nr1 : nr0;
                    while (__any_sync(0xffffffffu, mask != 0u)) {
                        const bool have = mask != 0u;
                        const int j = have ? __ffs(mask) - 1 : 0;
                        mask &= mask - 1u;
                        const int32_t nj = __shfl_sync(0xffffffffu, nrc, j);
                        if (!have) continue;
                        const int32_t r = row0 + 32 * c + j;
                        const uint32_t key = (uint32_t)(qnv + nj - 2 * (int32_t)pick32(v[c], j));
                        if (key < tkey || (key == tkey && __ldg(ids + r) <= tid))
                            buf.push(key, (uint32_t)r, counts, cand, cap, qi);
                    }
                }
            }
            if constexpr (EXACT) {
                if (qvalid) buf.flush(counts, cand, cap, qi);
            }
            // Two chunk tests per tile for each of the unit's queries.
            if (block_stats && qvalid) stat_add(stats, 2u * (uint32_t)(t1 - t0));
        }
        if constexpr (!EXACT) {
            chunk_block_close(chunk_out, blk_cur, blk_used, lane);
            chunk_block_close(chunk_out, blk_nxt, 0, lane);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc<1>(tmem_base, TMEM_COLS);
    }
    if (block_stats && threadIdx.x == 0)
        for (int i = 0; i < 3; i++)
            if (stats[i]) atomicAdd(block_stats + i, (unsigned long long)stats[i]);
}

using CfgNarrow = TcCfg<256, 1>;  // 128 queries per CTA

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

// The scans' bounded wait (mbar_wait) on a barrier nothing arrives on: it
// gives up after `budget` cycles, raises the abort flag and records
// kDevTimeout in status[0]; status[1] = 1 if the wait returned "ready".
__global__ void k_wait_timeout_probe(long long budget, int32_t* __restrict__ status) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int32_t abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool ok = mbar_wait<false>(smem_u32(&bar), 0, &abort_flag, status, budget);
        status[1] = ok ? 1 : 0;
    }
}

}  // namespace

void launch_wait_timeout_probe(long long budget, int32_t* status, cudaStream_t st) {
    k_wait_timeout_probe<<<1, 32, 0, st>>>(budget, status);
    MDH_CUDA(cudaGetLastError());
}

void encode_tmap_2d_sw128(CUtensorMap* map, int bf16, const void* base, uint64_t inner, uint64_t rows,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows) {
    MDH_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, MDH_ERR_INTERNAL, "TMA base must be 16-byte aligned");
    MDH_REQUIRE(row_stride_bytes % 16 == 0, MDH_ERR_INTERNAL, "TMA row stride must be a multiple of 16 bytes");
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_stride_bytes};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode()(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MDH_REQUIRE(r == CUDA_SUCCESS, MDH_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

void encode_u8_rows_tmap(CUtensorMap* map, const void* base, int64_t rows, int dpad, int box_rows) {
    MDH_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, MDH_ERR_INTERNAL, "TMA base must be 16-byte aligned");
    MDH_REQUIRE(dpad == BK, MDH_ERR_INTERNAL, "tensor-core rows are 128 bytes");
    cuuint64_t dims[2] = {(cuuint64_t)dpad, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)dpad};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode()(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MDH_REQUIRE(r == CUDA_SUCCESS, MDH_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
}

int choose_scan_chunks(int groups, int n_tiles, int workers, int min_unit_tiles) {
    // A large level: the smallest chunk count that makes the unit count
    // (groups x chunks) a multiple of the worker count (no tail round),
    // scaled up while chunks keep >= 64 tiles (neighbouring units share
    // chunks through L2), as long as units keep at least min_unit_tiles.
    int a = groups, b = workers;
    while (b) {
        int t = a % b;
        a = b;
        b = t;
    }
    const int base = workers / a;
    if (base <= std::max(1, n_tiles / std::max(1, min_unit_tiles))) {
        int mult = 1;
        while ((long long)base * (mult + 1) * 64 <= n_tiles && mult < 8) mult++;
        return base * mult;
    }
    // A small level (the sample levels): the chunk count with the shortest
    // last-finishing worker, rounds x (tiles per unit + a unit's fixed cost
    // of ~4 tiles), over units of at least 4 tiles.  Their tiles carry more
    // epilogue work than the full level's, so filling the SMs pays more than
    // long units.
    constexpr double kUnitCostTiles = 4.0;
    int best = 1;
    double best_cost = 1e300;
    for (int c = 1; c <= std::max(1, n_tiles / 4); c++) {
        const long long units = (long long)groups * c;
        const long long rounds = (units + workers - 1) / workers;
        const double cost = (double)rounds * ((double)n_tiles / c + kUnitCostTiles);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = c;
        }
    }
    return best;
}

bool tc_supported(const mdh_index* ix, const Level& lv) {
    return ix && !ix->is_f32 && ix->dpad == BK && ix->dim <= BK && lv.rows && lv.norms &&
           lv.n_pad % CfgNarrow::BN == 0 && lv.n_pad < (int64_t(1) << 31);
}

void make_tmap_rows(Level& lv, int dpad) {
    if (dpad != BK || !lv.rows) return;
    encode_u8_rows_tmap(&lv.tmap_rows, lv.rows, lv.n_pad, dpad, BOX_ROWS);
    lv.has_tmap = true;
}

template <class C>
void launch_tc(const Level& lv, const CUtensorMap& tq, const int32_t* qn, int nq, const uint32_t* thr_key,
               const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap, int dense, int32_t* status,
               unsigned long long* block_stats, int exact, cudaStream_t st) {
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    const int sms = device_sm_count(dev);
    Sched s;
    s.n_groups = (nq + C::QGROUP - 1) / C::QGROUP;
    s.n_tiles = (int)(lv.n_pad / C::BN);
    int ctas = sms;
    s.n_chunks = choose_scan_chunks(s.n_groups, s.n_tiles, ctas, 64);
    s.n_units = (long long)s.n_groups * s.n_chunks;
    if (s.n_units < ctas) ctas = (int)s.n_units;
    // A function attribute belongs to the current device: set it on every launch.
    // Dense levels (the first, with infinite thresholds) have their own
    // instantiation, so the others carry no dense store path.
    auto kern = dense   ? k_filter_tc_u8_l2<C, false, false, true>
                : exact ? k_filter_tc_u8_l2<C, false, true>
                        : k_filter_tc_u8_l2<C, false, false>;
    MDH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM_BYTES));
    kern<<<ctas, NUM_THREADS, C::SMEM_BYTES, st>>>(lv.tmap_rows, tq, lv.norms, lv.ids, (int32_t)lv.n, qn, nq, thr_key,
                                                   thr_id, counts, cand, cap, dense, s, status, nullptr, nullptr,
                                                   nullptr, nullptr, block_stats, ChunkOut{});
    MDH_CUDA(cudaGetLastError());
}

void launch_filter_tc_u8_l2(const Level& lv, int dpad, const uint8_t* q, const int32_t* qn, int nq,
                            const uint32_t* thr_key, const int32_t* thr_id, uint32_t* counts, uint2* cand, int cap,
                            int dense, int32_t* status, unsigned long long* block_stats, int exact, cudaStream_t st) {
    if (nq <= 0 || lv.n == 0) return;
    MDH_REQUIRE(dpad == BK && lv.has_tmap, MDH_ERR_INTERNAL, "tensor-core scan needs 128-byte rows and a TMA map");
    MDH_REQUIRE(!dense || cap >= lv.n, MDH_ERR_INTERNAL, "dense scan needs cap >= rows");
    MDH_REQUIRE(!dense || !exact, MDH_ERR_INTERNAL, "a dense scan forms no keys");
    CUtensorMap tq;
    encode_u8_rows_tmap(&tq, q, nq, dpad, BM);
    launch_tc<CfgNarrow>(lv, tq, qn, nq, thr_key, thr_id, counts, cand, cap, dense, status, block_stats, exact, st);
    if (!exact) {
        k_rekey_l2<<<nq, 128, 0, st>>>(counts, cand, cap, lv.norms, qn, dense ? (int)lv.n : 0);
        MDH_CUDA(cudaGetLastError());
    }
}

void launch_filter_tc_u8_l2_units(const Level& lv, int dpad, const uint8_t* qmat, int qmat_rows, const int32_t* qmap,
                                  const int32_t* qn, const ScanUnit* units, int n_units, const int32_t* n_units_dev,
                                  int32_t* unit_counter, const uint32_t* thr_key, const int32_t* thr_id,
                                  uint32_t* counts, uint2* cand, int cap, int32_t* status,
                                  unsigned long long* block_stats, const ChunkOut* defer, cudaStream_t st) {
    using C = CfgNarrow;
    if (n_units <= 0 || qmat_rows <= 0 || lv.n == 0) return;
    MDH_REQUIRE(!defer || (defer->x && defer->hdr && defer->counter && defer->nq > 0 &&
                           defer->capacity >= (uint32_t)kChunkBlock && defer->capacity % kChunkBlock == 0),
                MDH_ERR_INTERNAL, "deferred unit scan needs a chunk buffer of whole 64-entry blocks");
    MDH_REQUIRE(dpad == BK && lv.has_tmap, MDH_ERR_INTERNAL, "tensor-core scan needs 128-byte rows and a TMA map");
    CUtensorMap tq;
    encode_u8_rows_tmap(&tq, qmat, qmat_rows, dpad, BM);
    int dev;
    MDH_CUDA(cudaGetDevice(&dev));
    Sched s{};
    s.n_units = n_units;
    const int ctas = std::min(device_sm_count(dev), n_units);
    if (unit_counter) MDH_CUDA(cudaMemsetAsync(unit_counter, 0, sizeof(int32_t), st));
    if (defer) MDH_CUDA(cudaMemsetAsync(defer->counter, 0, sizeof(uint32_t), st));
    auto kern = defer ? k_filter_tc_u8_l2<C, true, false> : k_filter_tc_u8_l2<C, true, true>;
    MDH_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM_BYTES));
    kern<<<ctas, NUM_THREADS, C::SMEM_BYTES, st>>>(lv.tmap_rows, tq, lv.norms, lv.ids, (int32_t)lv.n, qn, qmat_rows,
                                                   thr_key, thr_id, counts, cand, cap, 0, s, status, units, qmap,
                                                   n_units_dev, unit_counter, block_stats,
                                                   defer ? *defer : ChunkOut{});
    MDH_CUDA(cudaGetLastError());
    if (defer) {
        k_rekey_chunks<<<device_sm_count(dev) * 8, 256, 0, st>>>(*defer, lv.norms, lv.ids, (int32_t)lv.n_pad, qn,
                                                                 defer->nq, thr_key, thr_id, counts, cand, cap,
                                                                 status);
        MDH_CUDA(cudaGetLastError());
    }
}

}  // namespace mdh
