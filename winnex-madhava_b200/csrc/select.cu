// Selection kernels: candidate lists -> per-query thresholds or final top-k,
// and the merge of per-shard top-k lists.
//
// A query's candidates are sorted in shared memory as 64-bit keys
// (rank key << 32 | row id), so ascending order is exactly the reference's
// (distance, index) order (src/winnex_madhava.cpp:1237-1239) and, for score
// metrics, descending score with the lower index first.
#include "internal.h"

namespace mdh {

namespace {

__device__ __forceinline__ void bitonic_sort_smem(unsigned long long* keys, int P) {
    for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < (P >> 1); i += blockDim.x) {
                int lo = 2 * i - (i & (stride - 1));
                int hi = lo + stride;
                bool asc = (lo & size) == 0;
                unsigned long long a = keys[lo], b = keys[hi];
                if ((a > b) == asc) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
        }
    }
    __syncthreads();
}

__device__ __forceinline__ int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Lowers a query's threshold (key, id) to `v` (key << 32 | id) when that is
// smaller.  Every threshold a selection computes is a valid upper bound on
// the query's k-th (key, id), and so is the one it replaces, so keeping the
// smaller of the two is valid too.  A candidate list may hold rows above the
// threshold that produced it (the scan keeps every row its block bound cannot
// exclude); the minimum keeps an overflow rerun from loosening the bound.
__device__ __forceinline__ void tighten_threshold(uint32_t* thr_key, int32_t* thr_id, int qo, unsigned long long v) {
    const unsigned long long cur = ((unsigned long long)thr_key[qo] << 32) | (uint32_t)thr_id[qo];
    if (v < cur) {
        thr_key[qo] = (uint32_t)(v >> 32);
        thr_id[qo] = (int32_t)(v & 0xffffffffu);
    }
}

__global__ void k_fill_u32(uint32_t* p, int n, uint32_t v) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

__global__ void k_fill_threshold(uint32_t* tk, int32_t* ti, int nq, uint32_t key, int32_t id) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < nq) {
        tk[i] = key;
        ti[i] = id;
    }
}

// k-th smallest (1-based rank k <= c) of keys[0, c) by an 8-bit radix select
// from the most significant digit: O(8 c) instead of a full sort.  Every
// thread of the block calls it and gets the result.
__device__ unsigned long long radix_select_kth(const unsigned long long* keys, int c, int k) {
    __shared__ unsigned int hist[256];
    __shared__ unsigned long long s_prefix;
    __shared__ int s_rem;
    unsigned long long prefix = 0, mask = 0;
    int rem = k;
    for (int d = 7; d >= 0; d--) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const int sh = 8 * d;
        for (int i = threadIdx.x; i < c; i += blockDim.x) {
            const unsigned long long v = keys[i];
            if ((v & mask) == prefix) atomicAdd(&hist[(v >> sh) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // Lane l owns bins [8l, 8l + 8); find the bin where the count reaches rem.
            const int l = threadIdx.x;
            unsigned int own = 0;
#pragma unroll
            for (int b = 0; b < 8; b++) own += hist[8 * l + b];
            unsigned int incl = own;
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) {
                const unsigned int o = __shfl_up_sync(0xffffffffu, incl, m);
                if (l >= m) incl += o;
            }
            const unsigned int excl = incl - own;
            const unsigned int hit = __ballot_sync(0xffffffffu, incl >= (unsigned int)rem);
            if (l == __ffs(hit) - 1) {
                unsigned int cum = excl;
                for (int b = 0; b < 8; b++) {
                    const unsigned int h = hist[8 * l + b];
                    if (cum + h >= (unsigned int)rem) {
                        s_prefix = prefix | ((unsigned long long)(8 * l + b) << sh);
                        s_rem = rem - (int)cum;
                        break;
                    }
                    cum += h;
                }
            }
        }
        __syncthreads();
        prefix = s_prefix;
        rem = s_rem;
        mask |= 0xFFull << sh;
        __syncthreads();
    }
    return prefix;
}

constexpr int kRadixMinCount = 1024;  // below this the bitonic sort is as fast

// One CTA per query.  qmap (optional) maps the CTA's query to the slot its
// threshold / output / flag is written to.
// Candidates are {key, row position in the scanned level}; `ids` maps a
// position to its global row id, which breaks ties.
__global__ void k_select(const uint32_t* __restrict__ counts, const uint2* __restrict__ cand, int cap,
                         const int32_t* __restrict__ ids, int k,
                         int final_, uint32_t* __restrict__ thr_key, int32_t* __restrict__ thr_id,
                         uint32_t* __restrict__ out_key, int32_t* __restrict__ out_id, int32_t* __restrict__ flags,
                         int32_t* __restrict__ n_flagged, const int32_t* __restrict__ qmap,
                         unsigned long long* __restrict__ n_cand) {
    extern __shared__ unsigned long long keys[];
    const int q = blockIdx.x;
    const int qo = qmap ? qmap[q] : q;
    const uint32_t c_all = counts[q];
    const int c = (int)(c_all < (uint32_t)cap ? c_all : (uint32_t)cap);
    const int P = next_pow2(c > k ? c : k);
    const uint2* src = cand + (size_t)q * cap;
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        if (i < c) {
            uint2 e = src[i];
            keys[i] = ((unsigned long long)e.x << 32) | (uint32_t)__ldg(ids + e.y);
        } else {
            keys[i] = ~0ull;
        }
    }
    if (!final_ && c >= k && c > kRadixMinCount) {
        // Only the k-th entry is needed: select it without sorting.
        __syncthreads();
        const unsigned long long kth = radix_select_kth(keys, c, k);
        if (threadIdx.x == 0) {
            tighten_threshold(thr_key, thr_id, qo, kth);
        }
        return;
    }
    bitonic_sort_smem(keys, P);
    if (!final_) {
        if (threadIdx.x == 0) {
            int idx = (c < k ? c : k) - 1;
            if (idx >= 0 && c >= k) {
                tighten_threshold(thr_key, thr_id, qo, keys[idx]);
            } else {
                // Fewer than k rows in this level: every row of the next
                // level stays a candidate.
                thr_key[qo] = kKeyInf;
                thr_id[qo] = kIdInf;
            }
        }
        return;
    }
    if (c_all > (uint32_t)cap) {
        // Overflow: the stored lists are a subset; their k-th key is a valid
        // (tighter) threshold for a rerun.  c == cap >= k here.
        if (threadIdx.x == 0) {
            flags[qo] = 1;
            tighten_threshold(thr_key, thr_id, qo, keys[k - 1]);
            atomicAdd(n_flagged, 1);
        }
        return;
    }
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        if (j < c) {
            out_key[(size_t)qo * k + j] = (uint32_t)(keys[j] >> 32);
            out_id[(size_t)qo * k + j] = (int32_t)(keys[j] & 0xffffffffu);
        } else {
            out_key[(size_t)qo * k + j] = kKeyInf;
            out_id[(size_t)qo * k + j] = -1;
        }
    }
    if (threadIdx.x == 0) {
        if (flags) flags[qo] = 0;
        if (n_cand) atomicAdd(n_cand, (unsigned long long)c);
    }
}

// The same contract as k_select for k <= kWarpSelectK, one warp per query:
// each lane keeps the kWarpSelectK smallest composite keys of its stride of
// the list in registers (ascending), reading a row's id only when its key
// could enter; the warp then pops the k smallest in order by warp minima.
// The block kernel sizes its shared memory by the list capacity, so on long
// lists it runs one query per SM at a time; this one streams the list.
constexpr int kWarpSelectK = 16;
constexpr int kWarpSelectWarps = 8;  // queries per 256-thread block

__global__ void __launch_bounds__(32 * kWarpSelectWarps)
    k_select_warp(const uint32_t* __restrict__ counts, const uint2* __restrict__ cand, int cap,
                  const int32_t* __restrict__ ids, int nq, int k, int final_, uint32_t* __restrict__ thr_key,
                  int32_t* __restrict__ thr_id, uint32_t* __restrict__ out_key, int32_t* __restrict__ out_id,
                  int32_t* __restrict__ flags, int32_t* __restrict__ n_flagged, const int32_t* __restrict__ qmap,
                  unsigned long long* __restrict__ n_cand) {
    constexpr int KM = kWarpSelectK;
    const int q = blockIdx.x * kWarpSelectWarps + (int)(threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (q >= nq) return;  // whole warps leave together
    const int qo = qmap ? qmap[q] : q;
    const uint32_t c_all = counts[q];
    const int c = (int)(c_all < (uint32_t)cap ? c_all : (uint32_t)cap);
    const uint2* src = cand + (size_t)q * cap;
    unsigned long long top[KM];
#pragma unroll
    for (int j = 0; j < KM; j++) top[j] = ~0ull;
    unsigned long long worst = ~0ull;  // this lane's k-th smallest so far
    // Eight loads per lane in flight per round: the list is streamed, not
    // walked one dependent load at a time.
    constexpr int U = 8;
    for (int i0 = lane; i0 < c; i0 += 32 * U) {
        uint2 e[U];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int i = i0 + 32 * u;
            e[u] = i < c ? src[i] : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            if (i0 + 32 * u >= c) break;
            const unsigned long long hi = (unsigned long long)e[u].x << 32;
            if (hi > worst) continue;  // its composite key is larger still
            const unsigned long long v = hi | (uint32_t)__ldg(ids + e[u].y);
            if (v >= worst) continue;
            // Insert into the ascending list (the last slot drops out).
#pragma unroll
            for (int j = KM - 1; j > 0; j--) top[j] = top[j - 1] > v ? top[j - 1] : (top[j] > v ? v : top[j]);
            top[0] = top[0] > v ? v : top[0];
            unsigned long long w = top[0];
#pragma unroll
            for (int j = 1; j < KM; j++) w = (j == k - 1) ? top[j] : w;
            worst = w;
        }
    }
    // The k smallest of the warp, ascending: lane r ends with the r-th.
    unsigned long long res = ~0ull;
    for (int r = 0; r < k; r++) {
        unsigned long long m = top[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, m, o);
            m = other < m ? other : m;
        }
        if (lane == r) res = m;
        if (m != ~0ull && top[0] == m) {  // composite keys are unique: one lane pops
#pragma unroll
            for (int j = 0; j < KM - 1; j++) top[j] = top[j + 1];
            top[KM - 1] = ~0ull;
        }
    }
    const unsigned long long kth = __shfl_sync(0xffffffffu, res, k - 1);
    if (!final_) {
        if (lane == 0) {
            if (c >= k) {
                tighten_threshold(thr_key, thr_id, qo, kth);
            } else {
                // Fewer than k rows in this level: every row of the next
                // level stays a candidate.
                thr_key[qo] = kKeyInf;
                thr_id[qo] = kIdInf;
            }
        }
        return;
    }
    if (c_all > (uint32_t)cap) {
        // Overflow: the stored lists are a subset; their k-th key is a valid
        // (tighter) threshold for a rerun.  c == cap >= k here.
        if (lane == 0) {
            flags[qo] = 1;
            tighten_threshold(thr_key, thr_id, qo, kth);
            atomicAdd(n_flagged, 1);
        }
        return;
    }
    if (lane < k) {
        if (lane < c) {
            out_key[(size_t)qo * k + lane] = (uint32_t)(res >> 32);
            out_id[(size_t)qo * k + lane] = (int32_t)(res & 0xffffffffu);
        } else {
            out_key[(size_t)qo * k + lane] = kKeyInf;
            out_id[(size_t)qo * k + lane] = -1;
        }
    }
    if (lane == 0) {
        if (flags) flags[qo] = 0;
        if (n_cand) atomicAdd(n_cand, (unsigned long long)c);
    }
}

// The same contract for kWarpSelectK < k <= kWarpSelectBigK, one warp per
// query.  A lane's 8 smallest keys (keys only, no ids) form, over the warp,
// a set U of min(c, 256) entries of the list; its k-th smallest key tau is at
// least the list's k-th smallest key, so every entry of the top k has a key
// <= tau.  The entries with key <= tau (usually little more than k) are
// collected with their ids into shared memory and sorted there (bitonic).
// If more than kBigBuf of them exist (many equal keys), the k smallest are
// instead taken one at a time by warp minima over the list.
constexpr int kWarpSelectBigK = 128;
constexpr int kBigT = 8;                // keys kept per lane in the first pass
constexpr int kBigWarps = 4;            // queries per 128-thread block
constexpr int kBigBuf = 1024;           // collected entries per warp (8 KB)
static_assert(kWarpSelectBigK <= 32 * kBigT, "the first pass keeps at least k keys");

__global__ void __launch_bounds__(32 * kBigWarps)
    k_select_warp_big(const uint32_t* __restrict__ counts, const uint2* __restrict__ cand, int cap,
                      const int32_t* __restrict__ ids, int nq, int k, int final_, uint32_t* __restrict__ thr_key,
                      int32_t* __restrict__ thr_id, uint32_t* __restrict__ out_key, int32_t* __restrict__ out_id,
                      int32_t* __restrict__ flags, int32_t* __restrict__ n_flagged, const int32_t* __restrict__ qmap,
                      unsigned long long* __restrict__ n_cand) {
    __shared__ unsigned long long bufs[kBigWarps][kBigBuf];
    const int wq = (int)(threadIdx.x >> 5);
    const int q = blockIdx.x * kBigWarps + wq;
    const int lane = threadIdx.x & 31;
    if (q >= nq) return;  // whole warps leave together
    unsigned long long* buf = bufs[wq];
    const int qo = qmap ? qmap[q] : q;
    const uint32_t c_all = counts[q];
    const int c = (int)(c_all < (uint32_t)cap ? c_all : (uint32_t)cap);
    const uint2* src = cand + (size_t)q * cap;
    // Pass 1: this lane's kBigT smallest keys, ascending (empty slots hold 2^32).
    unsigned long long t[kBigT];
#pragma unroll
    for (int j = 0; j < kBigT; j++) t[j] = 1ull << 32;
    for (int i = lane; i < c; i += 32) {
        const unsigned long long v = src[i].x;
        if (v >= t[kBigT - 1]) continue;
#pragma unroll
        for (int j = kBigT - 1; j > 0; j--) t[j] = t[j - 1] > v ? t[j - 1] : (t[j] > v ? v : t[j]);
        t[0] = t[0] > v ? v : t[0];
    }
    // tau: the k-th smallest of the warp's kept keys (all keys when c < k).
    unsigned long long tau = 1ull << 32;
    if (c >= k) {
        for (int r = 0; r < k; r++) {
            unsigned long long m = t[0];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, m, o);
                m = other < m ? other : m;
            }
            const unsigned own = __ballot_sync(0xffffffffu, t[0] == m);
            if (lane == __ffs(own) - 1) {
#pragma unroll
                for (int j = 0; j < kBigT - 1; j++) t[j] = t[j + 1];
                t[kBigT - 1] = 1ull << 32;
            }
            tau = m;
        }
    }
    // Pass 2: collect the entries with key <= tau, with their ids.
    int n = 0;  // entries found (may exceed kBigBuf)
    for (int i0 = 0; i0 < c; i0 += 32) {
        const int i = i0 + lane;
        bool take = false;
        uint2 e = make_uint2(0u, 0u);
        if (i < c) {
            e = src[i];
            take = (unsigned long long)e.x <= tau;
        }
        const unsigned b = __ballot_sync(0xffffffffu, take);
        const int pos = n + __popc(b & ((1u << lane) - 1u));
        if (take && pos < kBigBuf) buf[pos] = ((unsigned long long)e.x << 32) | (uint32_t)__ldg(ids + e.y);
        n += __popc(b);
    }
    __syncwarp();
    const int kk = c < k ? c : k;  // entries of the result
    if (n <= kBigBuf) {
        // Bitonic sort of buf[0, P), P = next power of two >= n, padded with the largest key.
        int P = 1;
        while (P < n) P <<= 1;
        for (int i = n + lane; i < P; i += 32) buf[i] = ~0ull;
        __syncwarp();
        for (int size = 2; size <= P; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = lane; i < (P >> 1); i += 32) {
                    const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                    const bool asc = (lo & size) == 0;
                    const unsigned long long a = buf[lo], b = buf[hi];
                    if ((a > b) == asc) {
                        buf[lo] = b;
                        buf[hi] = a;
                    }
                }
                __syncwarp();
            }
    } else {
        // Many entries share keys <= tau: take the k smallest (key, id) one at a
        // time; round r finds the smallest entry above round r-1's.
        unsigned long long prev = 0;
        for (int r = 0; r < kk; r++) {
            unsigned long long best = ~0ull;
            for (int i = lane; i < c; i += 32) {
                const uint2 e = src[i];
                if ((unsigned long long)e.x > tau || ((unsigned long long)e.x << 32) > best) continue;
                const unsigned long long v = ((unsigned long long)e.x << 32) | (uint32_t)__ldg(ids + e.y);
                if ((r == 0 || v > prev) && v < best) best = v;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                best = other < best ? other : best;
            }
            if (lane == 0) buf[r] = best;
            prev = best;
        }
        __syncwarp();
    }
    if (!final_) {
        if (lane == 0) {
            if (c >= k) {
                tighten_threshold(thr_key, thr_id, qo, buf[k - 1]);
            } else {
                // Fewer than k rows in this level: every row of the next
                // level stays a candidate.
                thr_key[qo] = kKeyInf;
                thr_id[qo] = kIdInf;
            }
        }
        return;
    }
    if (c_all > (uint32_t)cap) {
        // Overflow: the stored lists are a subset; their k-th key is a valid
        // (tighter) threshold for a rerun.  c == cap >= k here.
        if (lane == 0) {
            flags[qo] = 1;
            tighten_threshold(thr_key, thr_id, qo, buf[k - 1]);
            atomicAdd(n_flagged, 1);
        }
        return;
    }
    for (int j = lane; j < k; j += 32) {
        if (j < kk) {
            out_key[(size_t)qo * k + j] = (uint32_t)(buf[j] >> 32);
            out_id[(size_t)qo * k + j] = (int32_t)(buf[j] & 0xffffffffu);
        } else {
            out_key[(size_t)qo * k + j] = kKeyInf;
            out_id[(size_t)qo * k + j] = -1;
        }
    }
    if (lane == 0) {
        if (flags) flags[qo] = 0;
        if (n_cand) atomicAdd(n_cand, (unsigned long long)c);
    }
}

// Verification: query i of a compact list gets the threshold (key, id) of the
// kk-th entry of its result (an empty entry, id -1, means no threshold).
__global__ void k_verify_thresholds(const int32_t* __restrict__ list, int m, const uint32_t* __restrict__ out_key,
                                    const int32_t* __restrict__ out_id, int k, int kk, uint32_t* __restrict__ thr_key,
                                    int32_t* __restrict__ thr_id) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const size_t e = (size_t)list[i] * k + (kk - 1);
    const int32_t id = out_id[e];
    thr_key[i] = id >= 0 ? out_key[e] : kKeyInf;
    thr_id[i] = id >= 0 ? id : kIdInf;
}

// Every row at or before the kk-th result, by (key, id), was counted by an
// exact scan; an exact result has exactly kk of them.
__global__ void k_count_violations(const uint32_t* __restrict__ counts, int m, int kk,
                                   unsigned long long* __restrict__ violations) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= m) return;
    const long long d = (long long)counts[i] - kk;
    if (d != 0) atomicAdd(violations, (unsigned long long)(d > 0 ? d : -d));
}

// Merge [nshard][nq][k] lists into [nq][k]; id -1 marks an empty entry.
__global__ void k_merge_topk(const uint32_t* __restrict__ key_all, const int32_t* __restrict__ id_all, int nshard,
                             int nq, int k, uint32_t* __restrict__ key_out, int32_t* __restrict__ id_out) {
    extern __shared__ unsigned long long keys[];
    const int q = blockIdx.x;
    const int tot = nshard * k;
    const int P = next_pow2(tot);
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        unsigned long long v = ~0ull;
        if (i < tot) {
            int s = i / k, j = i - s * k;
            size_t off = ((size_t)s * nq + q) * k + j;
            int32_t id = id_all[off];
            if (id >= 0) v = ((unsigned long long)key_all[off] << 32) | (uint32_t)id;
        }
        keys[i] = v;
    }
    bitonic_sort_smem(keys, P);
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        unsigned long long v = keys[j];
        if (v == ~0ull) {
            key_out[(size_t)q * k + j] = kKeyInf;
            id_out[(size_t)q * k + j] = -1;
        } else {
            key_out[(size_t)q * k + j] = (uint32_t)(v >> 32);
            id_out[(size_t)q * k + j] = (int32_t)(v & 0xffffffffu);
        }
    }
}

// One thread per 16-byte piece of a gathered row (dpad is a multiple of 16).
__global__ void k_gather_queries_u8(const uint8_t* __restrict__ src, const int32_t* __restrict__ qn_src,
                                    const int32_t* __restrict__ list, int m, int dpad, uint8_t* __restrict__ dst,
                                    int32_t* __restrict__ qn_dst) {
    const int per_row = dpad >> 4;
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)m * per_row) return;
    const int i = (int)(t / per_row), b = (int)(t - (int64_t)i * per_row) * 16;
    const int s = list[i];
    *reinterpret_cast<uint4*>(dst + (size_t)i * dpad + b) = *reinterpret_cast<const uint4*>(src + (size_t)s * dpad + b);
    if (b == 0) qn_dst[i] = qn_src[s];
}

size_t select_smem(int P) { return (size_t)P * sizeof(unsigned long long); }

}  // namespace

void launch_fill_u32(uint32_t* p, int n, uint32_t v, cudaStream_t st) {
    if (n <= 0) return;
    k_fill_u32<<<(n + 255) / 256, 256, 0, st>>>(p, n, v);
    MDH_CUDA(cudaGetLastError());
}

void launch_fill_threshold(uint32_t* thr_key, int32_t* thr_id, int nq, uint32_t key, int32_t id, cudaStream_t st) {
    if (nq <= 0) return;
    k_fill_threshold<<<(nq + 255) / 256, 256, 0, st>>>(thr_key, thr_id, nq, key, id);
    MDH_CUDA(cudaGetLastError());
}

void launch_select(const uint32_t* counts, const uint2* cand, int cap, const int32_t* ids, int nq, int k, int final_,
                   uint32_t* thr_key,
                   int32_t* thr_id, uint32_t* out_key, int32_t* out_id, int32_t* flags, int32_t* n_flagged,
                   const int32_t* qmap, unsigned long long* n_cand, cudaStream_t st) {
    if (nq <= 0) return;
    if (k >= 1 && k <= kWarpSelectK) {
        k_select_warp<<<(nq + kWarpSelectWarps - 1) / kWarpSelectWarps, 32 * kWarpSelectWarps, 0, st>>>(
            counts, cand, cap, ids, nq, k, final_, thr_key, thr_id, out_key, out_id, flags, n_flagged, qmap, n_cand);
        MDH_CUDA(cudaGetLastError());
        return;
    }
    if (k <= kWarpSelectBigK) {
        k_select_warp_big<<<(nq + kBigWarps - 1) / kBigWarps, 32 * kBigWarps, 0, st>>>(
            counts, cand, cap, ids, nq, k, final_, thr_key, thr_id, out_key, out_id, flags, n_flagged, qmap, n_cand);
        MDH_CUDA(cudaGetLastError());
        return;
    }
    int pmax = 1;
    while (pmax < (cap > k ? cap : k)) pmax <<= 1;
    size_t smem = select_smem(pmax);
    MDH_REQUIRE(smem <= 220 * 1024, MDH_ERR_UNSUPPORTED, "candidate list too large for the selection kernel");
    if (smem > 48 * 1024) MDH_CUDA(cudaFuncSetAttribute(k_select, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    int threads = pmax >= 4096 ? 1024 : (pmax >= 1024 ? 512 : 256);
    k_select<<<nq, threads, smem, st>>>(counts, cand, cap, ids, k, final_, thr_key, thr_id, out_key, out_id, flags,
                                        n_flagged, qmap, n_cand);
    MDH_CUDA(cudaGetLastError());
}

namespace {

__global__ void k_thresholds_from_lists(const uint32_t* __restrict__ keys, const int32_t* __restrict__ ids, int nq,
                                        int k, uint32_t* __restrict__ thr_key, int32_t* __restrict__ thr_id) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    const size_t e = (size_t)q * k + (k - 1);
    const int32_t id = ids[e];
    thr_key[q] = id >= 0 ? keys[e] : kKeyInf;
    thr_id[q] = id >= 0 ? id : kIdInf;
}

}  // namespace

void launch_thresholds_from_lists(const uint32_t* keys, const int32_t* ids, int nq, int k, uint32_t* thr_key,
                                  int32_t* thr_id, cudaStream_t st) {
    if (nq <= 0 || k <= 0) return;
    k_thresholds_from_lists<<<(nq + 255) / 256, 256, 0, st>>>(keys, ids, nq, k, thr_key, thr_id);
    MDH_CUDA(cudaGetLastError());
}

void launch_verify_thresholds(const int32_t* list, int m, const uint32_t* out_key, const int32_t* out_id, int k, int kk,
                              uint32_t* thr_key, int32_t* thr_id, cudaStream_t st) {
    if (m <= 0) return;
    k_verify_thresholds<<<(m + 255) / 256, 256, 0, st>>>(list, m, out_key, out_id, k, kk, thr_key, thr_id);
    MDH_CUDA(cudaGetLastError());
}

void launch_count_violations(const uint32_t* counts, int m, int kk, unsigned long long* violations, cudaStream_t st) {
    if (m <= 0) return;
    k_count_violations<<<(m + 255) / 256, 256, 0, st>>>(counts, m, kk, violations);
    MDH_CUDA(cudaGetLastError());
}

void launch_merge_topk(const uint32_t* key_all, const int32_t* id_all, int nshard, int nq, int k, uint32_t* key_out,
                       int32_t* id_out, cudaStream_t st) {
    if (nq <= 0 || k <= 0) return;
    int P = 1;
    while (P < nshard * k) P <<= 1;
    size_t smem = select_smem(P);
    MDH_REQUIRE(smem <= 220 * 1024, MDH_ERR_UNSUPPORTED, "nshard * k too large for the merge kernel");
    if (smem > 48 * 1024)
        MDH_CUDA(cudaFuncSetAttribute(k_merge_topk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_merge_topk<<<nq, 256, smem, st>>>(key_all, id_all, nshard, nq, k, key_out, id_out);
    MDH_CUDA(cudaGetLastError());
}

namespace {

// Float query rows of a compact list: src [nq][dim] then [nq] aux, dst
// [m][dim] then [m] aux; one thread per element.
__global__ void k_gather_queries_f32(const float* __restrict__ src, int nq, int dim, const int32_t* __restrict__ list,
                                     int m, float* __restrict__ dst) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t per = (int64_t)dim + 1;
    if (t >= (int64_t)m * per) return;
    const int i = (int)(t / per), j = (int)(t - (int64_t)i * per);
    const int s = list[i];
    if (j < dim)
        dst[(size_t)i * dim + j] = src[(size_t)s * dim + j];
    else
        dst[(size_t)m * dim + i] = src[(size_t)nq * dim + s];
}

}  // namespace

void launch_gather_queries_f32(const float* src, int nq, int dim, const int32_t* list, int m, float* dst,
                               cudaStream_t st) {
    if (m <= 0) return;
    const int64_t total = (int64_t)m * (dim + 1);
    k_gather_queries_f32<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, nq, dim, list, m, dst);
    MDH_CUDA(cudaGetLastError());
}

void launch_gather_queries_u8(const uint8_t* src, const int32_t* qn_src, const int32_t* list, int m, int dpad,
                              uint8_t* dst, int32_t* qn_dst, cudaStream_t st) {
    if (m <= 0) return;
    MDH_REQUIRE(dpad % 16 == 0, MDH_ERR_INTERNAL, "query rows must be 16-byte multiples");
    const int64_t pieces = (int64_t)m * (dpad / 16);
    k_gather_queries_u8<<<(unsigned)((pieces + 255) / 256), 256, 0, st>>>(src, qn_src, list, m, dpad, dst, qn_dst);
    MDH_CUDA(cudaGetLastError());
}

}  // namespace mdh
