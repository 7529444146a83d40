// Device helpers shared by the CUDA-core scan kernels (scan_simt.cu,
// scan_stream.cu).
#pragma once

#include "common.cuh"

namespace mdh {

// 8-lane butterfly reduce-scatter of QG partial sums.  On return `s[0]` holds
// the complete sum for query `qsel`; `active` marks one lane per (row, query).
template <int QG>
__device__ __forceinline__ void reduce_scatter8(uint32_t (&s)[QG], int l8, int& qsel, bool& active) {
    int c = QG;
    int qbase = 0;
    bool act = true;
#pragma unroll
    for (int m = 4; m >= 1; m >>= 1) {
        if (c > 1) {
            const int h = c / 2;
            const bool up = (l8 & m) != 0;
#pragma unroll
            for (int i = 0; i < QG / 2; i++) {
                if (i < h) {
                    uint32_t send = up ? s[i] : s[i + h];
                    uint32_t keep = up ? s[i + h] : s[i];
                    s[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                }
            }
            if (up) qbase += h;
            c = h;
        } else {
            s[0] += __shfl_xor_sync(0xffffffffu, s[0], m);
            if (l8 & m) act = false;
        }
    }
    qsel = qbase;
    active = act;
}

// Offer row `pos` (key) of query q: dense levels write slot = pos; otherwise
// rows within the threshold (ties resolved by global id) take the next slot.
__device__ __forceinline__ void offer_candidate(uint32_t* counts, uint2* cand, int cap, int dense, int q, uint32_t key,
                                                int64_t pos, const int32_t* ids, uint32_t tkey, int32_t tid) {
    if (dense) {
        cand[(size_t)q * cap + pos] = make_uint2(key, (uint32_t)pos);
        return;
    }
    if (key > tkey) return;
    if (key == tkey && __ldg(ids + pos) > tid) return;
    uint32_t slot = atomicAdd(counts + q, 1u);
    if (slot < (uint32_t)cap) cand[(size_t)q * cap + slot] = make_uint2(key, (uint32_t)pos);
}

}  // namespace mdh
