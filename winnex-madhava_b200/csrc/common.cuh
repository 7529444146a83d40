// Shared definitions for the B200 exact top-K scan library.
//
// Candidate keys: every scan kernel ranks (query, row) pairs by a 32-bit
// unsigned "rank key" (smaller = better) and the global row id (smaller wins a
// tie).  For integer L2 the key is the squared distance itself; float scores
// go through an order-preserving bit map (ordered_key_*).  A candidate record
// is a uint2 {key, id}; a 64-bit sort key is (key << 32) | id.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "winnex_madhava_b200.h"

namespace mdh {

// Error raised inside the library; converted to an mdh_status at the C ABI.
struct Error : std::runtime_error {
    mdh_status code;
    Error(mdh_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void throw_cuda(cudaError_t e, const char* what, const char* file, int line);

#define MDH_CUDA(call)                                                   \
    do {                                                                 \
        cudaError_t e_ = (call);                                         \
        if (e_ != cudaSuccess) ::mdh::throw_cuda(e_, #call, __FILE__, __LINE__); \
    } while (0)

#define MDH_REQUIRE(cond, code, msg)                                     \
    do {                                                                 \
        if (!(cond)) throw ::mdh::Error((code), (msg));                  \
    } while (0)

constexpr int kRowAlign = 128;          // dimension padding unit (bytes) for u8 rows
constexpr int kTileRows = 256;          // row padding unit (one tensor-core N tile)
constexpr int32_t kNormPad = 1 << 30;   // |v|^2 stored for padding rows: never passes a filter
constexpr uint32_t kKeyInf = 0xFFFFFFFFu;
constexpr int32_t kIdInf = 0x7FFFFFFF;

// Device error codes written to the per-call status word.
enum DevErr : int32_t { kDevOk = 0, kDevTimeout = 1, kDevBadShape = 2 };

__host__ __device__ inline int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// Order-preserving float -> u32 map (ascending float -> ascending u32);
// -0.0 is folded onto +0.0 so the two compare equal as in C++.
__host__ __device__ inline uint32_t ordered_key_asc(float f) {
    if (f == 0.0f) f = 0.0f;
    uint32_t u;
#ifdef __CUDA_ARCH__
    u = __float_as_uint(f);
#else
    __builtin_memcpy(&u, &f, 4);
#endif
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Descending float (higher score = better = smaller key).
__host__ __device__ inline uint32_t ordered_key_desc(float f) { return ~ordered_key_asc(f); }

__host__ __device__ inline float key_to_float_asc(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    float f;
#ifdef __CUDA_ARCH__
    f = __uint_as_float(u);
#else
    __builtin_memcpy(&f, &u, 4);
#endif
    return f;
}

// Candidate threshold test: (key, id) <= (tkey, tid) lexicographically.
__device__ __forceinline__ bool within_threshold(uint32_t key, int32_t id, uint32_t tkey, int32_t tid) {
    return key < tkey || (key == tkey && id <= tid);
}

}  // namespace mdh
