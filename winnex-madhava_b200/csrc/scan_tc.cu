// Tensor-core scan (placeholder until the tcgen05 kernel lands).
#include "internal.h"

namespace mdh {

bool tc_supported(const mdh_index*, const Level&) { return false; }
void make_tmap_rows(Level&, int) {}
void launch_filter_tc_u8_l2(const Level&, int, const uint8_t*, const int32_t*, int, const uint32_t*, const int32_t*,
                            uint32_t*, uint2*, int, int32_t*, cudaStream_t) {
    throw Error(MDH_ERR_UNSUPPORTED, "tensor-core scan not built");
}

}  // namespace mdh
