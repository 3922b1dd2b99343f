// ============================================================================
//  launch.cuh -- launch bookkeeping shared by every kernel file.
// ============================================================================
#pragma once

#include "common.cuh"

namespace tg {

void count_launch();     // one per kernel launch (tg_kernel_launch_count)
void require_device();   // throws TG_ERR_NO_DEVICE without a GPU

// Launch `kernel<<<grid, block, smem, stream>>>(args...)`, count it and check
// the launch.  Empty grids launch nothing.
template <class K, class... A>
inline void launch(const char* name, K kernel, dim3 grid, dim3 block, size_t smem,
                   cudaStream_t s, A... args) {
    if (grid.x == 0 || grid.y == 0 || grid.z == 0) return;
    kernel<<<grid, block, smem, s>>>(args...);
    count_launch();
    TG_LAUNCH_CHECK(name);
}

// Common argument checks with the reference's wording.
inline void check_ld(const char* fn, const char* what, int64_t ld, int64_t cols) {
    if (ld < cols)
        invalid(std::string(fn) + ": leading dimension of " + what + " (" + std::to_string(ld) +
                ") is smaller than its column count (" + std::to_string(cols) + ")");
}

inline void check_ptr(const char* fn, const char* what, const void* p, bool needed) {
    if (needed && p == nullptr) invalid(std::string(fn) + ": " + what + " is NULL");
}

}  // namespace tg
