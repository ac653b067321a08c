// Host-side helpers shared by the backend's translation units: the
// thread-local error message, the device status word, and TMA tensor maps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>

#include "../../include/beatlm_b200.h"
#include "sm100.cuh"

namespace bl {

// Records a printf-style message as this thread's last error; returns `code`.
int fail(int code, const char* fmt, ...);

// The device address of the status word of the current device (looked up
// once per device; allocates nothing).
Status* status_ptr();

// Encodes a 3-D tiled tensor map of 16-bit elements, dims innermost first,
// with 128-byte swizzle, zero fill out of bounds. Returns BL_OK or an error.
int make_tmap_16bit_3d(CUtensorMap* map, const void* base, const uint64_t dims[3],
                       const uint64_t strides_bytes[2], const uint32_t box[3]);

// Same, 2-D.
int make_tmap_16bit_2d(CUtensorMap* map, const void* base, const uint64_t dims[2],
                       uint64_t row_stride_bytes, const uint32_t box[2]);

inline size_t dtype_size(int dt) { return dt == BL_F32 ? 4 : 2; }

}  // namespace bl

#define BL_CUDA_TRY(expr)                                                                \
    do {                                                                                 \
        cudaError_t e_ = (expr);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return ::bl::fail(BL_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                              __FILE__, __LINE__);                                       \
    } while (0)
