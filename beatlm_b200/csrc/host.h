// Host-side helpers shared by the backend's translation units: the
// thread-local error message, the device status word, and TMA tensor maps.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <functional>
#include <utility>

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

// A 2-D map of elements of `esz` bytes (2 or 4) with a swizzle of
// `swizzle_bytes` (0 = none, 64 or 128) matching the box's inner extent; zero
// fill out of bounds.
int make_tmap_2d(CUtensorMap* map, const void* base, int esz, const uint64_t dims[2],
                 uint64_t row_stride_bytes, const uint32_t box[2], int swizzle_bytes);

// The map of make_tmap_16bit_3d in two dimensions.
int make_tmap_16bit_2d(CUtensorMap* map, const void* base, const uint64_t dims[2],
                       uint64_t row_stride_bytes, const uint32_t box[2]);

inline size_t dtype_size(int dt) { return dt == BL_F32 ? 4 : 2; }

// A validated, fully prepared launch: tensor maps encoded, parameters packed,
// kernel attributes set. run() only enqueues (the reference's split between
// Kernels::new, which builds, and Kernels::encode, which records).
struct Launch {
    std::function<cudaError_t(cudaStream_t)> run;
    // set instead of `run` by launches that report a library status (a
    // collective); enqueue() prefers it
    std::function<int(cudaStream_t)> run_status;
    int op = 0;  // bl_op kind
};

int prepare_attention(const bl_attention_args& a, Launch* out);
int prepare_gemm(const bl_gemm_args& g, Launch* out);
// Rows [row_begin, row_end) of the output only (whole 128-row tiles): one
// part of a split kernel.
int prepare_gemm_rows(const bl_gemm_args& g, uint32_t row_begin, uint32_t row_end, Launch* out);
int prepare_layernorm(const bl_layernorm_args& a, Launch* out);
int prepare_layernorm_rows(const bl_layernorm_args& a, uint32_t row_begin, uint32_t row_end,
                           Launch* out);
int prepare_patchify(const bl_patchify_args& a, Launch* out);

// Whether launches carry the programmatic-stream-serialisation attribute
// (on unless the environment sets BEATLM_B200_PDL=0).
bool pdl_enabled();

// Launches `kern` on `s` with programmatic dependent launch when enabled;
// every kernel of this library executes pdl_wait() before touching global
// memory, so the attribute is always safe.
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// launch_k for a grid of thread-block clusters of `cluster` CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_k_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, dim3 cluster,
                             size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster.x;
    attr[1].val.clusterDim.y = cluster.y;
    attr[1].val.clusterDim.z = cluster.z;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Attention's automatic key-split count for these arguments given a
// workspace of `workspace_bytes` (0 = none: the cluster combine).
// Fills in the query tiles per CTA and key splits bl_attention would pick
// (fields left 0) for a workspace of this size (0 = cluster combine).
void attention_resolve(bl_attention_args& a, uint64_t workspace_bytes);

inline int enqueue(const Launch& l, cudaStream_t s) {
    if (l.run_status) return l.run_status(s);
    cudaError_t e = l.run(s);
    if (e != cudaSuccess) return fail(BL_ERR_CUDA, "launch failed: %s", cudaGetErrorString(e));
    return BL_OK;
}

}  // namespace bl

// The peer buffers of a head-parallel exchange (bl_peers_*): this rank's
// buffer, a 256-byte header (arrival flags, one 32-bit word per rank, at 0)
// and two output slots, plus every other rank's buffer mapped into this
// process.
struct bl_peers {
    static constexpr int kMax = 8;
    static constexpr uint64_t kHeader = 256;
    int device = -1;
    uint32_t rank = 0, world = 0;
    uint64_t slot_bytes = 0;   // as asked
    uint64_t slot_stride = 0;  // rounded up to 256
    uint8_t* local = nullptr;  // cudaMalloc'd at create
    uint8_t* base[kMax] = {};  // every rank's buffer in this address space
    bool ipc[kMax] = {};       // base[r] came from cudaIpcOpenMemHandle
    uint32_t epoch = 0;        // the last launch's flag value
};

#define BL_CUDA_TRY(expr)                                                                \
    do {                                                                                 \
        cudaError_t e_ = (expr);                                                         \
        if (e_ != cudaSuccess)                                                           \
            return ::bl::fail(BL_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                              __FILE__, __LINE__);                                       \
    } while (0)
