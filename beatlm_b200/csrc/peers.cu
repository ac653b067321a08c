// Peer buffers for the head-parallel exchange of the long-sequence attention:
// one device buffer per rank (an arrival-flag header and two output slots),
// exported as a CUDA IPC handle and mapped by the other ranks of the node, so
// that each rank's attention kernel stores its heads' rows straight into
// every rank's output over NVLink (bl_attention_peers). The reference runs on
// one device and has no counterpart; the buffers are allocated once at
// set-up, like the reference's arenas (crates/beatlm/src/gpu/arenas.rs:88).
#include <cstring>

#include "host.h"

static_assert(sizeof(cudaIpcMemHandle_t) == BL_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" uint64_t bl_peers_buffer_bytes(uint64_t slot_bytes) {
    const uint64_t stride = (slot_bytes + 255) / 256 * 256;
    return bl_peers::kHeader + 2 * stride;
}

extern "C" int bl_peers_create(uint32_t rank, uint32_t world, uint64_t slot_bytes,
                               bl_peers** out) {
    using namespace bl;
    if (out == nullptr) return fail(BL_ERR_INVALID, "peers: null argument");
    if (world < 1 || world > static_cast<uint32_t>(bl_peers::kMax) || rank >= world)
        return fail(BL_ERR_INVALID, "peers: rank %u of %u (at most %d ranks)", rank, world,
                    bl_peers::kMax);
    if (slot_bytes == 0) return fail(BL_ERR_INVALID, "peers: empty output slot");
    int dev = 0;
    BL_CUDA_TRY(cudaGetDevice(&dev));
    bl_peers* p = new bl_peers();
    p->device = dev;
    p->rank = rank;
    p->world = world;
    p->slot_bytes = slot_bytes;
    p->slot_stride = (slot_bytes + 255) / 256 * 256;
    void* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, bl_peers_buffer_bytes(slot_bytes));
    if (e == cudaSuccess) e = cudaMemset(mem, 0, bl_peers_buffer_bytes(slot_bytes));
    if (e != cudaSuccess) {
        if (mem) cudaFree(mem);
        delete p;
        return fail(BL_ERR_CUDA, "peers: %s", cudaGetErrorString(e));
    }
    p->local = static_cast<uint8_t*>(mem);
    p->base[rank] = p->local;
    *out = p;
    return BL_OK;
}

extern "C" int bl_peers_handle(const bl_peers* p, void* handle) {
    using namespace bl;
    if (p == nullptr || handle == nullptr) return fail(BL_ERR_INVALID, "peers: null argument");
    cudaIpcMemHandle_t h;
    BL_CUDA_TRY(cudaIpcGetMemHandle(&h, p->local));
    memcpy(handle, &h, sizeof h);
    return BL_OK;
}

extern "C" int bl_peers_open(bl_peers* p, const void* handles, size_t n) {
    using namespace bl;
    if (p == nullptr || (handles == nullptr && n > 0)) return fail(BL_ERR_INVALID, "peers: null argument");
    if (n != p->world) return fail(BL_ERR_INVALID, "peers: %zu handles for %u ranks", n, p->world);
    int dev = 0;
    BL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != p->device)
        return fail(BL_ERR_INVALID, "peers: made on device %d, opened on device %d", p->device, dev);
    for (uint32_t r = 0; r < p->world; ++r) {
        if (r == p->rank) continue;
        if (p->base[r] != nullptr) return fail(BL_ERR_INVALID, "peers: rank %u already mapped", r);
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + r * sizeof h, sizeof h);
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return fail(BL_ERR_CUDA, "peers: opening rank %u's buffer: %s", r, cudaGetErrorString(e));
        p->base[r] = static_cast<uint8_t*>(ptr);
        p->ipc[r] = true;
    }
    return BL_OK;
}

extern "C" int bl_peers_attach(bl_peers* p, uint32_t rank, void* buffer) {
    using namespace bl;
    if (p == nullptr || buffer == nullptr) return fail(BL_ERR_INVALID, "peers: null argument");
    if (rank >= p->world || rank == p->rank)
        return fail(BL_ERR_INVALID, "peers: cannot attach rank %u (this is rank %u of %u)", rank,
                    p->rank, p->world);
    if (p->base[rank] != nullptr) return fail(BL_ERR_INVALID, "peers: rank %u already mapped", rank);
    if (reinterpret_cast<uintptr_t>(buffer) & 255u)
        return fail(BL_ERR_INVALID, "peers: an attached buffer must be 256-byte aligned");
    p->base[rank] = static_cast<uint8_t*>(buffer);
    return BL_OK;
}

extern "C" void* bl_peers_slot(const bl_peers* p, uint32_t slot) {
    if (p == nullptr || slot > 1) return nullptr;
    return p->local + bl_peers::kHeader + slot * p->slot_stride;
}

extern "C" uint32_t bl_peers_next_epoch(const bl_peers* p) { return p ? p->epoch + 1 : 0; }

extern "C" void bl_peers_destroy(bl_peers* p) {
    if (p == nullptr) return;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != p->device) cudaSetDevice(p->device);
    for (int r = 0; r < bl_peers::kMax; ++r)
        if (p->ipc[r] && p->base[r] != nullptr) cudaIpcCloseMemHandle(p->base[r]);
    if (p->local) cudaFree(p->local);
    if (prev >= 0 && prev != p->device) cudaSetDevice(prev);
    cudaGetLastError();
    delete p;
}
