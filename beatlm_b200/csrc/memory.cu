// The static memory plan and its single device allocation.
//
// Plan: a restatement of MemoryPlan::new (crates/beatlm-core/src/memory.rs:285-375)
// with the same rules and the same placement decisions, so a plan made here
// equals the reference's for the same tensors and profile.
// Arenas: the reference makes one wgpu buffer per arena (crates/beatlm/src/gpu/
// arenas.rs:88-111). On a B200 nothing limits a binding below the device's
// memory, so the arenas become consecutive 256-byte-aligned ranges of ONE
// cudaMalloc, made once; the frame loop allocates nothing.

#include <algorithm>
#include <map>
#include <mutex>
#include <new>
#include <set>
#include <vector>

#include "host.h"

namespace {

constexpr uint64_t kStorageGranularity = 4;  // memory.rs:85, STORAGE_GRANULARITY
constexpr uint64_t kArenaBaseAlign = 256;    // base of each arena in the single allocation

bool round_up(uint64_t v, uint64_t m, uint64_t* out) {
    const uint64_t rem = v % m;
    if (rem == 0) {
        *out = v;
        return true;
    }
    if (v > UINT64_MAX - (m - rem)) return false;
    *out = v + (m - rem);
    return true;
}

bool overlaps(const bl_tensor_desc& a, const bl_tensor_desc& b) {
    return a.first_use <= b.last_use && b.first_use <= a.last_use;
}

uint64_t arena_cap(const bl_device_profile& p) {
    return std::min(p.max_binding_bytes, p.max_buffer_bytes);
}

struct Sized {
    bl_tensor_desc desc;
    uint64_t size;
};

struct Placed {
    bl_tensor_desc desc;
    uint64_t offset, size;
};

struct ArenaFill {
    std::vector<Placed> placed;
    uint64_t size = 0;

    // The lowest aligned offset where `item` fits beside every placed tensor
    // whose lifetime intersects its own, or false when it would pass `cap`
    // (Arena::lowest_fit, memory.rs:448-466): walk the busy ranges in order
    // of start and take the first gap that holds the aligned item.
    bool lowest_fit(const Sized& item, uint64_t alignment, uint64_t cap, uint64_t* out) const {
        std::vector<std::pair<uint64_t, uint64_t>> busy;
        for (const Placed& p : placed)
            if (overlaps(p.desc, item.desc))
                busy.emplace_back(p.offset, p.offset + std::min(p.size, UINT64_MAX - p.offset));
        std::sort(busy.begin(), busy.end());
        uint64_t candidate = 0;
        for (const auto& [start, end] : busy) {
            uint64_t aligned;
            if (!round_up(candidate, alignment, &aligned)) return false;
            if (aligned > UINT64_MAX - item.size) return false;
            if (aligned + item.size <= start) break;
            candidate = std::max(candidate, end);
        }
        uint64_t offset;
        if (!round_up(candidate, alignment, &offset)) return false;
        if (offset > UINT64_MAX - item.size || offset + item.size > cap) return false;
        *out = offset;
        return true;
    }
};

// The most bytes in use at one operation (peak_live, memory.rs:487-506).
uint64_t peak_live(const std::vector<Sized>& sized) {
    std::map<uint64_t, std::pair<uint64_t, uint64_t>> deltas;  // op -> (born, died)
    auto sat_add = [](uint64_t a, uint64_t b) { return a > UINT64_MAX - b ? UINT64_MAX : a + b; };
    for (const Sized& s : sized) {
        auto& born = deltas[s.desc.first_use];
        born.first = sat_add(born.first, s.size);
        auto& died = deltas[static_cast<uint64_t>(s.desc.last_use) + 1];
        died.second = sat_add(died.second, s.size);
    }
    uint64_t live = 0, peak = 0;
    for (const auto& [op, d] : deltas) {
        live = sat_add(live, d.first);
        live = live >= d.second ? live - d.second : 0;
        peak = std::max(peak, live);
    }
    return peak;
}

int plan_fail(bl_plan_error* err, int kind, uint32_t id, uint64_t a, uint64_t b) {
    if (err) *err = bl_plan_error{kind, id, a, b};
    switch (kind) {
    case BL_PLAN_DUPLICATE_TENSOR:
        return bl::fail(BL_ERR_INVALID, "tensor %u is described more than once", id);
    case BL_PLAN_INVALID_LIFETIME:
        return bl::fail(BL_ERR_INVALID,
                        "tensor %u is first used at operation %llu, after its last use at %llu",
                        id, (unsigned long long)a, (unsigned long long)b);
    case BL_PLAN_EMPTY_TENSOR:
        return bl::fail(BL_ERR_INVALID, "tensor %u has no elements", id);
    case BL_PLAN_SIZE_OVERFLOW:
        return bl::fail(BL_ERR_INVALID, "the size of tensor %u overflows", id);
    case BL_PLAN_TENSOR_TOO_LARGE:
        return bl::fail(BL_ERR_CAPACITY, "tensor %u needs %llu bytes but an arena holds at most %llu",
                        id, (unsigned long long)a, (unsigned long long)b);
    case BL_PLAN_INVALID_PROFILE:
        return bl::fail(BL_ERR_INVALID,
                        "the device profile has a zero offset alignment or a zero arena size");
    default:
        return bl::fail(BL_ERR_INVALID, "too many tensors to plan");
    }
}

}  // namespace

struct bl_plan {
    std::vector<uint64_t> arenas;
    std::map<uint32_t, bl_placement> placements;
    uint64_t peak_live_bytes = 0;
    uint64_t offset_alignment = 0;
};

struct bl_arenas {
    int device = 0;
    char* base = nullptr;
    uint64_t bytes = 0;
    uint64_t alignment = 0;
    std::vector<uint64_t> starts, sizes;  // per arena: offset in the allocation, size
};

extern "C" {

int bl_device_profile_webgpu_baseline(bl_device_profile* out) {
    if (!out) return bl::fail(BL_ERR_INVALID, "profile: null output");
    *out = bl_device_profile{128ull << 20, 256ull << 20, 256};
    return BL_OK;
}

int bl_device_profile_cuda(int device, bl_device_profile* out) {
    if (!out) return bl::fail(BL_ERR_INVALID, "profile: null output");
    int prev = 0;
    BL_CUDA_TRY(cudaGetDevice(&prev));
    BL_CUDA_TRY(cudaSetDevice(device));
    size_t free_b = 0, total_b = 0;
    const cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
    cudaSetDevice(prev);
    if (e != cudaSuccess)
        return bl::fail(BL_ERR_CUDA, "cudaMemGetInfo: %s", cudaGetErrorString(e));
    *out = bl_device_profile{total_b, total_b, 256};
    return BL_OK;
}

int bl_plan_create(const bl_tensor_desc* tensors, size_t n, const bl_device_profile* profile,
                   bl_plan** out, bl_plan_error* err) {
    if (err) *err = bl_plan_error{0, 0, 0, 0};
    if (!out || !profile || (n > 0 && !tensors))
        return bl::fail(BL_ERR_INVALID, "plan: null argument");
    *out = nullptr;
    const uint64_t alignment = profile->offset_alignment;
    const uint64_t cap = arena_cap(*profile);
    if (alignment == 0 || cap == 0) return plan_fail(err, BL_PLAN_INVALID_PROFILE, 0, 0, 0);
    if (n > UINT32_MAX) return plan_fail(err, BL_PLAN_TOO_MANY_TENSORS, 0, 0, 0);

    // validate (memory.rs:341-372): in listed order, the first problem wins
    std::set<uint32_t> seen;
    std::vector<Sized> sized;
    sized.reserve(n);
    for (size_t i = 0; i < n; ++i) {
        const bl_tensor_desc& d = tensors[i];
        if (!seen.insert(d.id).second) return plan_fail(err, BL_PLAN_DUPLICATE_TENSOR, d.id, 0, 0);
        if (d.first_use > d.last_use)
            return plan_fail(err, BL_PLAN_INVALID_LIFETIME, d.id, d.first_use, d.last_use);
        if (d.elements == 0) return plan_fail(err, BL_PLAN_EMPTY_TENSOR, d.id, 0, 0);
        if (d.elem_bytes == 0) return bl::fail(BL_ERR_INVALID, "tensor %u: zero element width", d.id);
        uint64_t size;
        if (d.elements > UINT64_MAX / d.elem_bytes ||
            !round_up(d.elements * d.elem_bytes, kStorageGranularity, &size))
            return plan_fail(err, BL_PLAN_SIZE_OVERFLOW, d.id, 0, 0);
        if (size > cap) return plan_fail(err, BL_PLAN_TENSOR_TOO_LARGE, d.id, size, cap);
        sized.push_back(Sized{d, size});
    }

    bl_plan* plan = new (std::nothrow) bl_plan;
    if (!plan) return bl::fail(BL_ERR_CAPACITY, "plan: out of host memory");
    plan->peak_live_bytes = peak_live(sized);
    plan->offset_alignment = alignment;

    // greedy by size, descending, ties by id (memory.rs:300-301)
    std::vector<Sized> order = sized;
    std::sort(order.begin(), order.end(), [](const Sized& a, const Sized& b) {
        return a.size != b.size ? a.size > b.size : a.desc.id < b.desc.id;
    });
    std::vector<ArenaFill> arenas;
    for (const Sized& item : order) {
        size_t index = arenas.size();
        uint64_t offset = 0;
        for (size_t i = 0; i < arenas.size(); ++i)
            if (arenas[i].lowest_fit(item, alignment, cap, &offset)) {
                index = i;
                break;
            }
        if (index == arenas.size()) {
            arenas.emplace_back();
            offset = 0;
        }
        ArenaFill& a = arenas[index];
        a.placed.push_back(Placed{item.desc, offset, item.size});
        a.size = std::max(a.size, offset + item.size);
        plan->placements[item.desc.id] =
            bl_placement{static_cast<uint32_t>(index), 0, offset, item.size};
    }
    for (const ArenaFill& a : arenas) plan->arenas.push_back(a.size);
    *out = plan;
    return BL_OK;
}

void bl_plan_destroy(bl_plan* p) { delete p; }

size_t bl_plan_arenas(const bl_plan* p, uint64_t* sizes, size_t cap) {
    if (!p) return 0;
    for (size_t i = 0; i < std::min(cap, p->arenas.size()); ++i) sizes[i] = p->arenas[i];
    return p->arenas.size();
}

int bl_plan_placement(const bl_plan* p, uint32_t id, bl_placement* out) {
    if (!p || !out) return bl::fail(BL_ERR_INVALID, "placement: null argument");
    auto it = p->placements.find(id);
    if (it == p->placements.end())
        return bl::fail(BL_ERR_INVALID, "tensor %u is not in the plan", id);
    *out = it->second;
    return BL_OK;
}

uint64_t bl_plan_peak_live_bytes(const bl_plan* p) { return p ? p->peak_live_bytes : 0; }

uint64_t bl_plan_total_bytes(const bl_plan* p) {
    if (!p) return 0;
    uint64_t sum = 0;
    for (uint64_t a : p->arenas) sum = a > UINT64_MAX - sum ? UINT64_MAX : sum + a;
    return sum;
}

int bl_plan_valid_on(const bl_plan* p, const bl_device_profile* profile) {
    if (!p || !profile) return 0;
    const uint64_t alignment = profile->offset_alignment;
    if (alignment == 0 || p->offset_alignment % alignment != 0) return 0;
    const uint64_t cap = arena_cap(*profile);
    for (uint64_t a : p->arenas)
        if (a > cap) return 0;
    return 1;
}

int bl_arenas_create(const bl_plan* p, int device, bl_arenas** out) {
    if (!p || !out) return bl::fail(BL_ERR_INVALID, "arenas: null argument");
    *out = nullptr;
    bl_device_profile prof;
    if (int rc = bl_device_profile_cuda(device, &prof)) return rc;
    if (!bl_plan_valid_on(p, &prof))
        return bl::fail(BL_ERR_INVALID,
                        "the memory plan is not valid on this device: arena cap %llu, alignment %u",
                        (unsigned long long)arena_cap(prof), prof.offset_alignment);
    bl_arenas* a = new (std::nothrow) bl_arenas;
    if (!a) return bl::fail(BL_ERR_CAPACITY, "arenas: out of host memory");
    a->device = device;
    a->alignment = prof.offset_alignment;
    uint64_t at = 0;
    for (uint64_t size : p->arenas) {
        uint64_t start;
        if (!round_up(at, kArenaBaseAlign, &start) || start > UINT64_MAX - size) {
            delete a;
            return bl::fail(BL_ERR_CAPACITY, "arenas: total size overflows");
        }
        a->starts.push_back(start);
        a->sizes.push_back(size);
        at = start + size;
    }
    a->bytes = at;
    if (at > 0) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(device);
        if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&a->base), at);
        cudaSetDevice(prev);
        if (e != cudaSuccess) {
            delete a;
            return bl::fail(e == cudaErrorMemoryAllocation ? BL_ERR_CAPACITY : BL_ERR_CUDA,
                            "arenas: cudaMalloc of %llu bytes: %s", (unsigned long long)at,
                            cudaGetErrorString(e));
        }
    }
    *out = a;
    return BL_OK;
}

void bl_arenas_destroy(bl_arenas* a) {
    if (!a) return;
    if (a->base) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(a->device);
        cudaFree(a->base);
        cudaSetDevice(prev);
    }
    delete a;
}

uint64_t bl_arenas_bytes(const bl_arenas* a) { return a ? a->bytes : 0; }

int bl_arenas_base(const bl_arenas* a, uint32_t arena, void** out) {
    if (!a || !out) return bl::fail(BL_ERR_INVALID, "arenas: null argument");
    if (arena >= a->starts.size())
        return bl::fail(BL_ERR_INVALID, "arena %u does not exist in this set", arena);
    *out = a->base + a->starts[arena];
    return BL_OK;
}

int bl_arenas_binding(const bl_arenas* a, const bl_placement* p, void** out) {
    if (!a || !p || !out) return bl::fail(BL_ERR_INVALID, "binding: null argument");
    if (p->arena >= a->starts.size())
        return bl::fail(BL_ERR_INVALID, "arena %u does not exist in this set", p->arena);
    const uint64_t size = a->sizes[p->arena];
    if (p->size == 0 || p->offset > size || p->size > size - p->offset)
        return bl::fail(BL_ERR_INVALID,
                        "placement at offset %llu of %llu bytes does not lie inside its arena",
                        (unsigned long long)p->offset, (unsigned long long)p->size);
    if (p->offset % a->alignment != 0)
        return bl::fail(BL_ERR_INVALID, "placement at offset %llu is not aligned to %llu bytes",
                        (unsigned long long)p->offset, (unsigned long long)a->alignment);
    *out = a->base + a->starts[p->arena] + p->offset;
    return BL_OK;
}

static int arenas_copy(const bl_arenas* a, const bl_placement* p, uint64_t offset, void* host,
                       uint64_t bytes, void* stream, bool write) {
    void* dev = nullptr;
    if (int rc = bl_arenas_binding(a, p, &dev)) return rc;
    if (!host && bytes) return bl::fail(BL_ERR_INVALID, "arenas: null host pointer");
    if (offset > p->size || bytes > p->size - offset)
        return bl::fail(BL_ERR_INVALID, "%llu bytes at %llu pass the end of a %llu-byte placement",
                        (unsigned long long)bytes, (unsigned long long)offset,
                        (unsigned long long)p->size);
    if (bytes == 0) return BL_OK;
    char* d = static_cast<char*>(dev) + offset;
    const cudaError_t e =
        write ? cudaMemcpyAsync(d, host, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream)
              : cudaMemcpyAsync(host, d, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    if (e != cudaSuccess) return bl::fail(BL_ERR_CUDA, "arenas copy: %s", cudaGetErrorString(e));
    return BL_OK;
}

int bl_arenas_write(const bl_arenas* a, const bl_placement* p, uint64_t offset, const void* src,
                    uint64_t bytes, void* stream) {
    return arenas_copy(a, p, offset, const_cast<void*>(src), bytes, stream, true);
}

int bl_arenas_read(const bl_arenas* a, const bl_placement* p, uint64_t offset, void* dst,
                   uint64_t bytes, void* stream) {
    return arenas_copy(a, p, offset, dst, bytes, stream, false);
}

}  // extern "C"
