// The program of a model on the device: prepared launches (the reference's
// Kernels), the row split of Program::split, CUDA-graph replay, and the
// cudaEvent slice timer with the reference SliceTimer's semantics.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <deque>
#include <string>
#include <vector>

#include "host.h"

// ------------------------------------------------------------------ split

extern "C" uint32_t bl_split_edges(uint32_t extent, uint32_t grain, uint32_t count,
                                   uint32_t* edges) {
    if (grain == 0) grain = 1;
    const uint64_t blocks = (static_cast<uint64_t>(extent) + grain - 1) / grain;
    const uint64_t maxp = blocks > 0 ? blocks : 1;
    uint64_t c = count < 1 ? 1 : count;
    if (c > maxp) c = maxp;
    if (edges != nullptr) {
        for (uint64_t i = 0; i <= c; ++i) {
            const uint64_t unit = blocks * i / c * grain;
            edges[i] = static_cast<uint32_t>(unit < extent ? unit : extent);
        }
    }
    return static_cast<uint32_t>(c);
}

extern "C" uint32_t bl_parts_within(uint64_t duration_us, uint64_t bound_us, uint32_t max_parts) {
    if (bound_us == 0) return 0;
    uint64_t want = duration_us / bound_us + (duration_us % bound_us != 0 ? 1 : 0);
    if (want < 1) want = 1;
    const uint64_t cap = max_parts < 1 ? 1 : max_parts;
    return static_cast<uint32_t>(want < cap ? want : cap);
}

// Program::parts_within (kernel.rs:2350-2366): bl_parts_within for every
// kernel with its own duration and max_parts.
extern "C" int bl_program_parts_within(const bl_kernel_spec* specs, size_t n,
                                       const uint64_t* durations_us, size_t n_durations,
                                       uint64_t bound_us, uint32_t* parts_out) {
    if (n_durations != n)
        return bl::fail(BL_ERR_INVALID, "parts_within: %zu durations for %zu kernels (PartCounts)",
                        n_durations, n);
    if (bound_us == 0)
        return bl::fail(BL_ERR_INVALID, "parts_within: no dispatch fits a bound of zero (ZeroBound)");
    if (n > 0 && (specs == nullptr || durations_us == nullptr || parts_out == nullptr))
        return bl::fail(BL_ERR_INVALID, "parts_within: null argument");
    for (size_t i = 0; i < n; ++i) {
        const uint32_t mp = bl_kernel_spec_max_parts(&specs[i]);
        parts_out[i] = bl_parts_within(durations_us[i], bound_us, mp > 0 ? mp : 1);
    }
    return BL_OK;
}

// ------------------------------------------------------------------ timer

namespace bl {

enum class SlotState { Free, Recording, Submitted, Held, Rejected, Invalid };

struct TimerSlot {
    SlotState state = SlotState::Free;
    uint64_t frame = 0;
    uint64_t seq = 0;  // submission order
    std::vector<cudaEvent_t> begin, end;
    std::vector<uint32_t> kernel;
    uint32_t used = 0;
};

}  // namespace bl

struct bl_timer {
    uint32_t max_slices = 0;
    bl::TimerSlot slots[BL_TIMER_RING_DEPTH];
    uint32_t next = 0;           // ring position of the next claim
    uint64_t next_seq = 0;
    std::deque<int> submitted;   // slot indices in submission order
    bl_timer_stats stats{};
};

namespace {
bool valid_handle(const bl_timer* t, int32_t h) {
    return t != nullptr && h >= 0 && h < BL_TIMER_RING_DEPTH;
}
void release(bl_timer* t, int i) {
    t->slots[i].state = bl::SlotState::Free;
    t->slots[i].used = 0;
}
}  // namespace

extern "C" int bl_timer_create(uint32_t max_slices, bl_timer** out) {
    using namespace bl;
    if (out == nullptr || max_slices == 0) return fail(BL_ERR_INVALID, "timer: max_slices must be > 0");
    bl_timer* t = new bl_timer();
    t->max_slices = max_slices;
    for (auto& s : t->slots) {
        s.begin.resize(max_slices);
        s.end.resize(max_slices);
        s.kernel.resize(max_slices);
        for (uint32_t i = 0; i < max_slices; ++i) {
            if (cudaEventCreate(&s.begin[i]) != cudaSuccess ||
                cudaEventCreate(&s.end[i]) != cudaSuccess) {
                bl_timer_destroy(t);
                return fail(BL_ERR_CUDA, "timer: cudaEventCreate failed");
            }
        }
    }
    *out = t;
    return BL_OK;
}

extern "C" void bl_timer_destroy(bl_timer* t) {
    if (t == nullptr) return;
    for (auto& s : t->slots) {
        for (auto e : s.begin) if (e) cudaEventDestroy(e);
        for (auto e : s.end) if (e) cudaEventDestroy(e);
    }
    delete t;
}

extern "C" uint32_t bl_timer_max_slices(const bl_timer* t) { return t ? t->max_slices : 0; }

extern "C" int bl_timer_begin_frame(bl_timer* t, uint64_t frame, int32_t* handle) {
    using namespace bl;
    if (t == nullptr || handle == nullptr) return fail(BL_ERR_INVALID, "timer: null argument");
    const int i = static_cast<int>(t->next);
    if (t->slots[i].state != SlotState::Free) {
        t->stats.frames_skipped += 1;
        *handle = -1;
        return BL_OK;
    }
    t->next = (t->next + 1) % BL_TIMER_RING_DEPTH;
    t->slots[i].state = SlotState::Recording;
    t->slots[i].frame = frame;
    t->slots[i].used = 0;
    *handle = i;
    return BL_OK;
}

static int submit(bl_timer* t, int32_t h, bool held) {
    using namespace bl;
    if (t == nullptr) return fail(BL_ERR_INVALID, "timer: null timer");
    if (h == -1) return BL_OK;
    if (!valid_handle(t, h) || t->slots[h].state != SlotState::Recording)
        return fail(BL_ERR_INVALID, "timer: handle %d is not a frame being recorded", h);
    t->slots[h].state = held ? SlotState::Held : SlotState::Submitted;
    t->slots[h].seq = t->next_seq++;
    t->submitted.push_back(h);
    return BL_OK;
}

extern "C" int bl_timer_submitted(bl_timer* t, int32_t h) { return submit(t, h, false); }
extern "C" int bl_timer_submitted_held(bl_timer* t, int32_t h) { return submit(t, h, true); }

extern "C" int bl_timer_settle(bl_timer* t, int32_t h, int accept) {
    using namespace bl;
    if (!valid_handle(t, h) || t->slots[h].state != SlotState::Held)
        return fail(BL_ERR_INVALID, "timer: handle %d is not a held frame", h);
    t->slots[h].state = accept ? SlotState::Submitted : SlotState::Rejected;
    return BL_OK;
}

extern "C" int bl_timer_drop(bl_timer* t, int32_t h) {
    using namespace bl;
    if (t == nullptr) return fail(BL_ERR_INVALID, "timer: null timer");
    if (h == -1) return BL_OK;
    if (!valid_handle(t, h) || t->slots[h].state != SlotState::Recording)
        return fail(BL_ERR_INVALID, "timer: handle %d is not a frame being recorded", h);
    release(t, h);
    return BL_OK;
}

extern "C" size_t bl_timer_invalidate_submitted(bl_timer* t) {
    if (t == nullptr) return 0;
    size_t n = 0;
    for (int i : t->submitted) {
        auto& s = t->slots[i];
        if (s.state == bl::SlotState::Submitted || s.state == bl::SlotState::Held) {
            s.state = bl::SlotState::Invalid;
            ++n;
        }
    }
    return n;
}

extern "C" size_t bl_timer_in_flight(const bl_timer* t) {
    if (t == nullptr) return 0;
    size_t n = 0;
    for (const auto& s : t->slots) n += s.state != bl::SlotState::Free;
    return n;
}

extern "C" int bl_timer_collect_ready(bl_timer* t, bl_slice_time* out, size_t cap, size_t* n,
                                      size_t* frames) {
    using namespace bl;
    if (t == nullptr || n == nullptr) return fail(BL_ERR_INVALID, "timer: null argument");
    size_t written = 0, done = 0;
    while (!t->submitted.empty()) {
        const int i = t->submitted.front();
        TimerSlot& s = t->slots[i];
        if (s.state == SlotState::Invalid || s.state == SlotState::Rejected) {
            // Never decoded; a marked frame holds nothing back once its
            // events can no longer be written (they may still be pending, but
            // nothing reads them before the slot is re-recorded in order).
            t->stats.frames_failed += 1;
            t->submitted.pop_front();
            release(t, i);
            continue;
        }
        if (s.state == SlotState::Held) break;  // unsettled: later frames wait
        bool failed = false;
        if (s.used > 0) {
            cudaError_t q = cudaEventQuery(s.end[s.used - 1]);
            if (q == cudaErrorNotReady) break;
            if (q != cudaSuccess) failed = true;
        }
        if (!failed && written + s.used > cap) break;  // whole frames only
        float ms = 0.0f;
        for (uint32_t k = 0; k < s.used && !failed; ++k) {
            float b = 0.0f;
            if (cudaEventElapsedTime(&ms, s.begin[k], s.end[k]) != cudaSuccess ||
                cudaEventElapsedTime(&b, s.begin[0], s.begin[k]) != cudaSuccess) {
                failed = true;
                break;
            }
            out[written + k].frame = s.frame;
            out[written + k].slice = k;
            out[written + k].kernel = s.kernel[k];
            out[written + k].begin_us = 1000.0 * b;
            out[written + k].micros = 1000.0 * ms;
        }
        t->submitted.pop_front();
        if (failed) {
            cudaGetLastError();  // a failed query must not leak into later calls
            t->stats.frames_failed += 1;
        } else {
            written += s.used;
            done += 1;
            t->stats.frames_collected += 1;
        }
        release(t, i);
    }
    *n = written;
    if (frames != nullptr) *frames = done;
    return BL_OK;
}

extern "C" int bl_timer_get_stats(const bl_timer* t, bl_timer_stats* out) {
    if (t == nullptr || out == nullptr) return bl::fail(BL_ERR_INVALID, "timer: null argument");
    *out = t->stats;
    return BL_OK;
}

// ------------------------------------------------------------------ kernels

// The launches of a program: kernel i (a part) under binding set j is
// launches[launch_of[i][j]]; a kernel that touches none of a set's
// substituted tensors shares set 0's launch (the reference shares its bind
// group between such sets, crates/beatlm/src/codegen/kernels.rs:1-10).
struct bl_kernels {
    std::vector<bl::Launch> launches;
    std::vector<std::vector<uint32_t>> launch_of;
    std::vector<std::string> labels;
    size_t sets = 1;
    const bl::Launch& at(size_t kernel, size_t set) const {
        return launches[launch_of[kernel][set]];
    }
};

struct bl_graph {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

namespace {

// The split dimension of a spec and its grain (the split_extent and
// split_grain of the reference's MainOp, kernel.rs:1975): query rows in
// 128-row tiles for attention, output rows in 128-row tiles for a matrix
// multiply, rows for a LayerNorm; a patch embedding runs whole. False for an
// unknown op.
bool split_dims(const bl_kernel_spec& s, uint32_t* extent, uint32_t* grain) {
    *extent = 1, *grain = 1;
    switch (s.op) {
        case BL_OP_ATTENTION: {
            const auto& a = *static_cast<const bl_attention_args*>(s.args);
            *extent = a.row_end > a.row_begin ? a.row_end - a.row_begin : 0;
            *grain = 128;
            return true;
        }
        case BL_OP_GEMM: *extent = static_cast<const bl_gemm_args*>(s.args)->m; *grain = 128; return true;
        case BL_OP_LAYERNORM: *extent = static_cast<const bl_layernorm_args*>(s.args)->rows; return true;
        case BL_OP_PATCHIFY:
        case BL_OP_ALLGATHER: return true;
        default: return false;
    }
}

// A binding set's substitutions applied to one pointer argument: a pointer
// into [from, from + bytes) moves to the same offset from `to`. Counts the
// pointers moved.
struct Rebind {
    const bl_binding_set* set = nullptr;
    int moved = 0;
    template <typename P>
    void operator()(P*& p) {
        if (set == nullptr || p == nullptr) return;
        const uintptr_t v = reinterpret_cast<uintptr_t>(p);
        for (size_t i = 0; i < set->n; ++i) {
            const bl_substitution& u = set->subs[i];
            const uintptr_t f = reinterpret_cast<uintptr_t>(u.from);
            if (v >= f && v - f < u.bytes) {
                p = reinterpret_cast<P*>(reinterpret_cast<uintptr_t>(u.to) + (v - f));
                ++moved;
                return;
            }
        }
    }
};

void rebind(bl_attention_args& a, Rebind& r) { r(a.qkv), r(a.out), r(a.workspace), r(a.trace); }
void rebind(bl_gemm_args& g, Rebind& r) {
    r(g.a), r(g.b), r(g.ln_x), r(g.ln_gamma), r(g.ln_beta), r(g.bias), r(g.chan_scale);
    r(g.residual), r(g.out), r(g.stats_out), r(g.ln_stats), r(g.norm_out), r(g.norm_gamma);
    r(g.norm_beta), r(g.norm_sync), r(g.workspace);
}
void rebind(bl_layernorm_args& a, Rebind& r) { r(a.x), r(a.gamma), r(a.beta), r(a.out); }
void rebind(bl_patchify_args& a, Rebind& r) { r(a.image), r(a.a), r(a.cls), r(a.pos), r(a.x); }
void rebind(bl_allgather_args& a, Rebind& r) { r(a.send), r(a.recv); }

// Part [edges[i], edges[i + 1]) of spec `s` with binding set `set` (NULL =
// as given); *moved = how many pointer arguments the set redirected.
int prepare_part(const bl_kernel_spec& s, const std::vector<uint32_t>& edges, uint32_t i,
                 const bl_binding_set* set, int* moved, bl::Launch* l, size_t index) {
    using namespace bl;
    Rebind r;
    r.set = set;
    switch (s.op) {
        case BL_OP_ATTENTION: {
            bl_attention_args a = *static_cast<const bl_attention_args*>(s.args);
            rebind(a, r);
            // Every part uses the whole kernel's key splits (and query
            // tiles), so each row is computed exactly as the whole kernel
            // computes it.
            attention_resolve(a, a.workspace != nullptr ? a.workspace_bytes : 0);
            const uint32_t r0 = a.row_begin;
            a.row_begin = r0 + edges[i];
            a.row_end = r0 + edges[i + 1];
            *moved = r.moved;
            return prepare_attention(a, l);
        }
        case BL_OP_GEMM: {
            bl_gemm_args g = *static_cast<const bl_gemm_args*>(s.args);
            rebind(g, r);
            *moved = r.moved;
            return prepare_gemm_rows(g, edges[i], edges[i + 1], l);
        }
        case BL_OP_LAYERNORM: {
            bl_layernorm_args a = *static_cast<const bl_layernorm_args*>(s.args);
            rebind(a, r);
            *moved = r.moved;
            return prepare_layernorm_rows(a, edges[i], edges[i + 1], l);
        }
        case BL_OP_ALLGATHER: {
            bl_allgather_args g = *static_cast<const bl_allgather_args*>(s.args);
            rebind(g, r);
            *moved = r.moved;
            if (g.comm == nullptr || g.send == nullptr || g.recv == nullptr)
                return fail(BL_ERR_INVALID, "kernel %zu: all-gather needs a communicator "
                                            "and buffers", index);
            l->op = BL_OP_ALLGATHER;
            l->run_status = [g](cudaStream_t st) {
                return bl_comm_all_gather(g.comm, g.send, g.recv, g.bytes, st);
            };
            return BL_OK;
        }
        default: {
            bl_patchify_args a = *static_cast<const bl_patchify_args*>(s.args);
            rebind(a, r);
            *moved = r.moved;
            return prepare_patchify(a, l);
        }
    }
}

int add_spec(bl_kernels* k, const bl_kernel_spec& s, size_t index, const bl_binding_set* sets,
             size_t nsets) {
    using namespace bl;
    if (s.args == nullptr) return fail(BL_ERR_INVALID, "kernel %zu: null args", index);
    const std::string base = s.label ? s.label : ("kernel " + std::to_string(index));
    uint32_t extent = 1, grain = 1;
    if (!split_dims(s, &extent, &grain))
        return fail(BL_ERR_INVALID, "kernel %zu: unknown op %d", index, s.op);
    std::vector<uint32_t> edges(static_cast<size_t>(s.parts > 1 ? s.parts : 1) + 1);
    const bool whole = s.op == BL_OP_PATCHIFY || s.op == BL_OP_ALLGATHER;
    const uint32_t count = whole ? 1 : bl_split_edges(extent, grain, s.parts, edges.data());
    if (whole) { edges[0] = 0; edges[1] = 1; }
    for (uint32_t i = 0; i < count; ++i) {
        std::vector<uint32_t> of(nsets == 0 ? 1 : nsets);
        for (size_t j = 0; j < of.size(); ++j) {
            Launch l;
            int moved = 0;
            int rc = prepare_part(s, edges, i, nsets == 0 ? nullptr : &sets[j], &moved, &l, index);
            if (rc != BL_OK) return rc;
            if (j > 0 && moved == 0) {
                of[j] = of[0];  // untouched by this set: set 0's launch
                continue;
            }
            of[j] = static_cast<uint32_t>(k->launches.size());
            k->launches.push_back(std::move(l));
        }
        k->launch_of.push_back(std::move(of));
        k->labels.push_back(count == 1 ? base
                                       : base + " [" + std::to_string(i + 1) + "/" +
                                             std::to_string(count) + "]");
    }
    return BL_OK;
}

int encode_one(const bl_kernels* k, size_t kernel, size_t set, cudaStream_t s, bl_timer* t,
               int32_t h) {
    using namespace bl;
    if (kernel >= k->launch_of.size())
        return fail(BL_ERR_INVALID, "encode: kernel %zu of %zu", kernel, k->launch_of.size());
    if (set >= k->sets)
        return fail(BL_ERR_INVALID, "encode: binding set %zu of %zu", set, k->sets);
    TimerSlot* slot = nullptr;
    if (t != nullptr && h >= 0) {
        if (!valid_handle(t, h) || t->slots[h].state != SlotState::Recording)
            return fail(BL_ERR_INVALID, "encode: timer handle %d is not being recorded", h);
        slot = &t->slots[h];
        if (slot->used >= t->max_slices)
            return fail(BL_ERR_CAPACITY, "encode: more than %u timed passes in one frame",
                        t->max_slices);
        BL_CUDA_TRY(cudaEventRecord(slot->begin[slot->used], s));
    }
    int rc = enqueue(k->at(kernel, set), s);
    if (rc != BL_OK) return rc;
    if (slot != nullptr) {
        BL_CUDA_TRY(cudaEventRecord(slot->end[slot->used], s));
        slot->kernel[slot->used] = static_cast<uint32_t>(kernel);
        slot->used += 1;
    }
    return BL_OK;
}

}  // namespace

extern "C" int bl_kernels_create(const bl_kernel_spec* specs, size_t n, const bl_binding_set* sets,
                                 size_t nsets, bl_kernels** out) {
    using namespace bl;
    if (out == nullptr || (specs == nullptr && n > 0) || (sets == nullptr && nsets > 0))
        return fail(BL_ERR_INVALID, "kernels: null argument");
    for (size_t j = 0; j < nsets; ++j) {
        if (sets[j].subs == nullptr && sets[j].n > 0)
            return fail(BL_ERR_INVALID, "kernels: binding set %zu: null substitutions", j);
        for (size_t i = 0; i < sets[j].n; ++i) {
            const bl_substitution& u = sets[j].subs[i];
            if (u.from == nullptr || u.to == nullptr || u.bytes == 0)
                return fail(BL_ERR_INVALID, "kernels: binding set %zu, substitution %zu: empty", j, i);
            const uintptr_t f = reinterpret_cast<uintptr_t>(u.from);
            for (size_t i2 = 0; i2 < i; ++i2) {
                const bl_substitution& w = sets[j].subs[i2];
                const uintptr_t g = reinterpret_cast<uintptr_t>(w.from);
                if (f < g + w.bytes && g < f + u.bytes)
                    return fail(BL_ERR_INVALID, "kernels: binding set %zu: substitutions %zu and "
                                                "%zu replace overlapping tensors", j, i2, i);
            }
        }
    }
    bl_kernels* k = new bl_kernels();
    k->sets = nsets == 0 ? 1 : nsets;
    for (size_t i = 0; i < n; ++i) {
        int rc = add_spec(k, specs[i], i, sets, nsets);
        if (rc != BL_OK) {
            delete k;
            return rc;
        }
    }
    *out = k;
    return BL_OK;
}

extern "C" void bl_kernels_destroy(bl_kernels* k) { delete k; }

extern "C" size_t bl_kernels_len(const bl_kernels* k) { return k ? k->launch_of.size() : 0; }

extern "C" size_t bl_kernels_sets(const bl_kernels* k) { return k ? k->sets : 0; }

extern "C" size_t bl_kernels_launches(const bl_kernels* k) { return k ? k->launches.size() : 0; }

extern "C" const char* bl_kernels_label(const bl_kernels* k, size_t kernel) {
    if (k == nullptr || kernel >= k->labels.size()) return nullptr;
    return k->labels[kernel].c_str();
}

extern "C" int bl_kernels_encode(const bl_kernels* k, size_t kernel, size_t set, void* stream,
                                 bl_timer* t, int32_t frame) {
    if (k == nullptr) return bl::fail(BL_ERR_INVALID, "encode: null kernels");
    return encode_one(k, kernel, set, static_cast<cudaStream_t>(stream), t, frame);
}

extern "C" int bl_kernels_encode_range(const bl_kernels* k, size_t begin, size_t end, size_t set,
                                       void* stream, bl_timer* t, int32_t frame) {
    if (k == nullptr || begin > end || end > k->launch_of.size())
        return bl::fail(BL_ERR_INVALID, "encode: range [%zu, %zu)", begin, end);
    for (size_t i = begin; i < end; ++i) {
        int rc = encode_one(k, i, set, static_cast<cudaStream_t>(stream), t, frame);
        if (rc != BL_OK) return rc;
    }
    return BL_OK;
}

extern "C" int bl_kernels_capture(const bl_kernels* k, size_t set, void* stream, bl_graph** out) {
    using namespace bl;
    if (k == nullptr || out == nullptr) return fail(BL_ERR_INVALID, "capture: null argument");
    if (set >= k->sets) return fail(BL_ERR_INVALID, "capture: binding set %zu of %zu", set, k->sets);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (s == nullptr) return fail(BL_ERR_INVALID, "capture: needs a non-default stream");
    BL_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
    int rc = BL_OK;
    for (size_t i = 0; i < k->launch_of.size() && rc == BL_OK; ++i) rc = enqueue(k->at(i, set), s);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (rc != BL_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return fail(BL_ERR_CUDA, "capture: %s", cudaGetErrorString(e));
    bl_graph* gr = new bl_graph();
    gr->graph = g;
    e = cudaGraphInstantiate(&gr->exec, g, 0);
    if (e != cudaSuccess) {
        cudaGraphDestroy(g);
        delete gr;
        return fail(BL_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    }
    *out = gr;
    return BL_OK;
}

extern "C" int bl_graph_launch(const bl_graph* g, void* stream) {
    if (g == nullptr) return bl::fail(BL_ERR_INVALID, "graph: null");
    BL_CUDA_TRY(cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream)));
    return BL_OK;
}

extern "C" void bl_graph_destroy(bl_graph* g) {
    if (g == nullptr) return;
    if (g->exec) cudaGraphExecDestroy(g->exec);
    if (g->graph) cudaGraphDestroy(g->graph);
    delete g;
}

// KernelSpec::max_parts (kernel.rs:1975): the split extent in grains.
extern "C" uint32_t bl_kernel_spec_max_parts(const bl_kernel_spec* s) {
    if (s == nullptr || s->args == nullptr) return 0;
    uint32_t extent = 1, grain = 1;
    if (!split_dims(*s, &extent, &grain)) return 0;
    if (s->op == BL_OP_PATCHIFY || s->op == BL_OP_ALLGATHER) return 1;
    return static_cast<uint32_t>((static_cast<uint64_t>(extent) + grain - 1) / grain);
}

// ------------------------------------------------------------------ pass cost
// What a launch costs apart from the work it does, with and without its
// event pair: the reference's pass-cost workload
// (crates/beatlm-host/src/pass_cost.rs:1-110) with a CUDA launch as the pass,
// a cudaEvent pair as its timestamp writes and a CUDA graph as "one pass".

namespace {

// One block of one thread per group adds one to its word, so every launch
// reads what the one before it wrote (the reference's SHADER, pass_cost.rs:128).
__global__ void pass_cost_kernel(uint32_t* sink) { sink[blockIdx.x] += 1u; }

// The same under programmatic dependent launch: the next launch may start
// at once, and each waits for the one before it to finish before its
// read-modify-write.
__global__ void pass_cost_kernel_pdl(uint32_t* sink) {
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    sink[blockIdx.x] += 1u;
}

struct EventSet {
    std::vector<cudaEvent_t> ev;
    ~EventSet() {
        for (cudaEvent_t e : ev) cudaEventDestroy(e);
    }
};

}  // namespace

extern "C" int bl_pass_cost_frame_run(const bl_pass_cost_args* a, bl_pass_cost_frame* out) {
    using namespace bl;
    if (a == nullptr || out == nullptr) return fail(BL_ERR_INVALID, "pass cost: null argument");
    const uint32_t P = a->passes;
    if (P < 1) return fail(BL_ERR_INVALID, "pass cost: at least one pass");
    if (a->variant < BL_PASS_PER_PASS || a->variant > BL_PASS_ONE_PASS_PDL)
        return fail(BL_ERR_INVALID, "pass cost: variant %d", a->variant);
    if (a->variant == BL_PASS_EVERY && a->every < 1)
        return fail(BL_ERR_INVALID, "pass cost: every:k needs k >= 1");
    if (a->kernels != nullptr) {
        if (P > a->kernels->launch_of.size())
            return fail(BL_ERR_INVALID, "pass cost: %u passes of a %zu-kernel program", P,
                        a->kernels->launch_of.size());
    } else if (a->sink == nullptr || a->groups < 1 || a->groups > 65535) {
        return fail(BL_ERR_INVALID, "pass cost: the trivial kernel needs a sink and 1..65535 groups");
    }
    cudaStream_t s = static_cast<cudaStream_t>(a->stream);
    const bool graph_form = a->variant == BL_PASS_ONE_PASS || a->variant == BL_PASS_ONE_PASS_PDL;
    auto launch = [&](uint32_t i, cudaStream_t st) -> int {
        if (a->kernels != nullptr) return enqueue(a->kernels->at(i, 0), st);
        if (a->variant == BL_PASS_ONE_PASS_PDL) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(a->groups);
            cfg.blockDim = dim3(1);
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            const cudaError_t e = cudaLaunchKernelEx(&cfg, pass_cost_kernel_pdl, a->sink);
            return e == cudaSuccess ? BL_OK : fail(BL_ERR_CUDA, "pass cost: %s", cudaGetErrorString(e));
        }
        pass_cost_kernel<<<a->groups, 1, 0, st>>>(a->sink);
        const cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? BL_OK : fail(BL_ERR_CUDA, "pass cost: %s", cudaGetErrorString(e));
    };
    // which passes carry a pair: every one (A), the first's begin and the
    // last's end (B), every k-th and the last (D); C has one pair around the graph
    auto timed = [&](uint32_t i) {
        return a->variant == BL_PASS_PER_PASS ||
               (a->variant == BL_PASS_EVERY && (i % a->every == 0 || i == P - 1));
    };
    EventSet ev;
    ev.ev.resize(2 * static_cast<size_t>(P));
    for (cudaEvent_t& e : ev.ev) BL_CUDA_TRY(cudaEventCreate(&e));
    cudaEvent_t* b = ev.ev.data();
    cudaEvent_t* en = ev.ev.data() + P;

    const auto t0 = std::chrono::steady_clock::now();
    uint32_t pairs = 0;
    int rc = BL_OK;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaStream_t cap = nullptr;
    if (graph_form) {
        BL_CUDA_TRY(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
        cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeRelaxed);
        for (uint32_t i = 0; i < P && rc == BL_OK && e == cudaSuccess; ++i) rc = launch(i, cap);
        const cudaError_t e2 = cudaStreamEndCapture(cap, &graph);
        if (e == cudaSuccess) e = e2;
        if (rc == BL_OK && e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
        if (rc == BL_OK && e == cudaSuccess) e = cudaEventRecord(b[0], s);
        if (rc == BL_OK && e == cudaSuccess) e = cudaGraphLaunch(exec, s);
        if (rc == BL_OK && e == cudaSuccess) e = cudaEventRecord(en[0], s);
        if (rc == BL_OK && e != cudaSuccess) rc = fail(BL_ERR_CUDA, "pass cost graph: %s", cudaGetErrorString(e));
        pairs = 1;
    } else {
        for (uint32_t i = 0; i < P && rc == BL_OK; ++i) {
            const bool pair = timed(i);
            if (pair || (a->variant == BL_PASS_ENDS && i == 0)) BL_CUDA_TRY(cudaEventRecord(b[i], s));
            rc = launch(i, s);
            if (rc == BL_OK && (pair || (a->variant == BL_PASS_ENDS && i == P - 1)))
                BL_CUDA_TRY(cudaEventRecord(en[i], s));
            pairs += pair ? 1 : 0;
        }
        if (a->variant == BL_PASS_ENDS) pairs = 1;
    }
    const auto t1 = std::chrono::steady_clock::now();
    const cudaError_t es = cudaStreamSynchronize(s);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (cap) cudaStreamDestroy(cap);
    if (rc != BL_OK) return rc;
    if (es != cudaSuccess) return fail(BL_ERR_CUDA, "pass cost: %s", cudaGetErrorString(es));

    float ms = 0.0f;
    const uint32_t last = graph_form ? 0 : P - 1;
    BL_CUDA_TRY(cudaEventElapsedTime(&ms, b[0], en[last]));
    out->span_us = 1000.0 * ms;
    double sum = 0.0;
    if (a->variant == BL_PASS_PER_PASS || a->variant == BL_PASS_EVERY) {
        for (uint32_t i = 0; i < P; ++i) {
            if (!timed(i)) continue;
            BL_CUDA_TRY(cudaEventElapsedTime(&ms, b[i], en[i]));
            sum += 1000.0 * ms;
        }
    } else {
        sum = out->span_us;
    }
    out->passes_us = sum;
    out->pairs = pairs;
    out->encode_us = std::chrono::duration<double, std::micro>(t1 - t0).count();
    return BL_OK;
}
