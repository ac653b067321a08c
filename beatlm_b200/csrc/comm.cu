// The communicator of the multi-GPU configs: NCCL created non-blocking, every
// call bounded by a host timeout, and aborted when the timeout runs out, so a
// rank that never joins or stops answering ends the others' waits with an
// error instead of a hang. The reference runs on one device and has no
// counterpart; NCCL's all-gather is the plain collective form of the
// long-sequence attention's exchange (the fused form is bl_attention_peers).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or the library named by
// BEATLM_B200_NCCL), never linked: the backend loads where NCCL is absent and
// bl_comm_* then report BL_ERR_UNSUPPORTED. A process that already loaded
// NCCL (through torch, say) gets that same library back from dlopen.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

#include "host.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    char why[256] = "";
};

NcclApi g_api;
std::once_flag g_api_once;

const NcclApi& api() {
    std::call_once(g_api_once, [] {
        const char* name = getenv("BEATLM_B200_NCCL");
        if (name == nullptr || name[0] == '\0') name = "libnccl.so.2";
        void* h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
        if (h == nullptr) {
            snprintf(g_api.why, sizeof g_api.why, "NCCL is not loadable (%s): %s", name, dlerror());
            return;
        }
        auto sym = [&](const char* s) { return dlsym(h, s); };
        g_api.get_unique_id = reinterpret_cast<decltype(g_api.get_unique_id)>(sym("ncclGetUniqueId"));
        g_api.init_rank_config =
            reinterpret_cast<decltype(g_api.init_rank_config)>(sym("ncclCommInitRankConfig"));
        g_api.get_async_error =
            reinterpret_cast<decltype(g_api.get_async_error)>(sym("ncclCommGetAsyncError"));
        g_api.abort = reinterpret_cast<decltype(g_api.abort)>(sym("ncclCommAbort"));
        g_api.finalize = reinterpret_cast<decltype(g_api.finalize)>(sym("ncclCommFinalize"));
        g_api.destroy = reinterpret_cast<decltype(g_api.destroy)>(sym("ncclCommDestroy"));
        g_api.all_gather = reinterpret_cast<decltype(g_api.all_gather)>(sym("ncclAllGather"));
        g_api.error_string = reinterpret_cast<decltype(g_api.error_string)>(sym("ncclGetErrorString"));
        g_api.ok = g_api.get_unique_id && g_api.init_rank_config && g_api.get_async_error &&
                   g_api.abort && g_api.finalize && g_api.destroy && g_api.all_gather &&
                   g_api.error_string;
        if (!g_api.ok) snprintf(g_api.why, sizeof g_api.why, "%s lacks an NCCL entry point", name);
    });
    return g_api;
}

const char* nccl_error(ncclResult_t r) {
    const NcclApi& a = api();
    return a.ok ? a.error_string(r) : "NCCL unavailable";
}

}  // namespace

struct bl_comm {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 0;
    uint32_t timeout_ms = 0;
    bool aborted = false;
};

namespace {

// Polls the communicator's asynchronous state until it leaves
// ncclInProgress or `timeout_ms` of host time pass; on expiry, or on an
// error, the communicator is aborted (ncclCommAbort) and unusable.
int settle(bl_comm* c, const char* what) {
    using namespace bl;
    const NcclApi& a = api();
    const auto t0 = std::chrono::steady_clock::now();
    for (uint32_t spin = 0;; ++spin) {
        ncclResult_t st = ncclInProgress;
        ncclResult_t q = a.get_async_error(c->comm, &st);
        if (q != ncclSuccess) st = q;
        if (st == ncclSuccess) return BL_OK;
        if (st != ncclInProgress) {
            a.abort(c->comm);
            c->aborted = true;
            return fail(BL_ERR_COMM, "comm: %s failed: %s (communicator aborted)", what,
                        nccl_error(st));
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
        if (ms >= static_cast<long long>(c->timeout_ms)) {
            a.abort(c->comm);
            c->aborted = true;
            return fail(BL_ERR_TIMEOUT, "comm: %s still in progress after %u ms (communicator "
                                        "aborted)", what, c->timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(spin < 100 ? 20 : 500));
    }
}

}  // namespace

extern "C" int bl_comm_available(void) { return api().ok ? 1 : 0; }

extern "C" int bl_comm_unique_id(void* id) {
    using namespace bl;
    if (id == nullptr) return fail(BL_ERR_INVALID, "comm: null id");
    const NcclApi& a = api();
    if (!a.ok) return fail(BL_ERR_UNSUPPORTED, "comm: %s", a.why);
    ncclUniqueId u;
    const ncclResult_t r = a.get_unique_id(&u);
    if (r != ncclSuccess) return fail(BL_ERR_COMM, "comm: ncclGetUniqueId: %s", nccl_error(r));
    memcpy(id, &u, sizeof u);
    return BL_OK;
}

extern "C" int bl_comm_init(const void* id, uint32_t world, uint32_t rank, uint32_t timeout_ms,
                            bl_comm** out) {
    using namespace bl;
    static_assert(sizeof(ncclUniqueId) == BL_COMM_ID_BYTES, "NCCL unique id size");
    if (id == nullptr || out == nullptr) return fail(BL_ERR_INVALID, "comm: null argument");
    if (world < 1 || rank >= world) return fail(BL_ERR_INVALID, "comm: rank %u of %u", rank, world);
    if (timeout_ms == 0) return fail(BL_ERR_INVALID, "comm: a timeout of 0 ms");
    const NcclApi& a = api();
    if (!a.ok) return fail(BL_ERR_UNSUPPORTED, "comm: %s", a.why);
    bl_comm* c = new bl_comm();
    c->rank = static_cast<int>(rank);
    c->world = static_cast<int>(world);
    c->timeout_ms = timeout_ms;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every call returns at once; progress is polled
    const ncclResult_t r = a.init_rank_config(&c->comm, c->world, u, c->rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        if (c->comm) a.abort(c->comm);
        delete c;
        return fail(BL_ERR_COMM, "comm: ncclCommInitRankConfig: %s", nccl_error(r));
    }
    const int rc = settle(c, "init");
    if (rc != BL_OK) {
        delete c;  // aborted by settle
        return rc;
    }
    *out = c;
    return BL_OK;
}

extern "C" int bl_comm_all_gather(bl_comm* c, const void* send, void* recv, uint64_t bytes,
                                  void* stream) {
    using namespace bl;
    if (c == nullptr || send == nullptr || recv == nullptr)
        return fail(BL_ERR_INVALID, "comm: null argument");
    if (c->aborted) return fail(BL_ERR_COMM, "comm: the communicator was aborted");
    const NcclApi& a = api();
    const ncclResult_t r = a.all_gather(send, recv, bytes, ncclUint8, c->comm,
                                        static_cast<cudaStream_t>(stream));
    if (r != ncclSuccess && r != ncclInProgress) {
        a.abort(c->comm);
        c->aborted = true;
        return fail(BL_ERR_COMM, "comm: ncclAllGather: %s (communicator aborted)", nccl_error(r));
    }
    // the enqueue completes in the background on a non-blocking communicator
    return r == ncclInProgress ? settle(c, "all-gather") : BL_OK;
}

extern "C" int bl_comm_check(bl_comm* c) {
    using namespace bl;
    if (c == nullptr) return fail(BL_ERR_INVALID, "comm: null communicator");
    if (c->aborted) return fail(BL_ERR_COMM, "comm: the communicator was aborted");
    return settle(c, "pending operations");
}

extern "C" int bl_comm_abort(bl_comm* c) {
    using namespace bl;
    if (c == nullptr) return fail(BL_ERR_INVALID, "comm: null communicator");
    if (!c->aborted) {
        api().abort(c->comm);
        c->aborted = true;
    }
    return BL_OK;
}

extern "C" int bl_comm_aborted(const bl_comm* c) { return c != nullptr && c->aborted ? 1 : 0; }

extern "C" int bl_comm_destroy(bl_comm* c) {
    using namespace bl;
    if (c == nullptr) return BL_OK;
    int rc = BL_OK;
    const NcclApi& a = api();
    if (!c->aborted) {
        // finalize flushes what was issued; bounded like everything else
        ncclResult_t r = a.finalize(c->comm);
        if (r == ncclSuccess || r == ncclInProgress) {
            rc = settle(c, "finalize");
            if (rc == BL_OK) a.destroy(c->comm);
        } else {
            a.abort(c->comm);
            rc = fail(BL_ERR_COMM, "comm: ncclCommFinalize: %s (communicator aborted)",
                      nccl_error(r));
        }
    }
    delete c;
    return rc;
}
