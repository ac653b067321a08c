/*
 * A stand-in for libnccl.so.2 for the CPU tests of the communicator's
 * failure handling (tests/test_comm.py): the entry points bl_comm_* loads,
 * with NCCL's non-blocking semantics (calls return ncclInProgress, progress is
 * read with ncclCommGetAsyncError), over ranks that are host processes
 * meeting through files in the directory $FAKE_NCCL_DIR. No GPU is touched:
 * buffers are host memory and the stream argument is ignored.
 *
 *   join:        <token>.join.<rank>      written by ncclCommInitRankConfig
 *   all-gather:  <token>.ag<seq>.<rank>   this rank's bytes of operation seq
 *   abort:       <token>.abort.<rank>     written by ncclCommAbort
 *   destroy:     <token>.destroy.<rank>   written by ncclCommDestroy
 *
 * $FAKE_NCCL_ASYNC_ERROR=<n>: ncclCommGetAsyncError reports result n once the
 * communicator has joined (a peer failing after set-up).
 * The fake refuses a blocking communicator (config->blocking != 0).
 * Test infrastructure only; built by the tests with gcc.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef enum {
    ncclSuccess = 0, ncclUnhandledCudaError = 1, ncclSystemError = 2, ncclInternalError = 3,
    ncclInvalidArgument = 4, ncclInvalidUsage = 5, ncclRemoteError = 6, ncclInProgress = 7
} ncclResult_t;
typedef struct { char internal[128]; } ncclUniqueId;
typedef struct {
    size_t size;
    unsigned int magic;
    unsigned int version;
    int blocking;
} ncclConfig_t;  /* the leading fields of NCCL's versioned config */

enum { IDLE = 0, JOINING = 1, GATHERING = 2 };
typedef struct fake_comm {
    int nranks, rank, state, seq;
    char token[112];
    unsigned char* recv;
    size_t bytes;
} fake_comm;
typedef fake_comm* ncclComm_t;

static void path(char* out, size_t cap, const fake_comm* c, const char* what, int seq, int rank) {
    const char* dir = getenv("FAKE_NCCL_DIR");
    if (seq >= 0)
        snprintf(out, cap, "%s/%s.%s%d.%d", dir ? dir : ".", c->token, what, seq, rank);
    else
        snprintf(out, cap, "%s/%s.%s.%d", dir ? dir : ".", c->token, what, rank);
}

static int touch(const char* p, const void* data, size_t n) {
    char tmp[600];
    snprintf(tmp, sizeof tmp, "%s.tmp%d", p, (int)getpid());
    FILE* f = fopen(tmp, "wb");
    if (!f) return -1;
    if (n && fwrite(data, 1, n, f) != n) { fclose(f); return -1; }
    fclose(f);
    return rename(tmp, p);
}

static int exists(const char* p) { return access(p, F_OK) == 0; }

const char* ncclGetErrorString(ncclResult_t r) {
    switch (r) {
        case ncclSuccess: return "no error (fake)";
        case ncclInProgress: return "operation in progress (fake)";
        case ncclInvalidUsage: return "invalid usage (fake)";
        case ncclInternalError: return "internal error (fake)";
        case ncclRemoteError: return "remote process exited or there was a network error (fake)";
        default: return "error (fake)";
    }
}

ncclResult_t ncclGetUniqueId(ncclUniqueId* id) {
    static int n = 0;
    memset(id, 0, sizeof *id);
    snprintf(id->internal, sizeof id->internal, "fake%d_%d", (int)getpid(), n++);
    return ncclSuccess;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank,
                                    ncclConfig_t* config) {
    if (config == NULL || config->blocking != 0) return ncclInvalidUsage;
    if (nranks < 1 || rank < 0 || rank >= nranks) return ncclInvalidArgument;
    fake_comm* c = calloc(1, sizeof *c);
    c->nranks = nranks;
    c->rank = rank;
    c->state = JOINING;
    memcpy(c->token, id.internal, sizeof c->token - 1);
    char p[600];
    path(p, sizeof p, c, "join", -1, rank);
    if (touch(p, NULL, 0) != 0) { free(c); return ncclSystemError; }
    *comm = c;
    return ncclInProgress;
}

ncclResult_t ncclCommGetAsyncError(ncclComm_t c, ncclResult_t* err) {
    char p[600];
    if (c->state == JOINING) {
        for (int r = 0; r < c->nranks; ++r) {
            path(p, sizeof p, c, "join", -1, r);
            if (!exists(p)) { *err = ncclInProgress; return ncclSuccess; }
        }
        c->state = IDLE;
    } else if (c->state == GATHERING) {
        for (int r = 0; r < c->nranks; ++r) {
            path(p, sizeof p, c, "ag", c->seq, r);
            if (!exists(p)) { *err = ncclInProgress; return ncclSuccess; }
        }
        for (int r = 0; r < c->nranks; ++r) {
            path(p, sizeof p, c, "ag", c->seq, r);
            FILE* f = fopen(p, "rb");
            if (!f || fread(c->recv + r * c->bytes, 1, c->bytes, f) != c->bytes) {
                if (f) fclose(f);
                *err = ncclSystemError;
                return ncclSuccess;
            }
            fclose(f);
        }
        c->seq += 1;
        c->state = IDLE;
    }
    const char* e = getenv("FAKE_NCCL_ASYNC_ERROR");
    *err = e ? (ncclResult_t)atoi(e) : ncclSuccess;
    return ncclSuccess;
}

ncclResult_t ncclAllGather(const void* send, void* recv, size_t count, int datatype,
                           ncclComm_t c, void* stream) {
    (void)stream;
    if (datatype != 0 /* ncclInt8 / ncclChar */ && datatype != 1 /* ncclUint8 */)
        return ncclInvalidArgument;
    if (c->state != IDLE) return ncclInvalidUsage;
    char p[600];
    path(p, sizeof p, c, "ag", c->seq, c->rank);
    if (touch(p, send, count) != 0) return ncclSystemError;
    c->recv = recv;
    c->bytes = count;
    c->state = GATHERING;
    return ncclInProgress;
}

ncclResult_t ncclCommAbort(ncclComm_t c) {
    char p[600];
    path(p, sizeof p, c, "abort", -1, c->rank);
    touch(p, NULL, 0);
    free(c);
    return ncclSuccess;
}

ncclResult_t ncclCommFinalize(ncclComm_t c) {
    (void)c;
    return ncclSuccess;
}

ncclResult_t ncclCommDestroy(ncclComm_t c) {
    char p[600];
    path(p, sizeof p, c, "destroy", -1, c->rank);
    touch(p, NULL, 0);
    free(c);
    return ncclSuccess;
}
