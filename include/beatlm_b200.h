/*
 * beatlm-b200: the C ABI of the B200 (sm_100a) backend for beatlm's ViT
 * attention hot path.
 *
 * Plain C: opaque handles, POD structs, plain pointers and sizes, an int
 * status (0 = ok) and a thread-local message behind bl_last_error(). Device
 * pointers are CUDA device addresses; `stream` is a cudaStream_t passed as
 * void* (NULL = the legacy default stream). No call allocates device memory
 * except where it says so.
 *
 * The reference (ynishi/beatlm) is Rust with `unsafe_code = "forbid"`
 * (Cargo.toml:55-57), so it has no FFI of its own; each entry point below
 * names the reference interface (file:line, crate-relative) whose role it
 * takes on this path.
 */
#ifndef BEATLM_B200_H
#define BEATLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ errors */

enum {
    BL_OK = 0,
    BL_ERR_INVALID = 1,     /* malformed arguments (reference: KernelError, kernel.rs:2454) */
    BL_ERR_UNSUPPORTED = 2, /* a shape or type this build does not implement */
    BL_ERR_CUDA = 3,        /* a CUDA runtime or driver call failed */
    BL_ERR_DEVICE = 4,      /* a kernel recorded an error in the device status word */
    BL_ERR_CAPACITY = 5,    /* a plan or buffer does not fit (reference: PlanError, memory.rs:220) */
    BL_ERR_COMM = 6,        /* a communicator call failed (the communicator is then aborted) */
    BL_ERR_TIMEOUT = 7      /* a communicator call did not complete within its timeout (aborted) */
};

/* Copies the calling thread's last error message (NUL-terminated, truncated
 * to cap) and returns its full length. */
size_t bl_last_error(char* buf, size_t cap);

/* Build identification, e.g. "beatlm-b200 0.1 sm_100a". */
const char* bl_version(void);

/* The device status word the kernels write instead of trapping: a wait that
 * ran out of time (about 1 s) records a code and the kernel unwinds. */
typedef struct bl_status_t {
    uint32_t code;  /* 0 = no error; 0x10.. = timeout by role; 0x50 = bad arguments */
    uint32_t block; /* linear index of the first block that recorded it */
    uint32_t where; /* role-specific position */
    uint32_t count; /* error events recorded */
} bl_status_t;

/* Synchronises the current device, copies its status word to *out and, when
 * reset != 0, clears it. */
int bl_status(bl_status_t* out, int reset);

/* How long a kernel's wait may spin before it gives up, records a timeout
 * code and unwinds: `cycles` SM clock cycles on the current device (0 = the
 * default of 1965e6, about 1 s; at most 60 s worth). It applies to launches
 * made after the call; bl_status resets leave it alone. No counterpart in
 * the reference, whose queue has no device-side waits: it lets a host (or a
 * test) bound a stalled exchange, such as a peer that never signals, tightly. */
int bl_set_wait_limit(uint64_t cycles);
/* The current device's wait limit as set (0 = the default). */
uint64_t bl_wait_limit(void);

/* ------------------------------------------------------------------ types */

typedef enum bl_dtype { BL_F32 = 0, BL_F16 = 1, BL_BF16 = 2 } bl_dtype;

/* ------------------------------------------------------------------ attention */

/*
 * The fused non-causal attention of one ViT layer: the reference's
 * AttentionScores -> Scale(1/sqrt(head_dim)) -> Softmax -> AttentionValues
 * chain (crates/beatlm-core/src/kernel.rs:722-777, built at
 * crates/beatlm/src/model/depth_anything_v2.rs:341-367, dispatched through
 * Kernels::encode at crates/beatlm/src/codegen/kernels.rs:217) as one kernel
 * with an online softmax; no scores tensor exists.
 *
 * Layouts are the reference's (kernel.rs:157-161): qkv is packed per token,
 * [batch][tokens][3][heads][head_dim] with `qkv_row_stride` elements between
 * tokens; the result is [batch][tokens][heads * head_dim] (heads side by
 * side), each token `out_row_stride` elements apart, head h at column
 * (h - out_head_base) * head_dim.
 *
 * Element types: Q and K are `qk_dtype` (BL_F16 or BL_BF16), V is BL_F16
 * (the probabilities multiply V in f16, whose 11-bit significand keeps the
 * result within the relative-L2 1e-3 bound; bf16 probabilities would not);
 * the Q/K/V sections of one packed row may hold different types. Scores,
 * softmax statistics and the accumulator are f32.
 *
 * A call computes query rows [row_begin, row_end) and heads
 * [head_begin, head_end): a row part in the sense of Program::split
 * (kernel.rs:2384) and a head slab for head-parallel runs. head_dim must be
 * 64. qkv and out must be 16-byte aligned and their row strides multiples of
 * 8 elements (16 bytes). Enqueues on `stream`; allocates nothing.
 *
 * Key splits: when the query tiles alone would leave SMs idle (ViT-S at one
 * frame: 36 CTAs for 148 SMs), the keys are split across CTAs and their
 * partial results combined. kv_splits = 0 picks the split count, 1 never
 * splits. Without a workspace the CTAs of one query group form a
 * thread-block cluster (at most 8 splits) and combine in distributed shared
 * memory. With a workspace the partials go through it and the last CTA of
 * each group combines them: a caller-owned device buffer of
 * bl_attention_workspace_bytes() bytes, 256-byte aligned, zero-filled once
 * before its first use (every call leaves its counters at zero again; calls
 * that overlap on the GPU must not share one); too small a workspace is
 * BL_ERR_CAPACITY. Both combines give the same result.
 */
typedef struct bl_attention_args {
    uint32_t batch;
    uint32_t tokens;
    uint32_t heads;
    uint32_t head_dim;
    uint32_t head_begin, head_end;
    uint32_t row_begin, row_end;
    float scale;
    int32_t qk_dtype;
    int32_t v_dtype;
    int32_t out_dtype;
    const void* qkv;
    uint64_t qkv_row_stride; /* 0 = 3 * heads * head_dim */
    void* out;
    uint64_t out_row_stride; /* 0 = heads * head_dim */
    uint32_t out_head_base;
    uint32_t kv_splits;      /* 0 = automatic (with query_tiles), 1 = none */
    void* workspace;
    uint64_t workspace_bytes;
    /* Optional per-CTA timeline (NULL = off): CTA b writes %globaltimer
     * stamps (ns) at trace[8b..8b+7]: entry, setup done, tile 0 softmax done,
     * tile 1 softmax done, partials stored (cluster combine), cluster barrier
     * passed, combine done (bl_attention_peers: rows stored), exit (slots a
     * path does not reach stay as they were). CTAs are numbered x-fastest over the grid (query groups, heads,
     * batch x splits); the buffer holds 8 * CTAs uint64 values. */
    uint64_t* trace;
    /* 128-row query tiles per CTA: 2 (a CTA of 12 warps, two softmax
     * warpgroups), 1 (8 warps, one softmax warpgroup: twice the CTAs, for
     * launches too small to fill the GPU), or 0 = automatic. With kv_splits
     * also 0 the pair with the least estimated time is taken. Every row's
     * result depends on the key splits only, never on this choice. */
    uint32_t query_tiles;
} bl_attention_args;

int bl_attention(const bl_attention_args* args, void* stream);

/* Workspace bytes bl_attention needs for these arguments (0: no split). */
uint64_t bl_attention_workspace_bytes(const bl_attention_args* args);

/* The query tiles per CTA and key splits bl_attention takes for these
 * arguments (its automatic choice for fields left 0; with args->workspace
 * NULL the cluster combine, else the workspace combine within
 * args->workspace_bytes). Queries the current device's cluster occupancy.
 * With kv_splits left 0 and no workspace the launch may be a mixed grid:
 * *unsplit_groups query groups (128 x query_tiles rows of one head), as many
 * as fill whole waves of clusters, run unsplit and the remaining groups are
 * split kv_splits ways, so the last wave is short; 0 = every group split
 * kv_splits ways. Rows of the unsplit groups are computed as with
 * kv_splits = 1, the others as with kv_splits = *kv_splits. */
int bl_attention_choice(const bl_attention_args* args, uint32_t* query_tiles,
                        uint32_t* kv_splits, uint32_t* unsplit_groups);

/*
 * bl_attention for callers that cannot allocate device memory. No counterpart
 * in the reference: it exists for hosts whose device memory is fixed up front
 * (a static memory plan realised once, nothing allocated in the frame loop),
 * for host runtimes reaching this library through an FFI without a CUDA
 * allocator of their own, and for code that must not allocate while it runs.
 * Such a caller cannot provide the split-key workspace, so this entry point
 * keeps that scratch in a 16 MiB array inside the library (every GPU that
 * loads the library holds it until the process exits) and allocates nothing:
 * no cudaMalloc, no cudaFree, no allocating library routine.
 *
 * args->workspace and args->workspace_bytes are ignored. kv_splits = 0 picks
 * the split count that fits the 16 MiB; an explicit count whose scratch would
 * exceed 16 MiB is rejected with BL_ERR_CAPACITY. The first call on each
 * device looks up the array's device address (once, with that device
 * current), so make that first call before any stream capture. After a
 * device reset (cudaDeviceReset) the device has a new context and the next
 * call looks the address up again, so that call too belongs outside a
 * capture. Each call
 * clears the split counters on `stream` before its launch. All calls share the
 * one array: calls that overlap on the GPU race and must not be issued.
 */
int bl_attention_noalloc(const bl_attention_args* args, void* stream);

/* ------------------------------------------------- head-parallel exchange */

/*
 * The long-sequence attention split by heads over the GPUs of one node, with
 * the exchange of head outputs fused into the attention kernel. The
 * reference runs on one device (queue order is its only synchronisation,
 * crates/beatlm-core/src/lib.rs:30-41); this takes the place of its
 * AttentionScores -> Softmax -> AttentionValues chain for the heads of one
 * rank plus the all-gather that assembles the [tokens][heads * 64] output
 * (kernel.rs:157-161) on every rank.
 *
 * Each rank owns a peer buffer: a 256-byte header of arrival flags (rank r's
 * flag is the 32-bit word at byte 4 r) and two output slots of slot_bytes each
 * (slot s at byte 256 + s * slot_bytes rounded up to 256), in one device
 * allocation made at create (the only allocation). The ranks exchange
 * 64-byte CUDA IPC handles of their
 * buffers by any host channel (bl_peers_handle on each, then bl_peers_open
 * with all of them in rank order), or a host that maps a rank's buffer
 * itself (another device of the same process with peer access, or a test)
 * hands it over with bl_peers_attach: the buffer must then be
 * bl_peers_buffer_bytes(slot_bytes) bytes, 256-byte aligned and zero-filled
 * once. Every rank needs every rank's buffer before its first launch.
 */
enum { BL_PEER_HANDLE_BYTES = 64, BL_MAX_PEERS = 8 };
typedef struct bl_peers bl_peers;
uint64_t bl_peers_buffer_bytes(uint64_t slot_bytes);
int bl_peers_create(uint32_t rank, uint32_t world, uint64_t slot_bytes, bl_peers** out);
int bl_peers_handle(const bl_peers* p, void* handle /* BL_PEER_HANDLE_BYTES */);
int bl_peers_open(bl_peers* p, const void* handles /* world x BL_PEER_HANDLE_BYTES */, size_t n);
int bl_peers_attach(bl_peers* p, uint32_t rank, void* buffer);
/* This rank's output slot 0 or 1 (device memory, slot_bytes long). */
void* bl_peers_slot(const bl_peers* p, uint32_t slot);
/* The flag value the next bl_attention_peers launch raises (launches count
 * from 1; a launch uses slot epoch % 2). */
uint32_t bl_peers_next_epoch(const bl_peers* p);
/* Unmaps the other ranks' buffers and frees this one's. Every rank's
 * launches must have completed first (synchronise, then a host barrier). */
void bl_peers_destroy(bl_peers* p);

/*
 * bl_attention of this rank's heads whose output rows the kernel stores
 * into EVERY rank's current output slot (16-bit rows, out_row_stride
 * elements apart; this rank's head h at column out_col + (h - out_head_base) *
 * 64), as soon as each row is final, so the exchange crosses NVLink while the
 * kernel still computes. args->out and args->workspace are ignored; key
 * splits combine in a thread-block cluster. The attention grid is followed
 * on `stream` by an arrival barrier, a one-warp kernel that starts once the
 * grid has completed (so its row stores are performed), raises this rank's
 * flag in every rank's header and waits until every rank's flag for this
 * launch has arrived in its own: when it completes, the whole output is in
 * this rank's slot (*slot_out). The wait is bounded (bl_set_wait_limit); a
 * rank that never launches makes the others record status 0x60 (peer
 * timeout) and return with their output incomplete. Every rank must make
 * the same sequence of calls. A slot is written again two launches later:
 * read a launch's output on the launching stream before the launch after
 * next. Enqueues on `stream`; allocates nothing.
 */
int bl_attention_peers(const bl_attention_args* args, bl_peers* peers, uint32_t out_col,
                       uint32_t* slot_out, void* stream);

/* ------------------------------------------------------------ communicator */

/*
 * NCCL for the multi-GPU configs, created non-blocking and never waited on
 * without a bound. The reference runs on one device (no collectives); this
 * is the collective form of the long-sequence attention's exchange (an
 * all-gather of head slabs) and a host's way to run collectives without
 * another runtime. NCCL is loaded at run time (libnccl.so.2, or the library
 * the environment variable BEATLM_B200_NCCL names); where it cannot be
 * loaded bl_comm_available() is 0 and the calls return BL_ERR_UNSUPPORTED.
 *
 * Every call that waits (init, a collective's enqueue, check, destroy) polls
 * ncclCommGetAsyncError for at most the communicator's timeout; when the
 * timeout runs out (a rank that never joins, a peer that stopped) or NCCL
 * reports an error, the communicator is aborted (ncclCommAbort) and the call
 * returns BL_ERR_TIMEOUT or BL_ERR_COMM. An aborted communicator refuses
 * further work; destroy it. Collectives are enqueued on `stream` and complete
 * there; every rank must issue the same collectives in the same order.
 */
enum { BL_COMM_ID_BYTES = 128 };
typedef struct bl_comm bl_comm;
int bl_comm_available(void);
/* A new unique id (ncclGetUniqueId), made by one rank and shared with the
 * others by any host channel. */
int bl_comm_unique_id(void* id /* BL_COMM_ID_BYTES */);
/* Joins rank `rank` of `world` (ncclCommInitRankConfig, blocking = 0) on the
 * current device, waiting at most timeout_ms for the others. */
int bl_comm_init(const void* id, uint32_t world, uint32_t rank, uint32_t timeout_ms,
                 bl_comm** out);
/* recv[r * bytes .. (r + 1) * bytes) = rank r's send (ncclAllGather). */
int bl_comm_all_gather(bl_comm* c, const void* send, void* recv, uint64_t bytes, void* stream);
/* Waits (bounded) until the communicator has no operation whose enqueue is
 * still in progress and reports its asynchronous error state. */
int bl_comm_check(bl_comm* c);
int bl_comm_abort(bl_comm* c);
int bl_comm_aborted(const bl_comm* c);
/* Finalizes (bounded) and destroys; an aborted communicator is only freed. */
int bl_comm_destroy(bl_comm* c);

/* ------------------------------------------------------------------ linear */

enum { BL_ACT_NONE = 0, BL_ACT_RELU = 1, BL_ACT_GELU_TANH = 2, BL_ACT_GELU_ERF = 3 };

/*
 * A linear layer with the reference's fusions, on the tensor cores:
 *   out = epilogue(A . W^T)   A [m][k], W [n][k] (out x in), f32 accumulate.
 * Replaces the MatMul kernel with its fused epilogue chain
 * (kernel.rs:781-794 MatMul, 1595-1615 Epilogue; WGSL tiled/matmul at
 * crates/beatlm/src/codegen/wgsl.rs:744-932, epilogue hook 297-326), and adds
 * the LayerNorm prologue of the QKV and fc1 projections.
 *
 * A: a 16-bit activation `a` (row stride lda), or, when ln_x != NULL,
 * LayerNorm(ln_x) computed inside the kernel from the f32 rows ln_x (stride
 * ln_ldx) with ln_gamma/ln_beta [k] and ln_eps (reference.rs:247-270), so the
 * normalised rows never reach memory. A and W are `ab_dtype` (f16 or bf16).
 *
 * Epilogue, in this order: + bias[n]; act; * scale (0 or 1 = none);
 * * chan_scale[n] (LayerScale, the reference's ChannelScale); + residual
 * (res_dtype, row stride res_ld, row index out_row % res_period when
 * res_period > 0). Stored as out_dtype, or as out_dtype_hi from column
 * split_col on (0 < split_col < n; used for packed Q|K|V rows with f16 V).
 * Output row of A-row r: r + (r / out_group_rows) * out_group_gap +
 * out_row_offset (out_group_rows = 0: r + out_row_offset), which places the
 * patch tokens of a frame after its class token.
 *
 * k must be a multiple of 64 and n a multiple of the tile width (32, 64, 96,
 * 128, or 256 with A given as `a`; tile_n = 0 chooses from a per-CTA cost
 * estimate). Pointers 16-byte aligned, row strides 16-byte
 * multiples. Enqueues on `stream`; allocates nothing.
 */
typedef struct bl_gemm_args {
    uint32_t m, n, k;
    int32_t ab_dtype;
    const void* a;
    uint64_t lda;
    const void* b;
    uint64_t ldb;
    const float* ln_x;
    uint64_t ln_ldx;
    const float* ln_gamma;
    const float* ln_beta;
    float ln_eps;
    const float* bias;
    int32_t act;
    float scale;
    const float* chan_scale;
    const void* residual;
    int32_t res_dtype;
    uint64_t res_ld;
    uint32_t res_period;
    void* out;
    int32_t out_dtype;
    uint64_t out_ld;
    uint32_t split_col;
    int32_t out_dtype_hi;
    uint32_t out_row_offset, out_group_rows, out_group_gap;
    uint32_t tile_n;
    /* Row statistics for a LayerNorm that follows (optional; f32 outputs
     * only). The epilogue also writes, for every output row and each of
     * `stats_parts` equal column slices (n / stats_parts columns, which is then
     * the kernel's tile width), the slice's mean and sum of squared deviations
     * of the stored values: float2 [out row][part]. */
    void* stats_out;
    uint32_t stats_parts;
    /* LayerNorm prologue only: take each row's mean and variance from such
     * partial statistics of ln_x (ln_stats_parts equal slices of the k
     * columns, combined by Chan's formula) instead of a pass over the row. */
    const void* ln_stats;
    uint32_t ln_stats_parts;
    /* LayerNorm of the stored rows in the epilogue (optional; no counterpart
     * in the reference, which runs its LayerNorm op, kernel.rs:644-659, as a
     * pass of its own): with norm_out set, every output row is also
     * normalised over its n stored f32 values (biased variance, then
     * norm_gamma / norm_beta, eps norm_eps) and written to norm_out (f16 or
     * bf16, row stride norm_out_ld elements; row r of the product lands in
     * row r). The 32-column tiles of a 128-row tile exchange partial
     * (mean, M2) statistics through norm_sync: a zero-filled device buffer of
     * at least bl_gemm_norm_sync_bytes() bytes, 16-byte aligned, that each
     * launch leaves zero-filled again (one launch at a time per buffer).
     * Requires an f32 output of one type without row groups, n <= 512,
     * 32-column tiles (tile_n 0 or 32), and no more tiles than the device has
     * SMs; otherwise BL_ERR_UNSUPPORTED. */
    void* norm_out;
    int32_t norm_out_dtype;
    uint64_t norm_out_ld;
    const float* norm_gamma;
    const float* norm_beta;
    float norm_eps;
    void* norm_sync;
    uint64_t norm_sync_bytes;
    /* Nonzero: b, bias and chan_scale are not written by the kernel launched
     * just before this one on the stream, so they may be fetched before that
     * kernel has finished (programmatic dependent launch; a, residual and the
     * outputs always wait for it). Model weights qualify. */
    uint32_t weights_static;
    /* Optional per-CTA timeline (NULL = off) of the persistent kernel and of
     * bl_conv3x3's: CTA b writes %globaltimer stamps (ns) at trace[8b..8b+7]:
     * entry, set-up done, first A load issued (past the dependency wait),
     * first stage landed (at the MMA issuer; bl_conv3x3: at the converting
     * warps), first tile's last MMA issued (bl_conv3x3: last A tile
     * written), first tile's accumulator seen by the epilogue, last tile
     * stored, exit. 8 * grid uint64 values (the persistent grid is
     * min(tiles, SMs) CTAs; bl_conv3x3's one CTA per tile). */
    uint64_t* trace;
    /* 2: 256-row tiles computed by CTA pairs (a cluster of two CTAs, one
     * cta_group::2 MMA per step: each CTA copies its 128 rows of A and half
     * of the tile's B, so each SM brings in half the B bytes per MMA of a
     * one-CTA tile); whole launches with A given as `a`, no LayerNorm
     * prologue or epilogue LayerNorm, 128- or 256-column tiles. 0 or 1: one
     * CTA per 128-row tile. */
    uint32_t pair_tiles;
    /* 2: the K range split over a cluster of two CTAs per 64-column tile,
     * each CTA adding the other's partial sums for its half of the columns
     * (distributed shared memory) and running the epilogue on that half;
     * for A given as `a`, N a multiple of 64, no LayerNorm or statistics.
     * 0: automatic, which takes it for K >= 1024 with N <= 512 when both
     * CTAs of every 64-column tile fit one wave (a rule of the whole
     * launch's shape, so row parts compute as their whole launch). 1: off. */
    uint32_t split_k;
    /* Stream-K: every tile's k-stages cut into S pieces that are dealt to
     * the CTAs in contiguous ranges, so a launch with fewer tiles than SMs,
     * or a short last wave, keeps every SM on its k-loop. Each piece is
     * accumulated on its own; the CTA that computes a tile's last piece
     * adds the others' f32 partial sums in piece order before its epilogue,
     * so the bits depend on the shape alone (S comes from the whole
     * launch's m, n and k: row parts compute as their whole launch). The
     * partials and their flags live in `workspace`: a zero-filled device
     * buffer of at least bl_gemm_workspace_bytes() bytes, 16-byte aligned,
     * that each launch leaves zero-filled again (one launch at a time per
     * buffer). For A given as `a`, one CTA per 128- or 256-column tile, no
     * LayerNorm, epilogue LayerNorm, statistics, K split or convolution; two
     * or three pieces, by an estimate of the busiest CTA's time. 2: on; 0 or
     * 1: whole tiles. Not automatic: at the ViT-L fc2 shape (88 tiles of
     * 4096-deep K) it measured no faster than whole tiles, the full grid's
     * operand reads meeting the L2's delivery rate. */
    uint32_t stream_k;
    void* workspace;
    uint64_t workspace_bytes;
    /* Optional row reduction (NULL = off): with dot_w set (n f32 values,
     * 16-byte aligned), each finished output row v (after bias, act, scale,
     * chan_scale and residual) is reduced to one f32 value,
     * out[r] = act2(sum_c v[c] * dot_w[c] + dot_bias) summed in column order
     * (act2 = max(x, 0) when dot_act is 1, none when 0), written to `out` as
     * m contiguous f32 values in place of the row: a 1x1 convolution to one
     * channel after this GEMM's convolution (the DPT head's last two,
     * model/depth_anything_v2.rs:680-982). Requires one column tile (n at
     * most 128; tile_n 0 or n), out_dtype BL_F32 with no split column, row
     * groups or row offset, and no statistics, LayerNorm (prologue or
     * epilogue), CTA pairs, K split or stream-K; else BL_ERR_UNSUPPORTED. */
    const float* dot_w;
    float dot_bias;
    int32_t dot_act;
} bl_gemm_args;

int bl_gemm(const bl_gemm_args* args, void* stream);

/* Bytes of workspace that bl_gemm's stream-K form needs for these arguments
 * (0 where the launch does not take it: stream_k other than 2, or a form it
 * does not apply to). */
size_t bl_gemm_workspace_bytes(const bl_gemm_args* args);

/* Bytes of norm_sync that bl_gemm needs for these arguments (m and n). */
size_t bl_gemm_norm_sync_bytes(const bl_gemm_args* args);

/*
 * Standalone LayerNorm over rows of `cols` f32 values (reference.rs:247-270;
 * OpKind::LayerNorm kernel.rs:644-659, WGSL layer_norm wgsl.rs:519-585), with
 * the reference's TokensToMap (kernel.rs:703-720) folded in: input row of
 * output row r is r + (r / in_group_rows) * in_group_gap + in_row_offset
 * (in_group_rows = 0: r + in_row_offset), so the final norm can skip each
 * frame's class token. One warp per row; out is f32/f16/bf16.
 */
typedef struct bl_layernorm_args {
    uint32_t rows, cols;
    const float* x;
    uint64_t ldx;
    const float* gamma;
    const float* beta;
    float eps;
    void* out;
    int32_t out_dtype;
    uint64_t ldo;
    uint32_t in_row_offset, in_group_rows, in_group_gap;
} bl_layernorm_args;

int bl_layernorm(const bl_layernorm_args* args, void* stream);

/*
 * The embedding front of the ViT encoder for `frames` images (NHWC f32,
 * [frames][side][side][cin]): writes the patch matrix A
 * [frames * grid^2][k_pad] (16-bit `a_dtype`, patches in row-major patch
 * order, taps in (ky, kx, ci) order, zero-padded from patch^2*cin to k_pad)
 * for the patch-embedding GEMM (the reference's PatchEmbed, kernel.rs:661-687,
 * reference.rs:388-420), and the class-token rows of the residual stream x
 * [frames][grid^2 + 1][dim] (f32): x[f][0] = cls + pos[0] (PrependToken and
 * the position Add, kernel.rs:689-701).
 */
typedef struct bl_patchify_args {
    uint32_t frames, side, patch, cin, k_pad, dim;
    const float* image;
    void* a;
    int32_t a_dtype;
    const float* cls;
    const float* pos;
    float* x;
} bl_patchify_args;

int bl_patchify(const bl_patchify_args* args, void* stream);

/* ------------------------------------------------------------------ splitting */

/*
 * Program::split's rule (crates/beatlm-core/src/kernel.rs:2006-2029, rule 6 at
 * 133-149): a split dimension of `extent` units in blocks of `grain` units is
 * cut into `count` parts, clamped to 1..=ceil(extent / grain); part i covers
 * blocks [B*i/count, B*(i+1)/count), so no part is empty and none differs
 * from another by more than one block. Writes count+1 unit edges (edges[0] =
 * 0, edges[count] = extent) and returns the clamped count.
 */
uint32_t bl_split_edges(uint32_t extent, uint32_t grain, uint32_t count, uint32_t* edges);

/* KernelSpec::parts_within (kernel.rs:2048-2056): ceil(duration / bound)
 * clamped to [1, max_parts]; 0 when bound is 0 (the reference's ZeroBound). */
uint32_t bl_parts_within(uint64_t duration_us, uint64_t bound_us, uint32_t max_parts);

/* ------------------------------------------------------------------ kernels */

enum { BL_OP_ATTENTION = 1, BL_OP_GEMM = 2, BL_OP_LAYERNORM = 3, BL_OP_PATCHIFY = 4,
       BL_OP_ALLGATHER = 5 };

/* The arguments of a BL_OP_ALLGATHER kernel spec: bl_comm_all_gather encoded
 * like a kernel (recorded into a program, replayed in its CUDA graph). */
typedef struct bl_allgather_args {
    bl_comm* comm;
    const void* send;
    void* recv;
    uint64_t bytes;
} bl_allgather_args;

/* One kernel of a program: an op and its arguments (the matching bl_*_args,
 * read during bl_kernels_create only), a label, and the number of row parts
 * it runs as (0 or 1 = whole). Split dimensions and grains: attention query
 * rows in 128-row tiles (every frame of the batch), GEMM output rows in
 * 128-row tiles, LayerNorm rows one by one; patchify and all-gather are
 * never split. */
typedef struct bl_kernel_spec {
    int32_t op;
    const void* args;
    const char* label;
    uint32_t parts;
} bl_kernel_spec;

typedef struct bl_kernels bl_kernels;

/*
 * A binding set: tensors of the specs replaced by stand-ins of the same size
 * (the reference's Substitution = (TensorId, TensorId),
 * crates/beatlm/src/codegen/kernels.rs:21-26, for a host that keeps one copy
 * of an input or output per job in flight). Tensors are device ranges here:
 * every pointer argument of a spec that points into [from, from + bytes) is
 * moved to the same offset from `to`. The ranges of one set must not overlap.
 */
typedef struct bl_substitution {
    const void* from;
    void* to;
    uint64_t bytes;
} bl_substitution;
typedef struct bl_binding_set {
    const bl_substitution* subs;
    size_t n;
} bl_binding_set;

/*
 * Builds every launch of a program once: validates each spec, splits it into
 * its parts, encodes the TMA tensor maps and packs the kernel parameters
 * (Kernels::new, crates/beatlm/src/codegen/kernels.rs:63-184), for every
 * binding set: nsets = 0 means one set that binds every spec as given.
 * A kernel that touches none of a set's substituted tensors shares one
 * launch between the sets (the reference shares its bind group).
 * Afterwards encoding does no host work beyond the launch. Kernel i of the
 * result is a part; bl_kernels_len counts parts.
 */
int bl_kernels_create(const bl_kernel_spec* specs, size_t n, const bl_binding_set* sets,
                      size_t nsets, bl_kernels** out);
void bl_kernels_destroy(bl_kernels* k);
size_t bl_kernels_len(const bl_kernels* k);
/* Kernels::sets (kernels.rs:200): how many binding sets (at least 1). */
size_t bl_kernels_sets(const bl_kernels* k);
/* How many distinct launches were built (parts x sets, less the shared). */
size_t bl_kernels_launches(const bl_kernels* k);
/* The spec's label with " [i/n]" appended for a part; NULL out of range. */
const char* bl_kernels_label(const bl_kernels* k, size_t kernel);
/* KernelSpec::max_parts (crates/beatlm-core/src/kernel.rs:1975): how many
 * parts a spec's split dimension allows (attention query rows and matrix
 * multiply output rows in 128-row tiles, LayerNorm rows one by one, a patch
 * embedding 1); 0 for a NULL or unknown spec. */
uint32_t bl_kernel_spec_max_parts(const bl_kernel_spec* spec);
/* Program::parts_within (kernel.rs:2350-2366): parts_out[i] =
 * bl_parts_within(durations_us[i], bound_us, max_parts of spec i). Fails with
 * BL_ERR_INVALID when n_durations != n (PartCounts) or bound_us == 0
 * (ZeroBound). The split itself is bl_kernels_create with these counts as
 * the specs' `parts`. */
int bl_program_parts_within(const bl_kernel_spec* specs, size_t n, const uint64_t* durations_us,
                            size_t n_durations, uint64_t bound_us, uint32_t* parts_out);

typedef struct bl_timer bl_timer;

/*
 * Enqueues kernel `kernel` with binding set `set` on `stream`
 * (Kernels::encode, kernels.rs:217-233; an index past those built is
 * BL_ERR_INVALID and enqueues nothing). When `timer` is non-NULL and `frame`
 * >= 0 (a handle from bl_timer_begin_frame), the launch is bracketed by the
 * frame's next pair of cudaEvents, the compute-pass timestamp writes of the
 * reference (FrameTimestamps::compute_pass, gpu/timer.rs:507).
 */
int bl_kernels_encode(const bl_kernels* k, size_t kernel, size_t set, void* stream,
                      bl_timer* timer, int32_t frame);
/* Kernels [begin, end) in order, each timed as bl_kernels_encode does. */
int bl_kernels_encode_range(const bl_kernels* k, size_t begin, size_t end, size_t set,
                            void* stream, bl_timer* timer, int32_t frame);

/* The whole program captured once into a CUDA graph (relaxed capture on
 * `stream`), replayed with one launch: the launch-bound ViT-S encoder's way
 * of paying the per-kernel launch cost once per frame instead of per kernel. */
typedef struct bl_graph bl_graph;
int bl_kernels_capture(const bl_kernels* k, size_t set, void* stream, bl_graph** out);
int bl_graph_launch(const bl_graph* g, void* stream);
void bl_graph_destroy(bl_graph* g);

/* ------------------------------------------------------------------ slice timer */

/*
 * Per-kernel GPU timing from cudaEvents, with the semantics of the
 * reference's SliceTimer (crates/beatlm/src/gpu/timer.rs:185-470): a ring of
 * BL_TIMER_RING_DEPTH frames; a frame whose slot is still in flight goes
 * untimed and is counted as skipped; only frames handed back as submitted are
 * read, in submission order; nothing ever blocks (cudaEventQuery).
 */
enum { BL_TIMER_RING_DEPTH = 3 };

int bl_timer_create(uint32_t max_slices, bl_timer** out);
void bl_timer_destroy(bl_timer* t);
uint32_t bl_timer_max_slices(const bl_timer* t);

/* SliceTimer::begin_frame (timer.rs:272): claims a ring slot for `frame` and
 * sets *handle to it, or to -1 when the slot is in flight (frame skipped). */
int bl_timer_begin_frame(bl_timer* t, uint64_t frame, int32_t* handle);
/* SliceTimer::submitted (timer.rs:307): the frame's launches are enqueued;
 * it becomes collectable. A handle of -1 is accepted and ignored. */
int bl_timer_submitted(bl_timer* t, int32_t handle);
/* SliceTimer::submitted_held (timer.rs:332): submitted, but collected only
 * once bl_timer_settle accepts it; settle(accept = 0) rejects it. */
int bl_timer_submitted_held(bl_timer* t, int32_t handle);
int bl_timer_settle(bl_timer* t, int32_t handle, int accept);
/* A begun frame dropped before submission (a ResolvedFrame dropped with its
 * encoder): its slot is freed unread. */
int bl_timer_drop(bl_timer* t, int32_t handle);
/* SliceTimer::invalidate_submitted (timer.rs:445): marks every submitted,
 * uncollected frame as failed; returns how many. */
size_t bl_timer_invalidate_submitted(bl_timer* t);
/* SliceTimer::in_flight (timer.rs:452). */
size_t bl_timer_in_flight(const bl_timer* t);

typedef struct bl_slice_time {
    uint64_t frame;    /* the frame index given to begin_frame */
    uint32_t slice;    /* order of the pass within the frame */
    uint32_t kernel;   /* the kernel index that was encoded */
    double begin_us;   /* pass begin, relative to the frame's first pass */
    double micros;     /* pass duration */
} bl_slice_time;

/* SliceTimer::collect_ready (timer.rs:371): writes the passes of every frame
 * whose events have completed, oldest submitted first, whole frames only, up
 * to `cap` entries; *n = entries written, *frames = frames completed. */
int bl_timer_collect_ready(bl_timer* t, bl_slice_time* out, size_t cap, size_t* n,
                           size_t* frames);

typedef struct bl_timer_stats {
    uint64_t frames_skipped;   /* TimerStats (timer.rs:135) */
    uint64_t frames_collected;
    uint64_t frames_failed;
} bl_timer_stats;
int bl_timer_get_stats(const bl_timer* t, bl_timer_stats* out);

/* Holds `stream` for `microseconds` of device time (at most 1 s) with one
 * single-warp kernel, so that work the host enqueues behind it meanwhile
 * starts back to back. Event pairs around each launch then time the kernels,
 * not the host's launch rate. A measurement aid with no counterpart in the
 * reference, whose timestamp queries are written inside the passes
 * (timer.rs:208). */
int bl_stream_hold(void* stream, uint32_t microseconds);

/* ------------------------------------------------------------ DPT decoder */

/*
 * The DPT decoder's kernels besides its GEMMs (the reference's Conv2d3x3,
 * Conv2d1x1, ConvTranspose2d and ResizeBilinear main ops with the ReLU
 * prologue, crates/beatlm-core/src/kernel.rs:265-319 and WGSL
 * wgsl.rs:387-514; CPU definitions crates/beatlm-bench/src/reference.rs:25-175).
 * Maps are NHWC f32. A convolution is bl_im2col then bl_gemm with the HWIO
 * weights as a [cout][k_pad] 16-bit matrix; a transposed convolution of
 * kernel = stride = f is bl_gemm into [pixels][f*f*cout] then
 * bl_blocks_to_map. Each call enqueues on `stream`.
 */
typedef struct bl_im2col_args {
    const void* input;   /* [h][w][cin] of in_dtype */
    uint32_t h, w, cin;
    uint32_t ksize;      /* 1 or 3 (3: zero padding 1) */
    uint32_t stride;     /* output pixel (y, x) centred on input (y stride, x stride) */
    uint32_t relu;       /* non-zero: max(x, 0) applied to every input value */
    void* out;           /* [oh * ow][k_pad] 16-bit, 16-byte aligned */
    int32_t out_dtype;   /* BL_F16 or BL_BF16 */
    uint32_t k_pad;      /* multiple of 64, >= ksize * ksize * cin; columns past it are 0 */
    int32_t in_dtype;    /* BL_F32 (0, the default), or out_dtype: a 16-bit map copied as it
                            is (cin a multiple of 8, input 16-byte aligned) */
} bl_im2col_args;
int bl_im2col(const bl_im2col_args* args, void* stream);
/* A 3x3 convolution, stride 1, zero padding 1, of an NHWC f32 image as an
 * implicit GEMM (no counterpart in the reference, whose conv kernel gathers
 * per output value, reference.rs:40-101): the tcgen05 GEMM of `gemm` whose A
 * operand is the image read through the nine taps, the rows of each tap's
 * 128 pixels copied by TMA and turned into the 16-bit A tile on chip, so no
 * [h w][9 cin] matrix reaches memory. `gemm` is filled as for bl_gemm with
 * a = NULL, m = h * w, k = 9 * cin rounded up to 64, b the weights from the
 * same [cout][k] tap-major layout bl_im2col's columns use, and any epilogue
 * (bias, activation, residual, output) but no LayerNorm or statistics; the
 * tile width is at most 128 columns. cin must be a multiple of 32. */
typedef struct bl_conv3x3_args {
    const float* input;  /* [h][w][cin] f32, 16-byte aligned */
    uint32_t h, w, cin;
    uint32_t relu;       /* non-zero: max(x, 0) applied to every input value */
} bl_conv3x3_args;
int bl_conv3x3(const bl_gemm_args* gemm, const bl_conv3x3_args* conv, void* stream);
/* out[(y f + ky)][(x f + kx)][co] = blocks[y * w + x][(ky f + kx) cout + co] + bias[co]
 * (bias may be NULL): the f x f block each input pixel of a transposed
 * convolution writes (reference.rs:103-140). */
int bl_blocks_to_map(const float* blocks, const float* bias, float* out, uint32_t h, uint32_t w,
                     uint32_t f, uint32_t cout, void* stream);
/* One output channel of a 1x1 convolution (reference.rs:79-101 with cout 1;
 * the depth head's last convolution, model/depth_anything_v2.rs:680-982):
 * out[p] = act(sum_i in[p][i] * w[i] + bias) over NHWC f32 rows of c values
 * (c a multiple of 4, at most 1024; in and w 16-byte aligned), act = max(x, 0)
 * when relu != 0, in f32 without a GEMM's padded output channels. */
int bl_conv1x1_one(const float* in, const float* w, float bias, float* out, uint32_t pixels,
                   uint32_t c, int32_t relu, void* stream);
/* Bilinear resampling with corners aligned, [ih][iw][c] -> [oh][ow][c]
 * (reference.rs:142-175), in f32. */
int bl_resize_bilinear(const float* in, float* out, uint32_t ih, uint32_t iw, uint32_t oh,
                       uint32_t ow, uint32_t c, void* stream);
/* The same resampling written as 16-bit rows (out_dtype BL_F16 or BL_BF16)
 * of ld values, channels c..ld-1 zero: the A operand of the 1x1 convolution
 * that follows each DPT fusion layer's resampling
 * (model/depth_anything_v2.rs:680-982), the f32 values of bl_resize_bilinear
 * rounded once to 16 bits, with no f32 map in between. c and ld multiples of
 * 8, ld >= c, in and out 16-byte aligned. */
int bl_resize_bilinear_rows16(const float* in, void* out, uint32_t ih, uint32_t iw, uint32_t oh,
                              uint32_t ow, uint32_t c, uint32_t ld, int32_t out_dtype,
                              void* stream);

/* ------------------------------------------------------------- pass cost */

/*
 * One frame of the reference's pass-cost workload
 * (crates/beatlm-host/src/pass_cost.rs:1-110): what a pass costs apart from
 * its work, with and without its timestamps. Here a pass is one CUDA launch,
 * its timestamp writes a cudaEvent pair, and "one pass" holding every
 * dispatch is one CUDA graph of the P launches (pass_cost.rs:148 Variant).
 * The dispatches are the trivial kernel (`groups` blocks of one thread, each
 * adding one to its word of `sink`, which must hold `groups` device words)
 * or, with `kernels`, the first `passes` kernels of that program. Blocks
 * until the frame is done (one frame in flight, pass_cost.rs:29-39).
 */
enum {
    BL_PASS_PER_PASS = 0, /* A: a pair on every launch */
    BL_PASS_ENDS = 1,     /* B: the first launch's begin and the last's end */
    BL_PASS_ONE_PASS = 2, /* C: one graph of all launches, one pair around it */
    BL_PASS_EVERY = 3,    /* D: a pair on every k-th launch, the first included, and the last */
    BL_PASS_ONE_PASS_PDL = 4 /* C with programmatic dependent launch between the graph's
                                trivial launches (no reference counterpart: the boundary
                                cost B200 kernels pay when each overlaps its predecessor) */
};
typedef struct bl_pass_cost_args {
    int32_t variant;           /* BL_PASS_* */
    uint32_t passes;           /* P >= 1 */
    uint32_t every;            /* k of BL_PASS_EVERY */
    uint32_t groups;           /* trivial kernel: 1..65535 blocks */
    uint32_t* sink;            /* trivial kernel: device words, at least `groups` */
    const bl_kernels* kernels; /* non-NULL: time this program's first `passes` kernels */
    void* stream;              /* a cudaStream_t */
} bl_pass_cost_args;
typedef struct bl_pass_cost_frame {
    double span_us;   /* first launch's begin to last launch's end (device) */
    double passes_us; /* sum of the timed launches' own durations (B and C: the span) */
    double encode_us; /* host time to enqueue the frame (C: capture, instantiate, launch) */
    uint32_t pairs;   /* event pairs the frame carried */
    uint32_t reserved;
} bl_pass_cost_frame;
int bl_pass_cost_frame_run(const bl_pass_cost_args* args, bl_pass_cost_frame* out);

/* ------------------------------------------------------------- cost model */

/*
 * Measured slice durations as the estimates the frame scheduler plans with:
 * the reference's CostModel (crates/beatlm-core/src/cost.rs:726-966), fed
 * from this library's cudaEvent slice timer (bl_cost_record_passes) instead
 * of wgpu timestamp queries. A slice is a kernel index of the program
 * (SliceId, cost.rs:273). Every duration is in whole microseconds. Nothing
 * here touches the GPU.
 */
enum {
    BL_EST_MEAN_PLUS_SIGMAS = 0,  /* Estimator::MeanPlusSigmas {alpha, sigmas} */
    BL_EST_WINDOWED_QUANTILE = 1, /* Estimator::WindowedQuantile {window, quantile} */
    BL_EST_CAPPED_DEVIATION = 2,  /* Estimator::CappedDeviation {alpha, sigmas, cap} */
    BL_EST_FRAME_SCALED = 3       /* Estimator::FrameScaled {window, frame_window,
                                     frame_quantile = quantile} */
};
/* CostError (cost.rs:298-325): which parameter bl_cost_create rejected. */
enum {
    BL_COST_INVALID_ALPHA = 1,
    BL_COST_INVALID_SIGMAS = 2,
    BL_COST_INVALID_WINDOW = 3,
    BL_COST_INVALID_QUANTILE = 4,
    BL_COST_INVALID_FRAME_WINDOW = 5,
    BL_COST_INVALID_CAP = 6,
    BL_COST_UNKNOWN_ESTIMATOR = 7 /* a `kind` outside the four above (no reference case) */
};
/* FrameScale (cost.rs:398-414). */
enum { BL_FRAME_SCALE_NONE = 0, BL_FRAME_SCALE_WARMING_UP = 1, BL_FRAME_SCALE_MEASURED = 2 };
enum { BL_COST_MAX_WINDOW = 4096 /* MAX_WINDOW, cost.rs:294 */ };

typedef struct bl_estimator {
    int32_t kind;          /* BL_EST_* */
    uint32_t window;       /* measurements kept per slice (quantile, frame-scaled) */
    uint32_t frame_window; /* frames whose ratio is kept (frame-scaled) */
    uint32_t reserved;
    double alpha;          /* weight of a new measurement (mean + sigmas, capped) */
    double sigmas;         /* standard deviations added to the mean */
    double cap;            /* most padding, as a multiple of the mean (capped) */
    double quantile;       /* the window's rank to read; frame-scaled: the frame quantile */
} bl_estimator;

typedef struct bl_cost bl_cost;

/* Estimator::default (cost.rs:416-425): the 0.9 quantile of the last 32. */
void bl_estimator_default(bl_estimator* out);
/* CostModel::new (cost.rs:748): BL_OK, or BL_ERR_INVALID with *cost_error =
 * the BL_COST_* of the first parameter out of range. */
int bl_cost_create(uint64_t prior_us, const bl_estimator* est, bl_cost** out, int32_t* cost_error);
int bl_cost_clone(const bl_cost* c, bl_cost** out);
void bl_cost_destroy(bl_cost* c);
/* CostModel::estimator (cost.rs:771). */
int bl_cost_estimator(const bl_cost* c, bl_estimator* out);
/* CostModel::record / record_calibration (cost.rs:779-795). */
void bl_cost_record(bl_cost* c, uint32_t slice, uint64_t measured_us);
void bl_cost_record_calibration(bl_cost* c, uint32_t slice, uint64_t measured_us);
/* CostModel::frame_estimate (cost.rs:851): 1 and *out set when the slice
 * counts in a frame's ratio, 0 when it is left out (None). */
int bl_cost_frame_estimate(const bl_cost* c, uint32_t slice, uint64_t* out);
/* CostModel::record_frame (cost.rs:871). */
void bl_cost_record_frame(bl_cost* c, uint64_t predicted_us, uint64_t measured_us);
/* CostModel::frame_scale (cost.rs:898): BL_FRAME_SCALE_*; *scale is set
 * when MEASURED, *recorded and *needed when WARMING_UP (any may be NULL). */
int32_t bl_cost_frame_scale(const bl_cost* c, double* scale, uint64_t* recorded, uint64_t* needed);
/* CostModel::frames_recorded / planning_estimate / estimate / samples
 * (cost.rs:910-975). */
uint64_t bl_cost_frames_recorded(const bl_cost* c);
uint64_t bl_cost_planning_estimate(const bl_cost* c, uint32_t slice);
uint64_t bl_cost_estimate(const bl_cost* c, uint32_t slice);
uint32_t bl_cost_samples(const bl_cost* c, uint32_t slice);
/* A timer duration in whole microseconds, rounded to nearest, saturating
 * (ticks_to_micros, crates/beatlm/src/gpu/timer.rs:781-800). */
uint64_t bl_micros_nearest(double micros);
/* Folds the passes bl_timer_collect_ready wrote: each pass's duration,
 * rounded by bl_micros_nearest, under its kernel index, as the loop's
 * measurements (calibration = 0, CostModel::record) or calibration's
 * (record_calibration; calibrate.rs:165-174). Returns the passes folded. */
size_t bl_cost_record_passes(bl_cost* c, const bl_slice_time* passes, size_t n, int calibration);

/* -------------------------------------------------------------- scheduler */

/*
 * The frame-slice scheduler (crates/beatlm-core/src/schedule.rs:160-790, with
 * sync.rs, budget.rs and the beat grids of time.rs): each submitted input
 * becomes a job with a deadline fixed by the sync policy; each frame the
 * budget is spent on pending jobs in submission order (jobs never
 * interleave), reading every slice at bl_cost_planning_estimate, so the
 * plan follows the cudaEvent-measured costs. Times are whole microseconds
 * on the host's clock. Host code only.
 */
enum { BL_SYNC_FIXED_LATENCY = 0, BL_SYNC_SAME_FRAME = 1, BL_SYNC_ON_BEAT = 2 };
enum { BL_MISS_HOLD_PREVIOUS = 0, BL_MISS_DROP = 1 };
enum { BL_DUE_FRAME = 0, BL_DUE_BEAT = 1 };

/* SyncPolicy (sync.rs): FixedLatency {frames}, SameFrame, or OnBeat {margin,
 * grid}: beats every grid_beat_us from grid_origin_us. */
typedef struct bl_sync_policy {
    int32_t kind;            /* BL_SYNC_* */
    uint32_t frames;         /* FixedLatency */
    uint64_t margin_us;      /* OnBeat */
    uint64_t grid_origin_us; /* OnBeat */
    uint64_t grid_beat_us;   /* OnBeat; 0 is ZeroBeat */
} bl_sync_policy;

/* FrameInfo (time.rs): a frame's index, start and period. */
typedef struct bl_frame_info {
    uint64_t index;
    uint64_t start_us;
    uint64_t period_us;
} bl_frame_info;

typedef struct bl_slice_run { /* SliceRun: submit before the frame's render pass */
    uint64_t job;
    uint32_t slice;
    uint32_t reserved;
    uint64_t position;        /* the slice's index within its job */
} bl_slice_run;
typedef struct bl_delivery { uint64_t job; uint64_t input; } bl_delivery;
typedef struct bl_due { int32_t kind; uint32_t reserved; uint64_t at; } bl_due; /* frame or beat */
typedef struct bl_missed {   /* Missed: the input with no result, and when it was due */
    uint64_t job;
    uint64_t input;
    bl_due due;
    int32_t policy;           /* BL_MISS_* */
    uint32_t reserved;
} bl_missed;
typedef struct bl_frame_plan_info {
    size_t runs, delivered, missed; /* counts of the plan's three lists */
    uint64_t spent_estimate_us;     /* summed planning estimates of the runs, <= budget */
    uint64_t budget_us;
} bl_frame_plan_info;

typedef struct bl_scheduler bl_scheduler;

/* Budget::for_frame (budget.rs): period - render - margin, saturating at 0. */
uint64_t bl_budget_for_frame(uint64_t period_us, uint64_t render_us, uint64_t margin_us);
/* BeatMap::next_beat_at_or_after (time.rs): `grids` holds n (from, origin,
 * beat) triples, the first in effect from 0 and each later one put in effect
 * from its `from` (BeatMap::replace_from); BL_ERR_INVALID for a zero beat. */
int bl_beat_map_next(const uint64_t* grids, size_t n, uint64_t t_us, uint64_t* out);
/* Scheduler::new (schedule.rs:525). */
int bl_scheduler_create(const bl_sync_policy* policy, int32_t miss, uint64_t expected_budget_us,
                        bl_scheduler** out);
void bl_scheduler_destroy(bl_scheduler* s);
/* Scheduler::set_expected_budget / expected_budget (schedule.rs:553-566). */
void bl_scheduler_set_expected_budget(bl_scheduler* s, uint64_t expected_us);
uint64_t bl_scheduler_expected_budget(const bl_scheduler* s);
/* Scheduler::replace_beat_grid (schedule.rs:574): BL_ERR_INVALID when the
 * policy is not OnBeat (NotOnBeat) or the beat is zero. */
int bl_scheduler_replace_beat_grid(bl_scheduler* s, uint64_t from_us, uint64_t origin_us,
                                   uint64_t beat_us);
/* Scheduler::submit (schedule.rs:618): *job = the new job's id; an empty
 * job is BL_ERR_INVALID (EmptyJob). */
int bl_scheduler_submit(bl_scheduler* s, const bl_frame_info* input, const uint32_t* slices,
                        size_t n, const bl_cost* cost, uint64_t* job);
/* Scheduler::plan_frame (schedule.rs:706): plans `frame` against
 * `budget_us`; the plan's lists are read with the three calls below (each
 * returns the list's length and copies up to `cap` entries). */
int bl_scheduler_plan_frame(bl_scheduler* s, const bl_frame_info* frame, uint64_t budget_us,
                            const bl_cost* cost, bl_frame_plan_info* info);
size_t bl_scheduler_plan_runs(const bl_scheduler* s, bl_slice_run* out, size_t cap);
size_t bl_scheduler_plan_delivered(const bl_scheduler* s, bl_delivery* out, size_t cap);
size_t bl_scheduler_plan_missed(const bl_scheduler* s, bl_missed* out, size_t cap);
/* Scheduler::pending / due (schedule.rs:773-790): due returns 1 and fills
 * *out while the job is pending, 0 otherwise. */
size_t bl_scheduler_pending(const bl_scheduler* s);
int bl_scheduler_due(const bl_scheduler* s, uint64_t job, bl_due* out);

/* ------------------------------------------------------------ memory plan */

/*
 * The static memory plan (MemoryPlan, crates/beatlm-core/src/memory.rs:285-375)
 * and its realisation as ONE device allocation (Arenas,
 * crates/beatlm/src/gpu/arenas.rs:65-140, which makes one buffer per arena;
 * here the arenas are consecutive 256-byte-aligned ranges of a single
 * cudaMalloc). Planning is host-only work and needs no GPU.
 *
 * The plan keeps the reference's five rules: tensors whose use ranges
 * intersect (inclusive at both ends) never share a byte of one arena;
 * offsets are multiples of the profile's alignment and sizes are the byte
 * size rounded up to 4; no arena exceeds the profile's arena cap, and a
 * larger tensor is an error, never split; the same set of tensors gives the
 * same plan whatever order they are listed in; malformed input is an error.
 * Algorithm: greedy by rounded size, descending, ties by id; each tensor goes
 * to the lowest aligned offset of the first arena where it fits beside the
 * already placed tensors whose lifetimes intersect its own; a new arena
 * opens when none fits.
 */

/* TensorDesc (memory.rs:158-170). elem_bytes is DType::size_bytes: 4 for
 * f32, 2 for f16 and bf16 (any non-zero width is accepted). */
typedef struct bl_tensor_desc {
    uint32_t id;
    uint32_t elem_bytes;
    uint64_t elements;   /* at least 1 */
    uint32_t first_use;  /* operation index in program order */
    uint32_t last_use;   /* not before first_use */
} bl_tensor_desc;

/* The profile fields the planner reads (DeviceProfile, crates/beatlm-core/
 * src/device.rs:97-125): the arena cap is min(max_binding_bytes,
 * max_buffer_bytes). */
typedef struct bl_device_profile {
    uint64_t max_binding_bytes;
    uint64_t max_buffer_bytes;
    uint32_t offset_alignment;
} bl_device_profile;

/* DeviceProfile::webgpu_baseline (device.rs:97): 128 MiB binding, 256 MiB
 * buffer, 256-byte alignment. */
int bl_device_profile_webgpu_baseline(bl_device_profile* out);
/* The profile of CUDA device `device`: 256-byte alignment and an arena cap
 * of the device's total memory (a kernel addresses any byte of one
 * allocation). Needs the device; allocates nothing. */
int bl_device_profile_cuda(int device, bl_device_profile* out);

/* PlanError (memory.rs:220-265). On failure bl_plan_create fills a
 * bl_plan_error: `id` the tensor, and a/b = first_use/last_use for
 * INVALID_LIFETIME or size/limit for TENSOR_TOO_LARGE. */
enum {
    BL_PLAN_DUPLICATE_TENSOR = 1,
    BL_PLAN_INVALID_LIFETIME = 2,
    BL_PLAN_EMPTY_TENSOR = 3,
    BL_PLAN_SIZE_OVERFLOW = 4,
    BL_PLAN_TENSOR_TOO_LARGE = 5,
    BL_PLAN_INVALID_PROFILE = 6,
    BL_PLAN_TOO_MANY_TENSORS = 7
};
typedef struct bl_plan_error {
    int32_t kind; /* 0 = none, else BL_PLAN_* */
    uint32_t id;
    uint64_t a;
    uint64_t b;
} bl_plan_error;

/* Placement (memory.rs:200-218). */
typedef struct bl_placement {
    uint32_t arena;
    uint32_t reserved;
    uint64_t offset;
    uint64_t size;
} bl_placement;

typedef struct bl_plan bl_plan;

/* MemoryPlan::new (memory.rs:285). Returns BL_OK, or BL_ERR_INVALID /
 * BL_ERR_CAPACITY (TENSOR_TOO_LARGE) with *err filled when err != NULL. */
int bl_plan_create(const bl_tensor_desc* tensors, size_t n, const bl_device_profile* profile,
                   bl_plan** out, bl_plan_error* err);
void bl_plan_destroy(bl_plan* p);
/* MemoryPlan::arenas (memory.rs:379): arena sizes, each the end of the last
 * byte used in it. Writes min(count, cap) sizes; returns the count. */
size_t bl_plan_arenas(const bl_plan* p, uint64_t* sizes, size_t cap);
/* MemoryPlan::placement (memory.rs:385): BL_OK, or BL_ERR_INVALID for a
 * tensor the plan was not made with. */
int bl_plan_placement(const bl_plan* p, uint32_t id, bl_placement* out);
/* MemoryPlan::peak_live_bytes / total_bytes (memory.rs:403-414). */
uint64_t bl_plan_peak_live_bytes(const bl_plan* p);
uint64_t bl_plan_total_bytes(const bl_plan* p);
/* MemoryPlan::valid_on (memory.rs:423): 1 when every arena fits the
 * profile's cap and the plan's alignment is a multiple of the profile's. */
int bl_plan_valid_on(const bl_plan* p, const bl_device_profile* profile);

typedef struct bl_arenas bl_arenas;

/* Arenas::new (arenas.rs:88): ONE cudaMalloc on `device` holding every
 * arena of the plan, arena i at a 256-byte-aligned base. BL_ERR_INVALID when
 * the plan is not valid on the device's profile (ArenaError::
 * PlanNotValidOnDevice). The only allocation a plan needs: nothing in the
 * steady state allocates. */
int bl_arenas_create(const bl_plan* p, int device, bl_arenas** out);
void bl_arenas_destroy(bl_arenas* a);
/* Bytes of the single allocation. */
uint64_t bl_arenas_bytes(const bl_arenas* a);
/* Arenas::buffer (arenas.rs:117): the device address of arena `arena`. */
int bl_arenas_base(const bl_arenas* a, uint32_t arena, void** out);
/* Arenas::binding (arenas.rs:131): the device address of a placement,
 * after the reference's checks (unknown arena, out of range or empty,
 * misaligned offset), each BL_ERR_INVALID with its reason in the message. */
int bl_arenas_binding(const bl_arenas* a, const bl_placement* p, void** out);
/* Host writes of weights and inputs into a placement, and reads of results
 * (the reference's queue.write_buffer and copy-out). `offset` is relative to
 * the placement and offset + bytes must lie inside it. Enqueued on `stream`;
 * pinned host memory makes them asynchronous. */
int bl_arenas_write(const bl_arenas* a, const bl_placement* p, uint64_t offset,
                    const void* src, uint64_t bytes, void* stream);
int bl_arenas_read(const bl_arenas* a, const bl_placement* p, uint64_t offset, void* dst,
                   uint64_t bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif
