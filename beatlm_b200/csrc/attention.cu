// Fused non-causal attention for head_dim 64 on sm_100a: the reference's
// AttentionScores -> Scale -> Softmax -> AttentionValues chain
// (crates/beatlm-core/src/kernel.rs:722-777; CPU definition in
// crates/beatlm-bench/src/reference.rs:437-494) as one kernel with an online
// softmax, so the [tokens][heads][tokens] scores never reach memory.
//
// One CTA computes one or two 128-row query tiles (QT, a template parameter)
// of one head of one sequence over a range of key tiles (all of them, or one
// split of them). With QT = 2, 12 warps in three warpgroups, the control
// warpgroup giving registers to the softmax ones (setmaxnreg); with QT = 1,
// 8 warps in two:
//   warp 0      TMA producer: the CTA's Q rows once, then K/V tiles of 128
//               keys into a 4-stage ring (128-byte swizzle, zero fill past
//               the last key).
//   warp 1      MMA issuer (one thread): S = Q_t K^T into TMEM (M=128,
//               N=128, K=64, f32) and O_t += P V with P read from TMEM
//               (M=128, N=64, K=128, f16). S buffers rotate over the slots
//               j = QT i + t (key tile i, query tile t), so the scores of the
//               next slots are computed before a softmax needs them (QT = 2,
//               three buffers: S_0 S_1 S_2 | PV_0 S_3 | PV_1 S_4 ...; QT = 1,
//               two: S_0 S_1 | PV_0 S_2 | PV_1 S_3 ...).
//   warps 4..7  softmax of tile 0 (warps 8..11 of tile 1): one thread per
//               query row (TMEM lane) holding its 128 scores in registers;
//               the running max is updated lazily (O is rescaled in TMEM
//               only when the max grew by more than 2^8); P is written as
//               f16 over the consumed S columns; exponentials on the MUFU
//               ex2 unit.
// With more than one key split, the splits of a query group either form a
// cluster and combine in distributed shared memory, or write their
// unnormalised O and (max, sum) per row to a workspace where the last CTA
// of the group (an atomic counter, no waiting) combines them.
// TMEM: S buffers at [128 b, 128 b + 128), then O_t (64 columns each);
// P aliases the S buffer it came from.
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

#include "host.h"

namespace bl {
namespace attn {

constexpr int BM = 128;       // query rows per tile
constexpr int BN = 128;       // keys per tile
constexpr int HD = 64;        // head width
constexpr int STAGES = 4;     // K/V ring depth
constexpr int kSoftmaxWarp0 = 4;
constexpr uint32_t kTileBytes = BM * HD * 2;  // 16 KiB per 128x64 tile
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;
// The kernel comes in two shapes, by the query tiles a CTA computes (QT):
//   QT = 2: 12 warps; the control warpgroup gives registers to the two
//           softmax warpgroups (setmaxnreg: 128 x 56 + 256 x 224 = 384 x
//           168, the launch allocation). Three S buffers rotate over the
//           slots j = 2 i + t (key tile i, query tile t).
//   QT = 1: 8 warps, one softmax warpgroup, no register split (a thread may
//           hold up to 255). Two S buffers rotate over the slots j = i.
// In both the S of slot j + kSBufs reuses slot j's buffer and is issued
// right after PV(j), so the S of tile t at key tile i is always issued after
// PV_t(i - 2). O_t lives at kColO + 64 t.
template <int kQT>
struct Shape {
    static_assert(kQT == 1 || kQT == 2, "one or two query tiles per CTA");
    static constexpr int QT = kQT;
    static constexpr int ROWS = BM * QT;  // query rows per CTA
    static constexpr int kThreads = 32 * (kSoftmaxWarp0 + 4 * QT);
    static constexpr int kSBufs = QT == 2 ? 3 : 2;
    static constexpr uint32_t kColO = 128 * kSBufs;
    static_assert(kColO + 64 * QT <= kTmemCols, "TMEM columns");
    // Register split (QT = 2 only): the launch gives every thread kLaunchRegs.
    static constexpr bool kRegSplit = QT == 2;
    static constexpr int kLaunchRegs = 168;
    static constexpr int kControlRegs = 56;
    static constexpr int kSoftmaxRegs = 224;
    static_assert(!kRegSplit ||
                      128 * kControlRegs + 32 * 4 * QT * kSoftmaxRegs <= kThreads * kLaunchRegs,
                  "register split exceeds the launch allocation");
};
// Lazy rescaling: the max used for exponents may trail the true max by up to
// this (log2 units), so p <= 2^8, well inside f16.
constexpr float kRescaleThreshold = 8.0f;

// Head-parallel exchange (bl_attention_peers): every output row of this
// rank's heads is stored into each rank's output buffer (peer memory over
// NVLink, the local buffer for this rank) as soon as it is final, and the
// CTAs exit without fences. A one-warp kernel launched right behind
// (peer_arrive_kernel) starts when the attention grid has completed, so all
// of its stores are performed, raises this rank's flag in every rank's
// buffer and waits, bounded, until every rank's flag for this launch has
// arrived in its own.
constexpr int kMaxPeers = 8;
struct PeerParams {
    int n;                         // ranks the rows go to; 0 = store to `out` only
    int rank;                      // this rank
    unsigned epoch;                // this launch's flag value (increases by one per launch)
    const unsigned* flags;         // this rank's arrival flags, one word per rank
    uint8_t* dst[kMaxPeers];       // rank r's output base for this launch (column-shifted)
    unsigned* flag_at[kMaxPeers];  // rank r's flag word of this rank
};

struct Params {
    int tokens;
    int head_begin;
    int heads_rel;        // heads in this launch (gridDim.y)
    int row_begin, row_end;
    int q_col0, k_col0, v_col0;  // element column of head 0's Q/K/V in a row
    float scale_log2;            // scale * log2(e)
    int qk_fmt;                  // 0 = f16, 1 = bf16
    void* out;
    long long out_row_stride;    // elements
    long long out_batch_stride;  // elements
    int out_head_base;
    int splits;       // key splits; gridDim.z = batch * splits (uniform grid)
    int cluster;      // 1: the splits of a query group are one cluster, combined in DSMEM
    // Mixed grid (cluster form only): a 1-D grid of clusters of `splits`
    // CTAs over the query groups u = (batch * heads_rel + head) * q_ctas +
    // tile; groups [0, head_units) run unsplit (a cluster then holds
    // `splits` different groups, which do not combine), the rest split
    // `splits` ways, one cluster each. 0 = the uniform grid.
    int head_units;
    int q_ctas;       // query groups per head
    int kv_tiles;     // ceil(tokens / BN)
    uint4* part_o;    // [unit][split][ROWS][HD / 8]: f16 O / l of each row
    float2* part_ml;  // [unit][split][ROWS]: (max, sum)
    unsigned* counters;  // [unit]
    unsigned long long* trace;  // optional per-CTA timeline
    Status* status;
};

template <int QT>
struct SmemTail {
    uint64_t q_full;
    uint64_t kv_full[STAGES];
    uint64_t kv_empty[STAGES];
    // S_t(i) ready / P_t(i) written: two barriers per tile, for even and odd
    // key tiles, so neither side can run two phases ahead of the other
    uint64_t s_full[QT][2];
    uint64_t p_full[QT][2];
    uint64_t o_done[QT];
    uint64_t o_final[QT];  // the last PV of tile t is complete
    uint64_t drain;
    uint64_t parts_full;  // cluster combine: the partials this CTA combines have landed
    uint32_t tmem_base;
    int abort;
    unsigned last;  // this CTA combines the splits
    // this CTA's query group, key split and the group's split count (written
    // once at set-up and read where needed, so no role keeps them live)
    int unit, split, nsplit;
};

constexpr int kMaxClusterSplits = 8;  // portable cluster size
// Cluster combine: a pushed partial is 9 vectors of 16 bytes (the row's O / l
// as 64 f16, then (max, sum)), stored k-major: vector v of every row a source
// pushes is contiguous, so a warp's remote store covers 512 consecutive bytes
// and the owner's reads are conflict-free. The area holds the splits - 1
// sources of up to ceil(8 / splits) warps of rows: most at 7 splits.
constexpr int kPartVecs = HD / 8 + 1;
template <int ROWS>
constexpr size_t part_area(int splits) {
    return static_cast<size_t>(splits - 1) * kPartVecs * ((ROWS / 32 + splits - 1) / splits) *
           32 * 16;
}
template <int ROWS>
constexpr size_t max_part_area(int s = 2) {
    return s > kMaxClusterSplits
               ? 0
               : (part_area<ROWS>(s) > max_part_area<ROWS>(s + 1) ? part_area<ROWS>(s)
                                                                  : max_part_area<ROWS>(s + 1));
}
template <int QT>
constexpr size_t kPartArea = max_part_area<BM * QT>();
template <int QT>
constexpr size_t kSmemBytes = 1024 /*align slack*/ + QT * kTileBytes /*Q*/ +
                              STAGES * 2 * kTileBytes /*K,V*/ + kPartArea<QT> +
                              sizeof(SmemTail<QT>);
static_assert(kSmemBytes<1> <= 232448 && kSmemBytes<2> <= 232448, "shared memory");

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
    return sdesc_sw128(addr, 16, 1024);
}
// V tile [keys][64] with the 64 columns contiguous is the MN-major B operand
// of O += P V: one 128-byte swizzle atom spans N = 64, groups of 8 keys are
// 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_v(uint32_t addr) {
    return sdesc_sw128(addr, kTileBytes, 1024);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ void store_row(void* base, int dt, const float* o, float inv_l) {
    if (dt == BL_F32) {
        float4* dst = reinterpret_cast<float4*>(base);
#pragma unroll
        for (int c = 0; c < HD / 4; ++c)
            dst[c] = make_float4(o[4 * c] * inv_l, o[4 * c + 1] * inv_l, o[4 * c + 2] * inv_l,
                                 o[4 * c + 3] * inv_l);
        return;
    }
    uint4* dst = reinterpret_cast<uint4*>(base);
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
        const float* v = o + 8 * c;
        if (dt == BL_F16)
            dst[c] = make_uint4(pack_f16x2(v[0] * inv_l, v[1] * inv_l),
                                pack_f16x2(v[2] * inv_l, v[3] * inv_l),
                                pack_f16x2(v[4] * inv_l, v[5] * inv_l),
                                pack_f16x2(v[6] * inv_l, v[7] * inv_l));
        else
            dst[c] = make_uint4(pack_bf16x2(v[0] * inv_l, v[1] * inv_l),
                                pack_bf16x2(v[2] * inv_l, v[3] * inv_l),
                                pack_bf16x2(v[4] * inv_l, v[5] * inv_l),
                                pack_bf16x2(v[6] * inv_l, v[7] * inv_l));
    }
}

// One output row of 64 values scaled by inv_l, as eight 16-byte vectors of
// the 16-bit output type.
template <int kOutDtype>
__device__ __forceinline__ void pack_row16(const float* o, float inv_l, uint4 (&pk)[HD / 8]) {
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
        const float* v = o + 8 * c;
        if (kOutDtype == BL_F16)
            pk[c] = make_uint4(pack_f16x2(v[0] * inv_l, v[1] * inv_l),
                               pack_f16x2(v[2] * inv_l, v[3] * inv_l),
                               pack_f16x2(v[4] * inv_l, v[5] * inv_l),
                               pack_f16x2(v[6] * inv_l, v[7] * inv_l));
        else
            pk[c] = make_uint4(pack_bf16x2(v[0] * inv_l, v[1] * inv_l),
                               pack_bf16x2(v[2] * inv_l, v[3] * inv_l),
                               pack_bf16x2(v[4] * inv_l, v[5] * inv_l),
                               pack_bf16x2(v[6] * inv_l, v[7] * inv_l));
    }
}

// The arrival barrier of a head-parallel launch: one warp, launched behind
// the attention grid with programmatic dependent launch; griddepcontrol.wait
// returns once that grid has completed and its memory operations (the row
// stores into every rank's buffer) are performed. Lane r raises this rank's
// flag in rank r's header (a system-scope release) and then waits for rank
// r's flag for this launch in this rank's header (a system-scope acquire),
// giving up after the wait limit with ST_TIMEOUT_PEER and the missing rank.
// Ranks run on different GPUs, so waiting here for the others cannot
// deadlock a GPU; a rank that never launches only costs the wait limit.
__global__ void __launch_bounds__(32, 1) peer_arrive_kernel(const __grid_constant__ PeerParams q,
                                                            Status* status) {
    pdl_wait();
    const int r = static_cast<int>(threadIdx.x);
    if (r < q.n) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        st_release_sys(q.flag_at[r], q.epoch);
        const long long t0 = clock64();
        while (static_cast<int>(ld_acquire_sys(q.flags + r) - q.epoch) < 0) {
            if (clock64() - t0 > wait_limit(status)) {
                record_status(status, ST_TIMEOUT_PEER, static_cast<uint32_t>(r));
                break;
            }
            __nanosleep(64);
        }
    }
}

// The softmax threads (warps 4..) only.
template <int QT>
__device__ __forceinline__ void softmax_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(32 * 4 * QT) : "memory");
}

template <int kQT, int kOutDtype, bool kPeers = false>
__global__ void __launch_bounds__(Shape<kQT>::kThreads, 1)
    attention_fwd(const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const Params p,
                  const __grid_constant__ PeerParams peers) {
    using Sh = Shape<kQT>;
    constexpr int QT = kQT;
    constexpr int ROWS = Sh::ROWS;
    constexpr int kSBufs = Sh::kSBufs;
    constexpr uint32_t kColO = Sh::kColO;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sQ = smem;                                          // tile t at + t*kTileBytes
    uint8_t* sK = smem + QT * kTileBytes;                        // stage s at + s*kTileBytes
    uint8_t* sV = smem + QT * kTileBytes + STAGES * kTileBytes;  // stage s at + s*kTileBytes
    uint8_t* sP = smem + QT * kTileBytes + 2 * STAGES * kTileBytes;  // cluster partials
    SmemTail<QT>* tail = reinterpret_cast<SmemTail<QT>*>(sP + kPartArea<QT>);
    volatile int* abort = &tail->abort;

    const int warp = warp_id();
    const int lane = lane_id();
    // This CTA's place, from the shared copy: its query group (unit), key
    // split and the group's split count; the group's head, sequence and
    // first query row; its key tiles [t0, t0 + n).
    const volatile int* coord = &tail->unit;
    auto c_unit = [&]() { return coord[0]; };
    auto c_split = [&]() { return coord[1]; };
    auto c_nsplit = [&]() { return coord[2]; };
    auto c_head = [&](int unit) { return p.head_begin + (unit / p.q_ctas) % p.heads_rel; };
    auto c_batch = [&](int unit) { return unit / (p.q_ctas * p.heads_rel); };
    auto c_q0 = [&](int unit) { return p.row_begin + (unit % p.q_ctas) * ROWS; };
    auto c_t0 = [&]() { return p.kv_tiles * c_split() / c_nsplit(); };
    auto c_n = [&]() { return p.kv_tiles * (c_split() + 1) / c_nsplit() - c_t0(); };

    if (threadIdx.x == 0) {
        trace_stamp(p.trace, 0);
        int unit, split, nsplit = p.splits;
        if (p.head_units > 0) {
            const int b = static_cast<int>(blockIdx.x);
            if (b < p.head_units) {
                unit = b, split = 0, nsplit = 1;
            } else {
                unit = p.head_units + (b - p.head_units) / p.splits;
                split = (b - p.head_units) % p.splits;
            }
        } else {
            unit = (static_cast<int>(blockIdx.z / p.splits) * p.heads_rel +
                    static_cast<int>(blockIdx.y)) * p.q_ctas + static_cast<int>(blockIdx.x);
            split = static_cast<int>(blockIdx.z % p.splits);
        }
        tail->unit = unit, tail->split = split, tail->nsplit = nsplit;
        mbar_init(smem_u32(&tail->q_full), 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->kv_full[s]), 1);
            mbar_init(smem_u32(&tail->kv_empty[s]), 1);
        }
        for (int t = 0; t < QT; ++t) {
            for (int e = 0; e < 2; ++e) {
                mbar_init(smem_u32(&tail->s_full[t][e]), 1);
                mbar_init(smem_u32(&tail->p_full[t][e]), BM);
            }
            mbar_init(smem_u32(&tail->o_done[t]), 1);
            mbar_init(smem_u32(&tail->o_final[t]), 1);
        }
        mbar_init(smem_u32(&tail->drain), 1);
        if (p.cluster && nsplit > 1) {
            // one arrival per pushing warp: the warps w = rank (mod splits) of
            // each other CTA of the cluster (the mixed grid's unsplit groups
            // never combine and leave it uninitialised)
            const int me = static_cast<int>(cluster_rank());
            const int nw = (ROWS / 32 - me + nsplit - 1) / nsplit;
            mbar_init(smem_u32(&tail->parts_full), static_cast<uint32_t>(nw * (nsplit - 1)));
        }
        tail->abort = 0;
        tail->last = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        tma_prefetch_desc(&tm_q);
        tma_prefetch_desc(&tm_k);
        tma_prefetch_desc(&tm_v);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    // the cluster barrier's arrive now (every CTA's barriers are initialised),
    // its wait just before the first remote access
    if (p.cluster) cluster_arrive();
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) trace_stamp(p.trace, 1);

    if (warp < kSoftmaxWarp0) {
        if constexpr (Sh::kRegSplit)
            asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(Sh::kControlRegs));
        if (warp == 0) {
            // -------------------------------------------------- producer
            // The warp runs the loop in step: lane 0 copies the CTA's Q rows
            // (one box) and each stage's K, arming the stage; lane 1 copies
            // each stage's V, so K and V are in flight together (a thread's
            // bulk copies complete one after another). Lane 0 alone waits
            // for a free stage and the vote hands the outcome to the warp.
            const uint32_t b_q = smem_u32(&tail->q_full);
            const int unit = c_unit(), head = c_head(unit), batch = c_batch(unit);
            const int t0 = c_t0(), n = c_n();
            if (lane == 0) {
                mbar_arrive_expect_tx(b_q, QT * kTileBytes);
                tma_load_3d(smem_u32(sQ), &tm_q, p.q_col0 + head * HD, c_q0(unit), batch, b_q);
            }
            int loaded = 0;  // key tiles whose loads were started
            for (int i = 0; i < n; ++i) {
                const int s = i % STAGES;
                const int r = i / STAGES;
                bool w = true;
                if (lane == 0 && r > 0)
                    w = mbar_wait(smem_u32(&tail->kv_empty[s]), (r - 1) & 1, abort, p.status,
                                  ST_TIMEOUT_TMA, i);
                if (!__all_sync(0xFFFFFFFFu, w)) break;
                const uint32_t bar = smem_u32(&tail->kv_full[s]);
                if (lane == 0) {
                    mbar_arrive_expect_tx(bar, 2 * kTileBytes);
                    tma_load_3d(smem_u32(sK + s * kTileBytes), &tm_k, p.k_col0 + head * HD,
                                (t0 + i) * BN, batch, bar);
                } else if (lane == 1) {
                    tma_load_3d(smem_u32(sV + s * kTileBytes), &tm_v, p.v_col0 + head * HD,
                                (t0 + i) * BN, batch, bar);
                }
                __syncwarp();
                ++loaded;
            }
            if (lane == 0 && *abort) {
                // Unwinding: let every copy this thread started land before
                // the CTA's shared memory is released.
                mbar_wait(b_q, 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0);
                for (int s = 0; s < STAGES && s < loaded; ++s) {
                    const int uses = (loaded - s - 1) / STAGES + 1;
                    mbar_wait(smem_u32(&tail->kv_full[s]), (uses - 1) & 1, nullptr, p.status,
                              ST_TIMEOUT_DRAIN, s);
                }
            }
            __syncwarp();
        } else if (warp == 1) {
            // -------------------------------------------------- MMA issuer
            // The whole warp runs the issuer's loop and one elected lane
            // issues, so descriptors and loop state stay warp-uniform (the
            // MMA's operands are uniform registers; single-lane code paid
            // about 75 cycles per MMA instead of about 30). One lane waits on
            // each barrier and the vote hands its outcome to the warp.
            const bool elected = elect_one();
            auto wait_all = [&](uint32_t bar, uint32_t parity, uint32_t where) -> bool {
                bool r = true;
                if (elected) r = mbar_wait(bar, parity, abort, p.status, ST_TIMEOUT_MMA, where);
                return __all_sync(0xFFFFFFFFu, r);
            };
            const uint32_t idesc_s = idesc_f16(BM, BN, p.qk_fmt, p.qk_fmt, 0, 0);
            const uint32_t idesc_o = idesc_f16(BM, HD, 0, 0, 0, 1);
            const int n = c_n();
            bool ok = wait_all(smem_u32(&tail->q_full), 0, 0xFFFF);
            tc_fence_after();
            auto wait_kv = [&](int i) -> bool {
                if (!wait_all(smem_u32(&tail->kv_full[i % STAGES]), (i / STAGES) & 1, i))
                    return false;
                tc_fence_after();
                return true;
            };
            // Slot j = QT i + t is (key tile i, query tile t); its S goes to
            // buffer j % kSBufs. The S of slot j + kSBufs reuses the buffer of
            // slot j, so it is issued right after slot j's PV (the tensor core
            // runs one thread's MMAs in order); the S of the slots between are
            // already issued by then, so a softmax warpgroup finds its next
            // scores ready when it finishes its current ones.
            // Descriptors are built once: a tile or stage moves the 14-bit
            // address field by kTileBytes / 16, a K step of 16 elements by 32
            // bytes (K-major Q, K) or 16 rows (V).
            const uint64_t dq = desc_kmajor(smem_u32(sQ));
            const uint64_t dk = desc_kmajor(smem_u32(sK));
            const uint64_t dv = desc_v(smem_u32(sV));
            constexpr uint64_t kTileStep = kTileBytes >> 4;
            auto issue_s = [&](int j) {
                const int t = j % QT, i = j / QT;
                const uint64_t a = dq + t * kTileStep;
                const uint64_t b = dk + (i % STAGES) * kTileStep;
                const uint32_t dst = tmem + kColS + 128 * (j % kSBufs);
                if (elected) {
                    mma_ss(dst, a, b, idesc_s, 0u);
#pragma unroll
                    for (int k = 1; k < HD / 16; ++k) mma_ss(dst, a + 2 * k, b + 2 * k, idesc_s, 1u);
                    mma_commit(smem_u32(&tail->s_full[t][i & 1]));
                }
                __syncwarp();
            };
            auto issue_pv = [&](int j) -> bool {
                const int t = j % QT, i = j / QT;
                if (!wait_all(smem_u32(&tail->p_full[t][i & 1]), (i >> 1) & 1,
                              0x10000 | (t << 12) | i))
                    return false;
                tc_fence_after();
                const uint64_t b = dv + (i % STAGES) * kTileStep;
                const uint32_t p_col = tmem + kColS + 128 * (j % kSBufs);
                const uint32_t o = tmem + kColO + 64 * t;
                if (elected) {
                    mma_ts(o, p_col, b, idesc_o, i > 0 ? 1u : 0u);
#pragma unroll
                    for (int k = 1; k < BN / 16; ++k)
                        mma_ts(o, p_col + k * 8, b + 128 * k, idesc_o, 1u);
                    // The stage is released after its last reader (the last
                    // tile's PV), and only if the producer will refill it, so no
                    // arrival lands after the CTA has finished.
                    if (t == QT - 1 && i + STAGES < n)
                        mma_commit(smem_u32(&tail->kv_empty[i % STAGES]));
                    mma_commit(smem_u32(&tail->o_done[t]));
                    if (i == n - 1) mma_commit(smem_u32(&tail->o_final[t]));
                }
                __syncwarp();
                return true;
            };
            const int slots = QT * n;
            for (int j = 0; j < kSBufs && j < slots && ok; ++j) {
                if (j % QT == 0) ok = wait_kv(j / QT);
                if (ok) issue_s(j);
            }
            for (int j = 0; j < slots && ok; ++j) {
                ok = issue_pv(j);
                const int next = j + kSBufs;
                if (ok && next < slots) {
                    if (next % QT == 0) ok = wait_kv(next / QT);
                    if (ok) issue_s(next);
                }
            }
            if (!ok) {
                // Unwinding: wait for the tensor core to finish what was
                // issued before TMEM is released.
                if (elected) {
                    mma_commit(smem_u32(&tail->drain));
                    mbar_wait(smem_u32(&tail->drain), 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0xD);
                }
                __syncwarp();
            }
        }
        if (p.cluster) {
            // the wait of the cluster barrier arrived on at set-up
            __syncwarp();
            cluster_wait();
        }
    } else {
        if constexpr (Sh::kRegSplit)
            asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(Sh::kSoftmaxRegs));
        // ------------------------------------------------------ softmax
        constexpr unsigned kFull = 0xFFFFFFFFu;
        const int t = (warp - kSoftmaxWarp0) / 4;  // query tile of this warpgroup
        const int sub = warp & 3;                  // TMEM sub-partition of this warp
        const int row = sub * 32 + lane;           // query row within the tile
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(sub * 32) << 16);
        const uint32_t o_col = t_lane + kColO + 64 * t;
        const uint32_t b_o = smem_u32(&tail->o_done[t]);
        const float c = p.scale_log2;
        const unsigned long long c2 = f2pack(c, c);
        float m_used = -INFINITY;
        float l = 0.0f;
        bool ok = true;
        const int t0 = c_t0(), n = c_n();
        for (int i = 0; i < n; ++i) {
            const uint32_t s_col = t_lane + kColS + 128 * ((QT * i + t) % kSBufs);
            const uint32_t b_p = smem_u32(&tail->p_full[t][i & 1]);
            ok = mbar_wait(smem_u32(&tail->s_full[t][i & 1]), (i >> 1) & 1, abort, p.status,
                           ST_TIMEOUT_SOFTMAX, (t << 12) | i);
            ok = __all_sync(kFull, ok);
            if (!ok) break;
            tc_fence_after();
            uint32_t s[BN];
            tmem_ld32(s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(s + 0));
            tmem_ld32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
            tmem_ld32(s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
            tmem_ld32(s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
            tmem_wait_ld();
            const int valid = p.tokens - (t0 + i) * BN;  // keys of this tile that exist
            if (valid < BN) {                            // only the sequence's last tile
#pragma unroll
                for (int k = 0; k < BN; ++k)
                    if (k >= valid) s[k] = __float_as_uint(-INFINITY);
            }
            // row max: four independent chains of three-input max
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int k = 0; k < BN; k += 8) {
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    mx[q] = fmax3(mx[q], __uint_as_float(s[k + 2 * q]),
                                  __uint_as_float(s[k + 2 * q + 1]));
            }
            const float m_row = fmax3(fmaxf(mx[0], mx[1]), mx[2], mx[3]);
            // Lazy rescaling, decided per row; the O read-modify-write is a
            // warp-collective TMEM access, so a warp does it when any of its
            // rows needs it (the others multiply by 1, which is exact).
            const float m_new = fmaxf(m_used, m_row * c);
            const bool need = m_new > m_used + kRescaleThreshold;
            float alpha = 1.0f;
            if (need) {
                alpha = ex2(m_used - m_new);
                l *= alpha;
                m_used = m_new;
            }
            if (i > 0 && __any_sync(kFull, need)) {
                // O_t after PV_t(i-1). The S of this slot was issued after
                // PV_t(i-2), so o_done is at most one phase behind here and
                // the parity names the right phase.
                ok = mbar_wait(b_o, (i - 1) & 1, abort, p.status, ST_TIMEOUT_SOFTMAX,
                               0x10000 | (t << 12) | i);
                ok = __all_sync(kFull, ok);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t o[32];
                    tmem_ld32(o_col + 32 * h, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 32; ++k)
                        o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
                    tmem_st32(o_col + 32 * h, o);
                }
                tmem_wait_st();
            }
            // exponents on the MUFU unit (measured: moving a share of them to
            // a polynomial on the FMA pipe slows the MMA thread, which shares
            // its issue slots with these warps, more than it unloads MUFU);
            // four partial sums; P packed to f16 in place (pair k lands in
            // s[k], whose own score was consumed at pair k/2)
            const unsigned long long nm2 = f2pack(-m_used, -m_used);
            unsigned long long acc[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) acc[q] = f2pack(0.0f, 0.0f);
#pragma unroll
            for (int k = 0; k < BN / 2; ++k) {
                const unsigned long long x2 =
                    ffma2(f2pack(__uint_as_float(s[2 * k]), __uint_as_float(s[2 * k + 1])), c2,
                          nm2);
                float p0, p1, x0, x1;
                f2unpack(x2, x0, x1);
                p0 = ex2(x0);
                p1 = ex2(x1);
                acc[k & 3] = fadd2(acc[k & 3], f2pack(p0, p1));
                s[k] = pack_f16x2(p0, p1);
            }
            const unsigned long long a01 = fadd2(acc[0], acc[1]);
            const unsigned long long a23 = fadd2(acc[2], acc[3]);
            float sa, sb;
            f2unpack(fadd2(a01, a23), sa, sb);
            l += sa + sb;
            tmem_st32(s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(s + 0));
            tmem_st32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(b_p);
        }
        // The final O_t: o_done may be up to two phases from here (PV_t(n-2)
        // can still be in flight), which one parity cannot tell apart, so the
        // last PV has a barrier of its own.
        if (ok) ok = mbar_wait(smem_u32(&tail->o_final[t]), 0, abort, p.status,
                               ST_TIMEOUT_SOFTMAX, 0x20000 | t);
        if (threadIdx.x == 32 * kSoftmaxWarp0) trace_stamp(p.trace, 2);
        if (threadIdx.x == 32 * (kSoftmaxWarp0 + 4)) trace_stamp(p.trace, 3);
        ok = __all_sync(kFull, ok);
        float o[HD];
        if (ok) {
            tc_fence_after();
            tmem_ld32(o_col, *reinterpret_cast<uint32_t(*)[32]>(o));
            tmem_ld32(o_col + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
            tmem_wait_ld();
        }
        const int crow = t * BM + row;  // row within the CTA's ROWS
        const int unit = c_unit(), split = c_split(), nsplit = c_nsplit();
        const int head = c_head(unit), batch = c_batch(unit);
        const int grow = c_q0(unit) + crow;
        const bool store = grow < p.row_end && grow < p.tokens;
        auto row_offset = [&]() {
            const size_t esz = kOutDtype == BL_F32 ? 4 : 2;
            return esz * (static_cast<size_t>(batch) * p.out_batch_stride +
                          static_cast<size_t>(grow) * p.out_row_stride +
                          static_cast<size_t>(head - p.out_head_base) * HD);
        };
        // The finished row into `out` (per thread; `valid` rows only). The
        // head-parallel exchange instead stores into every rank's output,
        // warp by warp: the warp's 32 rows (one per lane) are staged in its
        // quarter of this tile's Q buffer (free once the tile's last scores
        // are consumed) and each store instruction then writes four whole
        // 128-byte rows, so the writes to peers leave as full lines; the
        // ranks are visited starting with the next one so a rank's CTAs
        // spread their first stores over the peers. In that form every lane
        // of the warp must call it.
        auto store_out = [&](const float* v, float inv, bool valid) {
            if constexpr (kPeers && kOutDtype != BL_F32) {
                uint4 pk[HD / 8];
                pack_row16<kOutDtype>(v, inv, pk);
                uint8_t* stage = sQ + t * kTileBytes + sub * (32 * HD * 2);
#pragma unroll
                for (int c = 0; c < HD / 8; ++c)
                    *reinterpret_cast<uint4*>(stage + lane * (HD * 2) + ((c ^ (lane & 7)) << 4)) =
                        pk[c];
                __syncwarp();
                const unsigned long long off = row_offset();
                const int chunk = lane & 7;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int src = 4 * i + (lane >> 3);  // the lane whose row this is
                    const unsigned long long roff = __shfl_sync(0xFFFFFFFFu, off, src);
                    const bool rvalid = __shfl_sync(0xFFFFFFFFu, valid ? 1 : 0, src) != 0;
                    const uint4 val = *reinterpret_cast<const uint4*>(
                        stage + src * (HD * 2) + ((chunk ^ (src & 7)) << 4));
                    if (rvalid) {
                        for (int d = 0; d < peers.n; ++d) {
                            int r = peers.rank + 1 + d;
                            r = r >= peers.n ? r - peers.n : r;
                            *reinterpret_cast<uint4*>(peers.dst[r] + roff + (chunk << 4)) = val;
                        }
                    }
                }
                __syncwarp();
            } else {
                if (valid)
                    store_row(static_cast<uint8_t*>(p.out) + row_offset(), kOutDtype, v, inv);
            }
        };
        bool do_store = ok && store;
        float inv_l = 1.0f / l;
        if (nsplit > 1) {
            // ---------------------------------------------- split-key combine
            // Every split's partial for a row is O / l rounded to f16 (a
            // convex combination of f16 V rows, so within f16 range) and
            // (max, sum); the combiner forms
            //   O = sum_s W_s (O_s / l_s) / sum_s W_s,  W_s = 2^(m_s - M) l_s
            // over the splits in rank order, whichever form and whichever
            // CTA combines, so both forms and every row partition give the
            // same bits.
            const float il = ok && l > 0.0f ? 1.0f / l : 0.0f;
            const float mine_m = ok ? m_used : -INFINITY, mine_l = ok ? l : 0.0f;
            uint4 on[HD / 8];
#pragma unroll
            for (int k = 0; k < HD / 8; ++k)
                on[k] = make_uint4(pack_f16x2(o[8 * k] * il, o[8 * k + 1] * il),
                                   pack_f16x2(o[8 * k + 2] * il, o[8 * k + 3] * il),
                                   pack_f16x2(o[8 * k + 4] * il, o[8 * k + 5] * il),
                                   pack_f16x2(o[8 * k + 6] * il, o[8 * k + 7] * il));
            auto combine = [&](auto&& part_on, auto&& part_ml, bool valid) {
                float mxs = -INFINITY;
                for (int sp = 0; sp < nsplit; ++sp) mxs = fmaxf(mxs, part_ml(sp).x);
                float acc[HD];
#pragma unroll
                for (int k = 0; k < HD; ++k) acc[k] = 0.0f;
                float wsum = 0.0f;
#pragma unroll 1
                for (int sp = 0; sp < nsplit; ++sp) {
                    const float2 ml = part_ml(sp);
                    const float w = ml.y > 0.0f ? ex2(ml.x - mxs) * ml.y : 0.0f;
                    wsum += w;
#pragma unroll
                    for (int k = 0; k < HD / 8; ++k) {
                        const uint4 q = part_on(sp, k);
                        const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wd[e]));
                            acc[8 * k + 2 * e] += w * f.x;
                            acc[8 * k + 2 * e + 1] += w * f.y;
                        }
                    }
                }
                store_out(acc, 1.0f / wsum, valid);
            };
            do_store = false;
            if (p.cluster) {
                // ------------------------------ cluster form (distributed
                // shared memory). Rows are owned by warp: the 32 rows of warp
                // w (w = crow / 32) are combined in CTA w % splits of the
                // cluster by the threads that hold them. Every other CTA
                // pushes its partials for those rows into the owner's
                // partial area at [source][vector][slot] (source = rank with
                // the owner's own left out; vector 0..7 the f16 O / l, 8 the
                // (max, sum)), then arrives on the owner's barrier; the
                // owner waits for its arrivals only, not for the cluster.
                __syncwarp();
                cluster_wait();  // every barrier of the cluster is initialised
                if (threadIdx.x == 32 * kSoftmaxWarp0) trace_stamp(p.trace, 4);
                const int me = static_cast<int>(cluster_rank());
                const int owner = (crow >> 5) % nsplit;
                const int slot = ((crow >> 5) / nsplit) * 32 + (crow & 31);
                const int slots = ((ROWS / 32 + nsplit - 1) / nsplit) * 32;
                const uint32_t vstep = static_cast<uint32_t>(slots * 16);
                if (owner != me) {
                    const int src = me < owner ? me : me - 1;
                    const uint32_t dst = dsmem_addr(
                        smem_u32(sP) + static_cast<uint32_t>((src * kPartVecs * slots + slot) * 16),
                        static_cast<uint32_t>(owner));
                    if (store) {
#pragma unroll
                        for (int k = 0; k < HD / 8; ++k) dsmem_st4u(dst + k * vstep, on[k]);
                        dsmem_st2(dst + (HD / 8) * vstep, mine_m, mine_l);
                    }
                    fence_cluster();
                    __syncwarp();
                    if (lane == 0)
                        mbar_arrive_remote(dsmem_addr(smem_u32(&tail->parts_full),
                                                      static_cast<uint32_t>(owner)));
                } else {
                    const bool got = mbar_wait_cluster(smem_u32(&tail->parts_full), 0, abort,
                                                       p.status, ST_TIMEOUT_SOFTMAX, 0x30000 | t);
                    if (threadIdx.x == 32 * kSoftmaxWarp0) trace_stamp(p.trace, 5);
                    // the exchange's stores are warp-collective: the whole
                    // warp combines, rows past the end are not stored
                    if (kPeers ? __all_sync(0xFFFFFFFFu, got) : (got && store)) {
                        const uint4* part = reinterpret_cast<const uint4*>(sP);
                        auto at = [&](int sp, int v) -> const uint4& {
                            const int src = sp < me ? sp : sp - 1;
                            return part[(src * kPartVecs + v) * slots + slot];
                        };
                        combine(
                            [&](int sp, int k) { return sp == me ? on[k] : at(sp, k); },
                            [&](int sp) {
                                if (sp == me) return make_float2(mine_m, mine_l);
                                const uint4 q = at(sp, HD / 8);
                                return make_float2(__uint_as_float(q.x), __uint_as_float(q.y));
                            },
                            store);
                    }
                }
                if (threadIdx.x == 32 * kSoftmaxWarp0) trace_stamp(p.trace, 6);
            } else {
                // ------------------------------ workspace form: partials in
                // the caller's buffer, the last CTA of the group combines (an
                // atomic counter; nothing waits)
                // (the uniform grid: every group has p.splits splits)
                const size_t u = static_cast<size_t>(unit);
                uint4* po = p.part_o + ((u * p.splits + split) * ROWS + crow) * (HD / 8);
                float2* pml = p.part_ml + (u * p.splits + split) * ROWS + crow;
#pragma unroll
                for (int k = 0; k < HD / 8; ++k) po[k] = on[k];
                *pml = make_float2(mine_m, mine_l);
                __threadfence();
                softmax_bar<QT>();
                if (threadIdx.x == 32 * kSoftmaxWarp0) {
                    const unsigned prev = atomicAdd(p.counters + u, 1u);
                    tail->last = prev == static_cast<unsigned>(p.splits) - 1;
                }
                softmax_bar<QT>();
                if (tail->last) {
                    __threadfence();
                    if (kPeers || store) {
                        const uint4* bo = p.part_o + (u * p.splits * ROWS + crow) * (HD / 8);
                        const float2* bml = p.part_ml + u * p.splits * ROWS + crow;
                        combine([&](int sp, int k) { return __ldcg(bo + static_cast<size_t>(sp) * ROWS * (HD / 8) + k); },
                                [&](int sp) { return __ldcg(bml + static_cast<size_t>(sp) * ROWS); },
                                store);
                    }
                    if (threadIdx.x == 32 * kSoftmaxWarp0) p.counters[u] = 0u;  // self-cleaning
                }
            }
        }
        if (kPeers) {
            if (nsplit == 1) store_out(o, inv_l, do_store);  // warp-collective
        } else if (do_store) {
            store_out(o, inv_l, true);
        }
        // head-parallel exchange: trace slot 6 is the first softmax warp
        // past its row stores
        if (kPeers && threadIdx.x == 32 * kSoftmaxWarp0) trace_stamp(p.trace, 6);
        // an unsplit group in a cluster of a mixed grid: the wait of the
        // cluster barrier arrived on at set-up (no remote access follows)
        if (p.cluster && nsplit == 1) {
            __syncwarp();
            cluster_wait();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
    if (threadIdx.x == 0) trace_stamp(p.trace, 7);
}

struct Plan {
    int qt;      // query tiles per CTA
    int rows;    // query rows per CTA
    int splits;
    int q_ctas;
    int kv_tiles;
    size_t units;
    size_t bytes;    // workspace
    int head_units;  // mixed grid: the unsplit groups before the split ones (0: uniform)
};

Plan plan(const bl_attention_args& a, int splits, int qt) {
    Plan pl{};
    pl.qt = qt == 1 ? 1 : 2;
    pl.rows = BM * pl.qt;
    pl.q_ctas = static_cast<int>((a.row_end - a.row_begin + pl.rows - 1) / pl.rows);
    pl.kv_tiles = static_cast<int>((a.tokens + BN - 1) / BN);
    pl.units = static_cast<size_t>(a.batch) * (a.head_end - a.head_begin) * pl.q_ctas;
    pl.splits = splits < 1 ? 1 : (splits > pl.kv_tiles ? pl.kv_tiles : splits);
    // per unit: splits x rows of f16 O / l (HD x 2 bytes) and (max, sum)
    pl.bytes = pl.splits > 1 ? pl.units * (static_cast<size_t>(pl.splits) * pl.rows *
                                               (HD * 2 + 2 * sizeof(float)) +
                                           sizeof(unsigned))
                             : 0;
    return pl;
}

// The workspace: f16 O / l, then (max, sum), then one counter per unit.
size_t part_o_bytes(const Plan& pl) { return pl.units * pl.splits * pl.rows * HD * 2; }
size_t counters_offset(const Plan& pl) {
    return part_o_bytes(pl) + pl.units * pl.splits * pl.rows * 2 * sizeof(float);
}

int max_active_clusters(int qt, int splits);

// Estimated time (us) of one launch: a fixed launch cost plus waves of
// co-resident CTAs (clusters) times a wave's length, a wave being the key
// steps of one CTA, its set-up and drain, and the split combine. Unsplit and
// in the workspace form one CTA per SM. Fitted on B200 to launches replayed
// back to back in a CUDA graph (T = 1370 with 6 heads, T = 5477 with 2 to 16
// heads; one or two query tiles, 1 to 8 splits, both combine forms): a
// 128-key step takes 1.06 us with one query tile and 1.47 us with two; the
// cluster combine about 1.0 and 2.8 us; the workspace combine, where the
// last CTA of a group reads every split's partials back, 3.5 us and
// 6 + 1.5 (splits - 2) us.
constexpr double kStepUs[2] = {1.06, 1.47};
constexpr double kLaunchUs = 4.0;
constexpr double kWaveUs = 1.0;
double combine_us(const Plan& pl, bool cluster) {
    if (pl.splits < 2) return 0.0;
    if (cluster) return pl.qt == 1 ? 1.0 : 2.8;
    return pl.qt == 1 ? 3.5 : 6.0 + 1.5 * (pl.splits - 2);
}
double estimate_us(const Plan& pl, bool cluster) {
    if (pl.head_units > 0) {
        // mixed grid: full waves of unsplit groups in clusters, then the
        // remaining groups split, one cluster each
        const long long per_wave = max_active_clusters(pl.qt, pl.splits);
        if (per_wave <= 0) return -1.0;
        const long long head_waves = pl.head_units / (per_wave * pl.splits);
        const long long rest = static_cast<long long>(pl.units) - pl.head_units;
        const long long tail_waves = (rest + per_wave - 1) / per_wave;
        const int steps = (pl.kv_tiles + pl.splits - 1) / pl.splits;
        return kLaunchUs +
               static_cast<double>(head_waves) * (pl.kv_tiles * kStepUs[pl.qt - 1] + kWaveUs) +
               static_cast<double>(tail_waves) *
                   (steps * kStepUs[pl.qt - 1] + kWaveUs + combine_us(pl, true));
    }
    const long long ctas = static_cast<long long>(pl.units) * pl.splits;
    long long waves;
    if (cluster && pl.splits > 1) {
        const long long per_wave = max_active_clusters(pl.qt, pl.splits);
        if (per_wave <= 0) return -1.0;
        waves = (static_cast<long long>(pl.units) + per_wave - 1) / per_wave;
    } else {
        waves = (ctas + 147) / 148;
    }
    const int steps = (pl.kv_tiles + pl.splits - 1) / pl.splits;
    return kLaunchUs + static_cast<double>(waves) *
                           (steps * kStepUs[pl.qt - 1] + kWaveUs + combine_us(pl, cluster));
}

// Query tiles per CTA and key splits: as asked (nonzero fields), else the
// pair with the least estimated time. With a workspace (workspace_bytes > 0)
// the splits combine through it and a split count whose partials do not fit
// is not considered; without one the splits of a query group form a cluster
// (at most kMaxClusterSplits). Ties keep the earlier candidate (two query
// tiles first, fewer splits first), so asking again with a workspace of
// exactly the size the first answer needs gives the same answer.
// With `mixed` (the cluster form with the split count left automatic) the
// candidates also include mixed grids: as many groups as fill whole waves of
// clusters run unsplit and only the remainder is split, so the last wave is
// short instead of a third full.
struct Choice {
    int qt, splits, head_units;
};
Choice choose(const bl_attention_args& a, uint64_t workspace_bytes, bool mixed = false) {
    const int qts[2] = {2, 1};
    Choice best{a.query_tiles == 1 ? 1 : 2, a.kv_splits > 0 ? static_cast<int>(a.kv_splits) : 1, 0};
    double best_t = -1.0;
    const bool cluster = workspace_bytes == 0;
    for (int qt : qts) {
        if (a.query_tiles != 0 && static_cast<int>(a.query_tiles) != qt) continue;
        const Plan p1 = plan(a, 1, qt);
        int lo = 1, hi = std::max(1, p1.kv_tiles / 2);  // at least two key tiles per split
        if (cluster) hi = std::min(hi, kMaxClusterSplits);
        if (a.kv_splits > 0) lo = hi = static_cast<int>(a.kv_splits);
        for (int sp = lo; sp <= hi; ++sp) {
            const Plan pl = plan(a, sp, qt);
            if (!cluster && pl.bytes > workspace_bytes) continue;
            const double t = estimate_us(pl, cluster);
            if (t < 0.0) continue;
            if (best_t < 0.0 || t < best_t) best = Choice{qt, pl.splits, 0}, best_t = t;
        }
        if (!(mixed && cluster && a.kv_splits == 0)) continue;
        for (int sp = 2; sp <= hi; ++sp) {
            Plan pl = plan(a, sp, qt);
            if (pl.splits != sp) continue;
            const long long wave = static_cast<long long>(max_active_clusters(qt, sp)) * sp;
            if (wave <= 0) continue;
            pl.head_units = static_cast<int>(static_cast<long long>(pl.units) / wave * wave);
            if (pl.head_units == 0 || static_cast<size_t>(pl.head_units) == pl.units) continue;
            const double t = estimate_us(pl, true);
            if (t >= 0.0 && t < best_t) best = Choice{qt, sp, pl.head_units}, best_t = t;
        }
    }
    return best;
}

int validate(const bl_attention_args& a) {
    if (a.head_dim != HD) return fail(BL_ERR_UNSUPPORTED, "attention: head_dim %u (only 64)", a.head_dim);
    if (a.batch == 0 || a.tokens == 0 || a.heads == 0)
        return fail(BL_ERR_INVALID, "attention: zero dimension");
    if (a.query_tiles > 2)
        return fail(BL_ERR_INVALID, "attention: %u query tiles per CTA (0, 1 or 2)", a.query_tiles);
    if (a.head_begin >= a.head_end || a.head_end > a.heads)
        return fail(BL_ERR_INVALID, "attention: heads [%u, %u) outside [0, %u)", a.head_begin,
                    a.head_end, a.heads);
    if (a.row_begin >= a.row_end || a.row_end > a.tokens)
        return fail(BL_ERR_INVALID, "attention: rows [%u, %u) outside [0, %u)", a.row_begin,
                    a.row_end, a.tokens);
    return BL_OK;
}

template <int QT>
int make_launch(int out_dtype, bool peers, dim3 grid, const Plan& pl, bool cluster,
                const CUtensorMap& tm_q, const CUtensorMap& tm, const Params& p,
                const PeerParams& pq, Launch* out) {
    using Sh = Shape<QT>;
    auto kern = peers ? (out_dtype == BL_F16 ? attention_fwd<QT, BL_F16, true>
                                             : attention_fwd<QT, BL_BF16, true>)
              : out_dtype == BL_F32 ? attention_fwd<QT, BL_F32>
              : out_dtype == BL_F16 ? attention_fwd<QT, BL_F16>
                                    : attention_fwd<QT, BL_BF16>;
    constexpr size_t smem = kSmemBytes<QT>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
    if constexpr (Sh::kRegSplit) {
        // setmaxnreg.inc draws on the block's launch allocation: the split is
        // sized for exactly kLaunchRegs per thread, so refuse any other build.
        cudaFuncAttributes fa{};
        BL_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
        if (fa.numRegs != Sh::kLaunchRegs)
            return fail(BL_ERR_UNSUPPORTED,
                        "attention: kernel built with %d registers per thread, the register "
                        "split needs exactly %d",
                        fa.numRegs, Sh::kLaunchRegs);
    }
    out->op = 1;
    const CUtensorMap tq = tm_q, tk = tm;
    if (cluster) {
        const dim3 cdim = pl.head_units > 0 ? dim3(pl.splits, 1, 1) : dim3(1, 1, pl.splits);
        out->run = [=](cudaStream_t s) {
            return launch_k_cluster(kern, grid, dim3(Sh::kThreads), cdim, smem, s, tq, tk, tk, p,
                                    pq);
        };
    } else {
        out->run = [=](cudaStream_t s) {
            return launch_k(kern, grid, dim3(Sh::kThreads), smem, s, tq, tk, tk, p, pq);
        };
    }
    return BL_OK;
}

int prepare(const bl_attention_args& a, void* workspace, uint64_t workspace_bytes, Launch* out,
            const PeerParams* peers = nullptr) {
    int rc = validate(a);
    if (rc != BL_OK) return rc;
    if (a.qk_dtype != BL_F16 && a.qk_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "attention: Q/K dtype %d (f16 or bf16)", a.qk_dtype);
    if (a.v_dtype != BL_F16)
        return fail(BL_ERR_UNSUPPORTED, "attention: V dtype %d (f16 only)", a.v_dtype);
    if (a.out_dtype != BL_F32 && a.out_dtype != BL_F16 && a.out_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "attention: out dtype %d", a.out_dtype);
    if (!(a.scale > 0.0f) || !isfinite(a.scale))
        return fail(BL_ERR_INVALID, "attention: scale must be finite and positive");
    if (a.qkv == nullptr || (a.out == nullptr && peers == nullptr))
        return fail(BL_ERR_INVALID, "attention: null pointer");
    const uint64_t row = a.qkv_row_stride ? a.qkv_row_stride : 3ull * a.heads * HD;
    const uint64_t orow = a.out_row_stride ? a.out_row_stride : 1ull * a.heads * HD;
    if (row < 3ull * a.heads * HD || row % 8 != 0)
        return fail(BL_ERR_INVALID, "attention: qkv row stride %llu", (unsigned long long)row);
    if (a.out_head_base > a.head_begin ||
        orow < 1ull * (a.head_end - a.out_head_base) * HD ||
        (orow * dtype_size(a.out_dtype)) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(a.out) & 15u) != 0)
        return fail(BL_ERR_INVALID, "attention: output stride/alignment");
    if (peers != nullptr) {
        if (a.out_dtype == BL_F32)
            return fail(BL_ERR_UNSUPPORTED, "attention: the peer exchange stores 16-bit rows");
        if (peers->n < 1 || peers->n > kMaxPeers || peers->rank < 0 || peers->rank >= peers->n)
            return fail(BL_ERR_INVALID, "attention: rank %d of %d peers", peers->rank, peers->n);
        for (int r = 0; r < peers->n; ++r)
            if (peers->dst[r] == nullptr || (reinterpret_cast<uintptr_t>(peers->dst[r]) & 15u) ||
                peers->flag_at[r] == nullptr)
                return fail(BL_ERR_INVALID, "attention: peer %d has no aligned output", r);
    }

    // Query tiles per CTA and key splits: as asked, or automatic (0). With
    // a workspace the partials go through it (global combine); without one
    // the splits of a query group form a thread-block cluster that combines
    // in distributed shared memory.
    const Choice ch = choose(a, workspace != nullptr ? workspace_bytes : 0, true);
    Plan pl = plan(a, ch.splits, ch.qt);
    pl.head_units = ch.head_units;
    const bool cluster = pl.splits > 1 && workspace == nullptr;
    if (cluster && pl.splits > kMaxClusterSplits)
        return fail(BL_ERR_CAPACITY,
                    "attention: %d key splits exceed a cluster (%d); give a %zu-byte workspace",
                    pl.splits, kMaxClusterSplits, pl.bytes);
    if (pl.splits > 1 && !cluster) {
        if (workspace_bytes < pl.bytes)
            return fail(BL_ERR_CAPACITY, "attention: %d key splits need a %zu-byte workspace",
                        pl.splits, pl.bytes);
        if (reinterpret_cast<uintptr_t>(workspace) & 255u)
            return fail(BL_ERR_INVALID, "attention: workspace must be 256-byte aligned");
    }

    CUtensorMap tm, tm_q;  // K / V tiles; the CTA's query tiles as one box
    const uint64_t dims[3] = {row, a.tokens, a.batch};
    const uint64_t strides[2] = {row * 2, row * 2 * a.tokens};
    const uint32_t box[3] = {HD, BM, 1};
    rc = make_tmap_16bit_3d(&tm, a.qkv, dims, strides, box);
    if (rc != BL_OK) return rc;
    const uint32_t qbox[3] = {HD, static_cast<uint32_t>(pl.rows), 1};
    rc = make_tmap_16bit_3d(&tm_q, a.qkv, dims, strides, qbox);
    if (rc != BL_OK) return rc;

    Params p{};
    p.tokens = static_cast<int>(a.tokens);
    p.head_begin = static_cast<int>(a.head_begin);
    p.heads_rel = static_cast<int>(a.head_end - a.head_begin);
    p.row_begin = static_cast<int>(a.row_begin);
    p.row_end = static_cast<int>(a.row_end);
    p.q_col0 = 0;
    p.k_col0 = static_cast<int>(a.heads * HD);
    p.v_col0 = static_cast<int>(2 * a.heads * HD);
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.qk_fmt = a.qk_dtype == BL_BF16 ? 1 : 0;
    p.out = a.out;
    p.out_row_stride = static_cast<long long>(orow);
    p.out_batch_stride = static_cast<long long>(orow) * a.tokens;
    p.out_head_base = static_cast<int>(a.out_head_base);
    p.splits = pl.splits;
    p.cluster = cluster ? 1 : 0;
    p.kv_tiles = pl.kv_tiles;
    p.head_units = cluster ? pl.head_units : 0;
    p.q_ctas = pl.q_ctas;
    if (pl.splits > 1 && !cluster) {
        uint8_t* ws = static_cast<uint8_t*>(workspace);
        p.part_o = reinterpret_cast<uint4*>(ws);
        p.part_ml = reinterpret_cast<float2*>(ws + part_o_bytes(pl));
        p.counters = reinterpret_cast<unsigned*>(ws + counters_offset(pl));
    }
    p.trace = reinterpret_cast<unsigned long long*>(a.trace);
    p.status = status_ptr();
    const PeerParams pq = peers != nullptr ? *peers : PeerParams{};

    // the uniform grid: (query groups, heads, batch x splits); the mixed
    // grid: the unsplit groups, then `splits` CTAs for each remaining group
    const dim3 grid = p.head_units > 0
                          ? dim3(static_cast<unsigned>(p.head_units +
                                                       (pl.units - p.head_units) * pl.splits))
                          : dim3(pl.q_ctas, a.head_end - a.head_begin, a.batch * pl.splits);
    if (grid.y > 65535 || grid.z > 65535 || pl.units * pl.splits >= (1u << 31))
        return fail(BL_ERR_INVALID, "attention: grid too large");
    return pl.qt == 1 ? make_launch<1>(a.out_dtype, peers != nullptr, grid, pl, cluster, tm_q, tm, p,
                                       pq, out)
                      : make_launch<2>(a.out_dtype, peers != nullptr, grid, pl, cluster, tm_q, tm, p,
                                       pq, out);
}

// How many clusters of `splits` CTAs (this kernel's shared memory, one CTA
// per SM) the B200 runs at once; clusters must sit within one GPC, so this
// is below 148 / splits. Queried once per (query tiles, split count).
template <int QT>
int query_active_clusters(int splits) {
    auto kern = attention_fwd<QT, BL_F32>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes<QT>)) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(1, 1, splits);
    cfg.blockDim = dim3(Shape<QT>::kThreads);
    cfg.dynamicSmemBytes = kSmemBytes<QT>;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = splits;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

int max_active_clusters(int qt, int splits) {
    static int cache[2][kMaxClusterSplits + 1] = {};
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    if (splits < 1 || splits > kMaxClusterSplits || qt < 1 || qt > 2) return 0;
    int& c = cache[qt - 1][splits];
    if (c == 0) {
        const int n = qt == 1 ? query_active_clusters<1>(splits) : query_active_clusters<2>(splits);
        c = n > 0 ? n : -1;
    }
    return c > 0 ? c : 0;
}

}  // namespace attn

void attention_resolve(bl_attention_args& a, uint64_t workspace_bytes) {
    const attn::Choice ch = attn::choose(a, workspace_bytes);
    a.query_tiles = static_cast<uint32_t>(ch.qt);
    a.kv_splits = static_cast<uint32_t>(ch.splits);
}

int prepare_attention(const bl_attention_args& a, Launch* out) {
    return attn::prepare(a, a.workspace, a.workspace_bytes, out);
}

}  // namespace bl

// ---------------------------------------------------------------- no-alloc
// bl_attention_noalloc: the same kernel with its split-key scratch in a
// file-scope device array instead of a caller-owned workspace, for callers
// that cannot allocate device memory (see the header).
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB
// Every GPU that loads this library holds this array until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
struct NoAllocSetup {
    unsigned long long ctx_id = 0;  // the device context the address belongs to
    void* addr = nullptr;
};
NoAllocSetup g_noalloc[64];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// The unique id of the calling thread's current CUDA context (cuCtxGetId):
// a device reset destroys the primary context and the next one gets a new
// id, so an address looked up in the old one is never reused.
int current_context_id(unsigned long long* id) {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    if (get_current == nullptr || get_id == nullptr) {
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess ||
            cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
            q2 != cudaDriverEntryPointSuccess)
            return bl::fail(BL_ERR_CUDA, "no-alloc attention: cuCtxGetCurrent/cuCtxGetId unavailable");
        get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
        get_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS)
        return bl::fail(BL_ERR_CUDA, "no-alloc attention: no current CUDA context");
    return BL_OK;
}

// The array's device address on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress at set-up: once per device (with that device
// current), and again only if the device's context was replaced (a device
// reset), so a call never launches on an address from a destroyed context.
int noalloc_scratch(void** out) {
    int dev = 0;
    BL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return bl::fail(BL_ERR_UNSUPPORTED, "no-alloc attention: device %d", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocSetup& su = g_noalloc[dev];
    unsigned long long ctx = 0;
    if (su.addr != nullptr) {
        int rc = current_context_id(&ctx);
        if (rc != BL_OK) return rc;
        if (ctx == su.ctx_id) {
            *out = su.addr;
            return BL_OK;
        }
    }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // loads the module if needed
    if (e != cudaSuccess || p == nullptr)
        return bl::fail(BL_ERR_CUDA, "no-alloc attention: cudaGetSymbolAddress: %s",
                        cudaGetErrorString(e));
    int rc = current_context_id(&ctx);
    if (rc != BL_OK) return rc;
    su.addr = p;
    su.ctx_id = ctx;
    *out = p;
    return BL_OK;
}
}  // namespace

extern "C" int bl_attention_noalloc(const bl_attention_args* args, void* stream) {
    using namespace bl;
    if (args == nullptr) return fail(BL_ERR_INVALID, "no-alloc attention: null args");
    int rc = attn::validate(*args);
    if (rc != BL_OK) return rc;
    // the choice bl_attention makes with a workspace of this size
    const attn::Choice ch = attn::choose(*args, kNoAllocScratchBytes);
    const attn::Plan pl = attn::plan(*args, ch.splits, ch.qt);
    if (pl.bytes > kNoAllocScratchBytes)
        return fail(BL_ERR_CAPACITY,
                    "no-alloc attention: %d key splits need %zu bytes of scratch, more than "
                    "the %zu-byte static scratch",
                    pl.splits, pl.bytes, kNoAllocScratchBytes);
    void* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch)) != BL_OK) return rc;
    Launch l;
    rc = attn::prepare(*args, scratch, kNoAllocScratchBytes, &l);
    if (rc != BL_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (pl.splits > 1) {
        // The array keeps the last call's contents: the split counters must
        // start at zero, so clear them (no allocation involved).
        BL_CUDA_TRY(cudaMemsetAsync(static_cast<unsigned char*>(scratch) + attn::counters_offset(pl),
                                    0, pl.units * sizeof(unsigned), s));
    }
    return enqueue(l, s);
}

extern "C" int bl_attention_peers(const bl_attention_args* args, bl_peers* peers,
                                  uint32_t out_col, uint32_t* slot_out, void* stream) {
    using namespace bl;
    if (args == nullptr || peers == nullptr) return fail(BL_ERR_INVALID, "peer attention: null argument");
    int dev = 0;
    BL_CUDA_TRY(cudaGetDevice(&dev));
    if (dev != peers->device)
        return fail(BL_ERR_INVALID, "peer attention: peers of device %d used on device %d",
                    peers->device, dev);
    for (uint32_t r = 0; r < peers->world; ++r)
        if (peers->base[r] == nullptr)
            return fail(BL_ERR_INVALID, "peer attention: rank %u's buffer is not mapped", r);
    bl_attention_args a = *args;
    const uint64_t orow = a.out_row_stride ? a.out_row_stride : 1ull * a.heads * attn::HD;
    const uint64_t esz = dtype_size(a.out_dtype);
    if (a.out_dtype == BL_F32)
        return fail(BL_ERR_UNSUPPORTED, "peer attention: the exchange stores 16-bit rows");
    if ((out_col * esz) % 16 != 0 ||
        out_col + 1ull * (a.head_end - a.out_head_base) * attn::HD > orow)
        return fail(BL_ERR_INVALID, "peer attention: column %u of %llu-element rows", out_col,
                    (unsigned long long)orow);
    if (1ull * a.batch * a.tokens * orow * esz > peers->slot_bytes)
        return fail(BL_ERR_CAPACITY, "peer attention: the output needs %llu bytes, a slot holds %llu",
                    (unsigned long long)(1ull * a.batch * a.tokens * orow * esz),
                    (unsigned long long)peers->slot_bytes);
    const uint32_t epoch = peers->epoch + 1;
    const uint32_t slot = epoch & 1u;
    attn::PeerParams pp{};
    pp.n = static_cast<int>(peers->world);
    pp.rank = static_cast<int>(peers->rank);
    pp.epoch = epoch;
    pp.flags = reinterpret_cast<const unsigned*>(peers->local);
    const uint64_t off = bl_peers::kHeader + slot * peers->slot_stride + out_col * esz;
    for (uint32_t r = 0; r < peers->world; ++r) {
        pp.dst[r] = peers->base[r] + off;
        pp.flag_at[r] = reinterpret_cast<unsigned*>(peers->base[r]) + peers->rank;
    }
    a.out = pp.dst[peers->rank];
    a.out_row_stride = orow;
    a.workspace = nullptr;  // key splits combine in a cluster
    a.workspace_bytes = 0;
    Launch l;
    int rc = attn::prepare(a, nullptr, 0, &l, &pp);
    if (rc != BL_OK) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    rc = enqueue(l, st);
    if (rc != BL_OK) return rc;
    // the arrival barrier; from here on the launch counts (the attention
    // grid is queued and the peers expect this rank's flag)
    peers->epoch = epoch;
    const cudaError_t e = launch_k(attn::peer_arrive_kernel, dim3(1), dim3(32), 0, st, pp,
                                   status_ptr());
    if (e != cudaSuccess)
        return fail(BL_ERR_CUDA, "peer attention: arrival barrier: %s", cudaGetErrorString(e));
    if (slot_out != nullptr) *slot_out = slot;
    return BL_OK;
}

extern "C" uint64_t bl_attention_workspace_bytes(const bl_attention_args* args) {
    if (args == nullptr || bl::attn::validate(*args) != BL_OK) return 0;
    const bl::attn::Choice ch = bl::attn::choose(*args, ~0ull);
    return bl::attn::plan(*args, ch.splits, ch.qt).bytes;
}

extern "C" int bl_attention_choice(const bl_attention_args* args, uint32_t* query_tiles,
                                   uint32_t* kv_splits, uint32_t* unsplit_groups) {
    using namespace bl;
    if (args == nullptr || query_tiles == nullptr || kv_splits == nullptr ||
        unsplit_groups == nullptr)
        return fail(BL_ERR_INVALID, "attention choice: null argument");
    int rc = attn::validate(*args);
    if (rc != BL_OK) return rc;
    const attn::Choice ch =
        attn::choose(*args, args->workspace != nullptr ? args->workspace_bytes : 0, true);
    *query_tiles = static_cast<uint32_t>(ch.qt);
    *kv_splits = static_cast<uint32_t>(attn::plan(*args, ch.splits, ch.qt).splits);
    *unsplit_groups = static_cast<uint32_t>(ch.head_units);
    return BL_OK;
}

extern "C" int bl_attention(const bl_attention_args* args, void* stream) {
    if (args == nullptr) return bl::fail(BL_ERR_INVALID, "attention: null args");
    bl::Launch l;
    int rc = bl::prepare_attention(*args, &l);
    return rc != BL_OK ? rc : bl::enqueue(l, static_cast<cudaStream_t>(stream));
}
