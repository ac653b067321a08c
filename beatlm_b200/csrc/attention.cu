// Fused non-causal attention for head_dim 64 on sm_100a: the reference's
// AttentionScores -> Scale -> Softmax -> AttentionValues chain
// (crates/beatlm-core/src/kernel.rs:722-777; CPU definition in
// crates/beatlm-bench/src/reference.rs:437-494) as one kernel with an online
// softmax, so the [tokens][heads][tokens] scores never reach memory.
//
// One CTA computes a 128-row query tile of one head of one sequence:
//   warp 0      TMA producer: Q once, then K/V tiles of 128 keys into a
//               4-stage ring (128-byte swizzle, zero fill past the last key).
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into TMEM (M=128,
//               N=128, K=64, f32), then O += P_{j-1} V_{j-1} with P read
//               from TMEM (M=128, N=64, K=128, f16) so the next score tile
//               is computed while the softmax works on this one.
//   warps 2..5  softmax, one thread per query row (TMEM lane): reads its S
//               row, updates the running max (rescaling O in TMEM only when
//               the max grew by more than 2^8), writes P as f16 over the
//               consumed S columns, and finally normalises O and stores it.
// TMEM columns: S0 [0,128), S1 [128,256), O [256,320); P_j aliases S_{j%2}.
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "host.h"

namespace bl {
namespace attn {

constexpr int BM = 128;      // query rows per CTA
constexpr int BN = 128;      // keys per tile
constexpr int HD = 64;       // head width
constexpr int STAGES = 4;    // K/V ring depth
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = BM * HD * 2;  // 16 KiB per 128x64 16-bit tile
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256;
// Lazy rescaling: the running max used for exponents may trail the true
// max by up to this (log2 units), so p <= 2^8, well inside f16.
constexpr float kRescaleThreshold = 8.0f;

struct Params {
    int tokens;
    int head_begin;
    int row_begin, row_end;
    int q_col0, k_col0, v_col0;  // element column of head 0's Q/K/V in a row
    float scale_log2;            // scale * log2(e)
    int qk_fmt;                  // 0 = f16, 1 = bf16
    int out_dtype;               // BL_F32 / BL_F16 / BL_BF16
    void* out;
    long long out_row_stride;    // elements
    long long out_batch_stride;  // elements
    int out_head_base;
    Status* status;
};

struct SmemTail {
    uint64_t q_full;
    uint64_t kv_full[STAGES];
    uint64_t kv_empty[STAGES];
    uint64_t s_full[2];
    uint64_t p_full[2];
    uint64_t o_done;
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

constexpr size_t kSmemBytes = 1024 /*align slack*/ + kTileBytes /*Q*/ +
                              STAGES * 2 * kTileBytes /*K,V*/ + sizeof(SmemTail);

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
    return sdesc_sw128(addr, 16, 1024);
}
// V tile [keys][64] with the 64 columns contiguous is the MN-major B operand
// of O += P V: one 128-byte swizzle atom spans N = 64, groups of 8 keys are
// 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_v(uint32_t addr) {
    return sdesc_sw128(addr, kTileBytes, 1024);
}

template <int kOutDtype>
__device__ __forceinline__ void store_row(void* base, const float* o, float inv_l);

template <>
__device__ __forceinline__ void store_row<BL_F32>(void* base, const float* o, float inv_l) {
    float4* dst = reinterpret_cast<float4*>(base);
#pragma unroll
    for (int c = 0; c < HD / 4; ++c)
        dst[c] = make_float4(o[4 * c] * inv_l, o[4 * c + 1] * inv_l, o[4 * c + 2] * inv_l,
                             o[4 * c + 3] * inv_l);
}
template <>
__device__ __forceinline__ void store_row<BL_F16>(void* base, const float* o, float inv_l) {
    uint4* dst = reinterpret_cast<uint4*>(base);
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
        const float* v = o + 8 * c;
        dst[c] = make_uint4(pack_f16x2(v[0] * inv_l, v[1] * inv_l),
                            pack_f16x2(v[2] * inv_l, v[3] * inv_l),
                            pack_f16x2(v[4] * inv_l, v[5] * inv_l),
                            pack_f16x2(v[6] * inv_l, v[7] * inv_l));
    }
}
template <>
__device__ __forceinline__ void store_row<BL_BF16>(void* base, const float* o, float inv_l) {
    uint4* dst = reinterpret_cast<uint4*>(base);
#pragma unroll
    for (int c = 0; c < HD / 8; ++c) {
        const float* v = o + 8 * c;
        dst[c] = make_uint4(pack_bf16x2(v[0] * inv_l, v[1] * inv_l),
                            pack_bf16x2(v[2] * inv_l, v[3] * inv_l),
                            pack_bf16x2(v[4] * inv_l, v[5] * inv_l),
                            pack_bf16x2(v[6] * inv_l, v[7] * inv_l));
    }
}

template <int kOutDtype>
__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd(const __grid_constant__ CUtensorMap tm_q,
                  const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = smem + kTileBytes;                       // stage s at + s*kTileBytes
    uint8_t* sV = smem + kTileBytes + STAGES * kTileBytes;  // stage s at + s*kTileBytes
    SmemTail* tail = reinterpret_cast<SmemTail*>(smem + kTileBytes + 2 * STAGES * kTileBytes);
    volatile int* abort = &tail->abort;

    const int warp = warp_id();
    const int lane = lane_id();
    const int head = p.head_begin + blockIdx.y;
    const int batch = blockIdx.z;
    const int q0 = p.row_begin + blockIdx.x * BM;
    const int n_kv = (p.tokens + BN - 1) / BN;

    const uint32_t b_q_full = smem_u32(&tail->q_full);
    const uint32_t b_o_done = smem_u32(&tail->o_done);
    const uint32_t b_drain = smem_u32(&tail->drain);

    if (threadIdx.x == 0) {
        mbar_init(b_q_full, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->kv_full[s]), 1);
            mbar_init(smem_u32(&tail->kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tail->s_full[b]), 1);
            mbar_init(smem_u32(&tail->p_full[b]), BM);
        }
        mbar_init(b_o_done, 1);
        mbar_init(b_drain, 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            tma_prefetch_desc(&tm_q);
            tma_prefetch_desc(&tm_k);
            tma_prefetch_desc(&tm_v);
            mbar_arrive_expect_tx(b_q_full, kTileBytes);
            tma_load_3d(smem_u32(sQ), &tm_q, p.q_col0 + head * HD, q0, batch, b_q_full);
            int issued[STAGES];
#pragma unroll
            for (int s = 0; s < STAGES; ++s) issued[s] = 0;
            bool ok = true;
            for (int j = 0; j < n_kv && ok; ++j) {
                const int s = j % STAGES;
                const int r = j / STAGES;
                if (r > 0)
                    ok = mbar_wait(smem_u32(&tail->kv_empty[s]), (r - 1) & 1, abort, p.status,
                                   ST_TIMEOUT_TMA, j);
                if (!ok) break;
                const uint32_t bar = smem_u32(&tail->kv_full[s]);
                mbar_arrive_expect_tx(bar, 2 * kTileBytes);
                tma_load_3d(smem_u32(sK + s * kTileBytes), &tm_k, p.k_col0 + head * HD, j * BN,
                            batch, bar);
                tma_load_3d(smem_u32(sV + s * kTileBytes), &tm_v, p.v_col0 + head * HD, j * BN,
                            batch, bar);
                issued[s] += 1;
            }
            if (*abort) {
                // Unwinding: let every copy this thread started land before
                // the CTA's shared memory is released.
                mbar_wait(b_q_full, 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0);
                for (int s = 0; s < STAGES; ++s)
                    if (issued[s] > 0)
                        mbar_wait(smem_u32(&tail->kv_full[s]), (issued[s] - 1) & 1, nullptr,
                                  p.status, ST_TIMEOUT_DRAIN, s);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc_s = idesc_f16(BM, BN, p.qk_fmt, p.qk_fmt, 0, 0);
            const uint32_t idesc_o = idesc_f16(BM, HD, 0, 0, 0, 1);
            const uint32_t q_addr = smem_u32(sQ);
            bool ok = mbar_wait(b_q_full, 0, abort, p.status, ST_TIMEOUT_MMA, 0xFFFF);
            tc_fence_after();
            auto issue_pv = [&](int i) -> bool {
                const int bb = i & 1;
                if (!mbar_wait(smem_u32(&tail->p_full[bb]), (i >> 1) & 1, abort, p.status,
                               ST_TIMEOUT_MMA, 0x10000 | i))
                    return false;
                tc_fence_after();
                const int s = i % STAGES;
                const uint32_t v_addr = smem_u32(sV + s * kTileBytes);
                const uint32_t p_col = tmem + (bb ? kColS1 : kColS0);
#pragma unroll
                for (int k = 0; k < BN / 16; ++k)
                    mma_ts(tmem + kColO, p_col + k * 8, desc_v(v_addr + k * 16 * 128), idesc_o,
                           (i > 0 || k > 0) ? 1u : 0u);
                // Only stages the producer will refill are released, so no
                // arrival lands after the CTA has finished.
                if (i + STAGES < n_kv) mma_commit(smem_u32(&tail->kv_empty[s]));
                mma_commit(b_o_done);
                return true;
            };
            for (int j = 0; j < n_kv && ok; ++j) {
                const int s = j % STAGES;
                ok = mbar_wait(smem_u32(&tail->kv_full[s]), (j / STAGES) & 1, abort, p.status,
                               ST_TIMEOUT_MMA, j);
                if (!ok) break;
                tc_fence_after();
                const int b = j & 1;
                const uint32_t k_addr = smem_u32(sK + s * kTileBytes);
                const uint32_t d = tmem + (b ? kColS1 : kColS0);
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                    mma_ss(d, desc_kmajor(q_addr + k * 32), desc_kmajor(k_addr + k * 32), idesc_s,
                           k > 0 ? 1u : 0u);
                mma_commit(smem_u32(&tail->s_full[b]));
                if (j > 0) ok = issue_pv(j - 1);
            }
            if (ok) ok = issue_pv(n_kv - 1);
            if (!ok) {
                // Unwinding: wait for the tensor core to finish what was
                // issued before TMEM is released.
                mma_commit(b_drain);
                mbar_wait(b_drain, 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0xD);
            }
        }
    } else {
        // ------------------------------------------------------ softmax
        const int sub = warp & 3;                 // TMEM sub-partition of this warp
        const int row = sub * 32 + lane;          // query row within the tile
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(sub * 32) << 16);
        const float c = p.scale_log2;
        float m_used = -INFINITY;
        float l = 0.0f;
        bool ok = true;
        constexpr unsigned kFull = 0xFFFFFFFFu;
        for (int j = 0; j < n_kv; ++j) {
            const int b = j & 1;
            ok = mbar_wait(smem_u32(&tail->s_full[b]), (j >> 1) & 1, abort, p.status,
                           ST_TIMEOUT_SOFTMAX, j);
            ok = __all_sync(kFull, ok);
            if (!ok) break;
            tc_fence_after();
            const uint32_t s_col = t_lane + (b ? kColS1 : kColS0);
            uint32_t s[BN];
            tmem_ld32(s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(s + 0));
            tmem_ld32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
            tmem_ld32(s_col + 64, *reinterpret_cast<uint32_t(*)[32]>(s + 64));
            tmem_ld32(s_col + 96, *reinterpret_cast<uint32_t(*)[32]>(s + 96));
            tmem_wait_ld();
            const int valid = min(BN, p.tokens - j * BN);
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < BN; ++i) {
                float v = (i < valid) ? __uint_as_float(s[i]) : -INFINITY;
                s[i] = __float_as_uint(v);
                mx = fmaxf(mx, v);
            }
            // Lazy rescaling, decided per row; the O read-modify-write is a
            // warp-collective TMEM access, so a warp does it when any of its
            // rows needs it (the others multiply by 1, which is exact).
            const float m_new = fmaxf(m_used, mx * c);
            const bool need = m_new > m_used + kRescaleThreshold;
            float alpha = 1.0f;
            if (need) {
                alpha = ex2(m_used - m_new);
                l *= alpha;
                m_used = m_new;
            }
            if (j > 0 && __any_sync(kFull, need)) {
                ok = mbar_wait(b_o_done, (j - 1) & 1, abort, p.status, ST_TIMEOUT_SOFTMAX,
                               0x10000 | j);
                ok = __all_sync(kFull, ok);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t o[32];
                    tmem_ld32(t_lane + kColO + 32 * h, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(t_lane + kColO + 32 * h, o);
                }
                tmem_wait_st();
            }
            float sum = 0.0f;
            uint32_t pk[BN / 2];
#pragma unroll
            for (int i = 0; i < BN / 2; ++i) {
                const float p0 = ex2(fmaf(__uint_as_float(s[2 * i]), c, -m_used));
                const float p1 = ex2(fmaf(__uint_as_float(s[2 * i + 1]), c, -m_used));
                sum += p0 + p1;
                pk[i] = pack_f16x2(p0, p1);
            }
            l += sum;
            tmem_st32(s_col + 0, *reinterpret_cast<uint32_t(*)[32]>(pk + 0));
            tmem_st32(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(pk + 32));
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(smem_u32(&tail->p_full[b]));
        }
        if (ok) ok = mbar_wait(b_o_done, (n_kv - 1) & 1, abort, p.status, ST_TIMEOUT_SOFTMAX,
                               0x20000);
        ok = __all_sync(kFull, ok);
        if (ok) {
            tc_fence_after();
            float o[HD];
            tmem_ld32(t_lane + kColO, *reinterpret_cast<uint32_t(*)[32]>(o));
            tmem_ld32(t_lane + kColO + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
            tmem_wait_ld();
            const int grow = q0 + row;
            if (grow < p.row_end && grow < p.tokens) {
                const float inv_l = 1.0f / l;
                const size_t esz = kOutDtype == BL_F32 ? 4 : 2;
                uint8_t* dst = static_cast<uint8_t*>(p.out) +
                               esz * (static_cast<size_t>(batch) * p.out_batch_stride +
                                      static_cast<size_t>(grow) * p.out_row_stride +
                                      static_cast<size_t>(head - p.out_head_base) * HD);
                store_row<kOutDtype>(dst, o, inv_l);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

int prepare(const bl_attention_args& a, Launch* out) {
    if (a.head_dim != HD) return fail(BL_ERR_UNSUPPORTED, "attention: head_dim %u (only 64)", a.head_dim);
    if (a.batch == 0 || a.tokens == 0 || a.heads == 0)
        return fail(BL_ERR_INVALID, "attention: zero dimension");
    if (a.head_begin >= a.head_end || a.head_end > a.heads)
        return fail(BL_ERR_INVALID, "attention: heads [%u, %u) outside [0, %u)", a.head_begin,
                    a.head_end, a.heads);
    if (a.row_begin >= a.row_end || a.row_end > a.tokens)
        return fail(BL_ERR_INVALID, "attention: rows [%u, %u) outside [0, %u)", a.row_begin,
                    a.row_end, a.tokens);
    if (a.qk_dtype != BL_F16 && a.qk_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "attention: Q/K dtype %d (f16 or bf16)", a.qk_dtype);
    if (a.v_dtype != BL_F16)
        return fail(BL_ERR_UNSUPPORTED, "attention: V dtype %d (f16 only)", a.v_dtype);
    if (a.out_dtype != BL_F32 && a.out_dtype != BL_F16 && a.out_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "attention: out dtype %d", a.out_dtype);
    if (!(a.scale > 0.0f) || !isfinite(a.scale))
        return fail(BL_ERR_INVALID, "attention: scale must be finite and positive");
    if (a.qkv == nullptr || a.out == nullptr) return fail(BL_ERR_INVALID, "attention: null pointer");
    const uint64_t row = a.qkv_row_stride ? a.qkv_row_stride : 3ull * a.heads * HD;
    const uint64_t orow = a.out_row_stride ? a.out_row_stride : 1ull * a.heads * HD;
    if (row < 3ull * a.heads * HD || row % 8 != 0)
        return fail(BL_ERR_INVALID, "attention: qkv row stride %llu", (unsigned long long)row);
    if (a.out_head_base > a.head_begin ||
        orow < 1ull * (a.head_end - a.out_head_base) * HD ||
        (orow * dtype_size(a.out_dtype)) % 16 != 0 ||
        (reinterpret_cast<uintptr_t>(a.out) & 15u) != 0)
        return fail(BL_ERR_INVALID, "attention: output stride/alignment");

    CUtensorMap tm;
    const uint64_t dims[3] = {row, a.tokens, a.batch};
    const uint64_t strides[2] = {row * 2, row * 2 * a.tokens};
    const uint32_t box[3] = {HD, BM, 1};
    int rc = make_tmap_16bit_3d(&tm, a.qkv, dims, strides, box);
    if (rc != BL_OK) return rc;

    Params p{};
    p.tokens = static_cast<int>(a.tokens);
    p.head_begin = static_cast<int>(a.head_begin);
    p.row_begin = static_cast<int>(a.row_begin);
    p.row_end = static_cast<int>(a.row_end);
    p.q_col0 = 0;
    p.k_col0 = static_cast<int>(a.heads * HD);
    p.v_col0 = static_cast<int>(2 * a.heads * HD);
    p.scale_log2 = a.scale * 1.4426950408889634f;
    p.qk_fmt = a.qk_dtype == BL_BF16 ? 1 : 0;
    p.out_dtype = a.out_dtype;
    p.out = a.out;
    p.out_row_stride = static_cast<long long>(orow);
    p.out_batch_stride = static_cast<long long>(orow) * a.tokens;
    p.out_head_base = static_cast<int>(a.out_head_base);
    p.status = status_ptr();

    dim3 grid((a.row_end - a.row_begin + BM - 1) / BM, a.head_end - a.head_begin, a.batch);
    if (grid.y > 65535 || grid.z > 65535) return fail(BL_ERR_INVALID, "attention: grid too large");
    auto kern = a.out_dtype == BL_F32   ? attention_fwd<BL_F32>
                : a.out_dtype == BL_F16 ? attention_fwd<BL_F16>
                                        : attention_fwd<BL_BF16>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kSmemBytes)));
    out->op = 1;
    out->run = [=](cudaStream_t s) {
        kern<<<grid, kThreads, kSmemBytes, s>>>(tm, tm, tm, p);
        return cudaGetLastError();
    };
    return BL_OK;
}

}  // namespace attn

int prepare_attention(const bl_attention_args& a, Launch* out) { return attn::prepare(a, out); }

}  // namespace bl

extern "C" int bl_attention(const bl_attention_args* args, void* stream) {
    if (args == nullptr) return bl::fail(BL_ERR_INVALID, "attention: null args");
    bl::Launch l;
    int rc = bl::prepare_attention(*args, &l);
    return rc != BL_OK ? rc : bl::enqueue(l, static_cast<cudaStream_t>(stream));
}
