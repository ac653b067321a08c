// tcgen05 GEMM for the ViT linear layers, with the reference's fusions:
//   C[M][N] = epilogue(A[M][K] . B[N][K]^T)
// A is either a 16-bit activation loaded by TMA, or produced in the kernel by
// a LayerNorm prologue from the f32 residual stream (the LN before the QKV
// projection and before fc1), so the normalised activation never reaches
// memory. B is the weight in [out][in] order (K-major), loaded by TMA.
// The epilogue chain is the reference's Epilogue (kernel.rs:1595-1615) in
// its canonical order: + bias (the MatMul's own), activation (ReLU, GELU
// tanh, GELU erf), Scale, ChannelScale (LayerScale), Add (residual), then a
// store in f32, f16 or bf16 (optionally a second type from a given column,
// for the packed Q|K|V rows whose V part is f16).
//
// CTA: warp 0 TMA producer, warp 1 MMA issuer (M=128, N=BN, K=16 steps,
// f32 accumulator in TMEM), warps 2..5 LN producers (LN mode) and then the
// epilogue, one accumulator row (TMEM lane) per thread. Tiles 128 x BN x 64,
// a 4-stage ring.
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <algorithm>

#include "host.h"

namespace bl {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kMaxStages = 8;
constexpr uint32_t kSmemLimit = 232448;  // 227 KiB of dynamic shared memory per CTA
constexpr int kThreads = 192;
constexpr int kMaxBN = 256;  // the widest tile (the persistent kernel only)
constexpr uint32_t kTileA = BM * BK * 2;  // 16 KiB

struct Params {
    int M, N, K;
    int ab_fmt;  // 0 = f16, 1 = bf16 (A and B)
    // LayerNorm prologue (LN mode only)
    const float* x;
    long long ldx;
    const float* gamma;
    const float* beta;
    float eps;
    // epilogue
    const float* bias;
    int act;
    float scale;
    const float* chan_scale;
    const void* residual;
    int res_dtype;
    long long res_ld;
    int res_period;  // residual row = out_row % res_period (0: out_row)
    void* out;
    int out_dtype;
    int out_dtype_hi;
    int split_col;
    long long out_ld;
    int out_row_offset;
    int out_group_rows;  // out_row = m + (m / group_rows) * group_gap + offset
    int out_group_gap;
    int m_tile0, m_tiles;  // row tiles [m_tile0, m_tile0 + m_tiles) of this launch (a part)
    float2* stats_out;     // [out row][stats_parts] (mean, M2) of the stored row slice
    int stats_parts;
    const float2* ln_stats;  // LN prologue: [row][ln_stats_parts] partials of x
    int ln_stats_parts;
    int tma_store;  // persistent kernel: rows leave through the output tensor map
    int weights_static;  // B and the epilogue vectors may be read before the PDL wait
    // LayerNorm of the stored rows in the epilogue (32-column tiles, one tile
    // per CTA): per-slice statistics meet in norm_stats, row tiles count their
    // published slices in norm_ctr[2 * tile] and their readers in [2 * tile + 1]
    void* norm_out;
    int norm_dtype;
    const float* norm_gamma;
    const float* norm_beta;
    float norm_eps;
    unsigned* norm_ctr;
    float2* norm_stats;
    unsigned long long* trace;  // optional per-CTA timeline (persistent kernel)
    // Stream-K (persistent kernel, sk_pieces > 1): every tile's stages are
    // cut into sk_pieces pieces, accumulated separately; slot t * sk_pieces
    // + i of sk_part holds the f32 partial sums of piece i < sk_pieces - 1
    // of tile t and sk_flag marks it written; the CTA that computes the
    // last piece adds them to its own in piece order. A slot is laid out
    // [32-column chunk][32-row quarter][4-column group][row in quarter] of
    // float4, so the 32 rows (one per lane) of a warp's access to one
    // column group are 512 contiguous bytes.
    int sk_pieces;
    float* sk_part;
    unsigned* sk_flag;
    // implicit 3x3 convolution (gemm_conv): an NHWC f32 image of conv_w
    // columns and conv_pix pixels, conv_cin channels; K columns past conv_k
    // (9 cin) are zero; conv_relu: max(x, 0) on every input value
    int conv_w, conv_pix, conv_cin, conv_k, conv_relu;
    // row reduction (generic epilogue, one column tile): out[row] =
    // act2(sum_c v[c] dot_w[c] + dot_bias), no row stored
    const float* dot_w;
    float dot_bias;
    int dot_act;
    Status* status;
};

// A stage holds KC k-blocks: KC A tiles, then KC B tiles, each a 128-byte
// swizzled K-major tile. One TMA copy brings all KC tiles of an operand (a
// 3-D view whose third dimension steps 64 columns): a thread's bulk copies
// complete one after another, each in about 530 SM clocks whatever its size
// up to 64 KiB (measured), so bytes per copy set a CTA's feed rate.
// Output staging of the persistent kernel's epilogue: one 32 x 32 block of
// up to 4-byte values per epilogue warp, stored to global memory by TMA.
constexpr uint32_t kEpiBlock = 32 * 32 * 4;
// Stream-K partial slot: floats per 32-column chunk of 128 rows
constexpr uint32_t kSkChunk = BM * 32;
// a row's float4 of column group k (0..7) in its chunk, from its row base
// (sk_row_base): 32 float4 (one per row of the quarter) per column group
constexpr uint32_t kSkGroup = 32;
__device__ __forceinline__ uint32_t sk_row_base(int row) {
    return static_cast<uint32_t>((row >> 5) * 8 * 32 + (row & 31)) * 4;  // floats
}
// At most three pieces per tile: the finishing piece loads the other two
// pieces' values of a chunk at once (registers), one L2 round trip a chunk
constexpr int kMaxSkPieces = 3;
constexpr int kMaxSkParts = kMaxSkPieces - 1;
constexpr uint32_t kEpiBytes = 4 * kEpiBlock;

template <int BN, int KC = 1, bool kEpi = false>
struct Layout {
    static constexpr uint32_t kTileB = BN * BK * 2;
    static constexpr uint32_t kStage = KC * (kTileA + kTileB);
    static constexpr uint32_t kReserve = 4096 + (kEpi ? kEpiBytes : 0);
    // As deep a TMA ring as shared memory holds (4 KiB kept for the barriers,
    // the staged epilogue vectors and the alignment slack, plus the output
    // staging).
    static constexpr int kStages =
        static_cast<int>((kSmemLimit - kReserve) / kStage) < kMaxStages
            ? static_cast<int>((kSmemLimit - kReserve) / kStage)
            : kMaxStages;
    static constexpr uint32_t kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

struct Tail {
    uint64_t full[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t acc_full[2];   // accumulator b holds a finished tile (the persistent
    uint64_t acc_empty[2];  // kernel alternates two; the one-tile kernel uses [0])
    uint64_t drain;
    uint64_t conv[kMaxStages];  // gemm_ln_staged: a stage's A tile is normalised
    uint32_t tmem_base;
    int abort;
    // the tile's bias and channel-scale columns, staged by the epilogue warps
    // while the main loop runs
    alignas(16) float bias[kMaxBN];
    alignas(16) float chan[kMaxBN];
};

template <int BN, int KC = 1, bool kEpi = false>
constexpr size_t smem_bytes() {
    using L = Layout<BN, KC, kEpi>;
    return 1024 + L::kStages * L::kStage + (kEpi ? kEpiBytes : 0) + sizeof(Tail);
}

__device__ __forceinline__ uint64_t desc_k(uint32_t addr) { return sdesc_sw128(addr, 16, 1024); }

__device__ __forceinline__ uint32_t pack2(float a, float b, int dt) {
    return dt == BL_BF16 ? pack_bf16x2(a, b) : pack_f16x2(a, b);
}

// GELU through erf, Abramowitz and Stegun 7.1.26 (the reference's
// GELU_ERF_P / GELU_ERF_A, kernel.rs:355-372), in f32 as its kernels do:
//   z = |x| / sqrt(2), t = 1 / (1 + p z),
//   q = 0.5 t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) 2^(-z^2 log2 e),
//   GELU(x) = x (1 - q) for x >= 0, x q otherwise.
// Two values at once, the arithmetic in packed f32x2 instructions; the
// reciprocal is the MUFU approximation (relative error ~2^-22, which moves
// GELU by under 5e-8 against the formula's own 1.5e-7 in erf; the bound the
// reference states for GELU, 5e-7, is tested).
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void gelu_erf2(float& x0, float& x1) {
    const float p = 0.3275911f;
    const float a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f, a4 = -1.453152027f,
                a5 = 1.061405429f;
    const unsigned long long z =
        fmul2(f2pack(fabsf(x0), fabsf(x1)), f2pack(0.70710678118654752f, 0.70710678118654752f));
    float d0, d1;
    f2unpack(ffma2(f2pack(p, p), z, f2pack(1.0f, 1.0f)), d0, d1);
    const unsigned long long t = f2pack(rcp_approx(d0), rcp_approx(d1));
    unsigned long long poly = ffma2(t, f2pack(a5, a5), f2pack(a4, a4));
    poly = ffma2(t, poly, f2pack(a3, a3));
    poly = ffma2(t, poly, f2pack(a2, a2));
    poly = ffma2(t, poly, f2pack(a1, a1));
    poly = fmul2(t, poly);
    float e0, e1;
    f2unpack(fmul2(fmul2(z, z), f2pack(-1.4426950408889634f, -1.4426950408889634f)), e0, e1);
    float q0, q1;
    f2unpack(fmul2(fmul2(f2pack(0.5f, 0.5f), poly), f2pack(ex2(e0), ex2(e1))), q0, q1);
    x0 = x0 * (x0 >= 0.0f ? 1.0f - q0 : q0);
    x1 = x1 * (x1 >= 0.0f ? 1.0f - q1 : q1);
}

__device__ __forceinline__ float gelu_tanh(float x) {
    const float k = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(k * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ void load16(const void* base, int dt, float* v) {
    // 16 consecutive values of a residual row
    if (dt == BL_F32) {
        const float4* p = static_cast<const float4*>(base);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float4 q = p[i];
            v[4 * i] = q.x; v[4 * i + 1] = q.y; v[4 * i + 2] = q.z; v[4 * i + 3] = q.w;
        }
    } else {
        const uint4* p = static_cast<const uint4*>(base);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            uint4 q = p[i];
            uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                if (dt == BL_BF16) {
                    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w[j]);
                    float2 f = __bfloat1622float2(h);
                    v[8 * i + 2 * j] = f.x; v[8 * i + 2 * j + 1] = f.y;
                } else {
                    __half2 h = *reinterpret_cast<__half2*>(&w[j]);
                    float2 f = __half22float2(h);
                    v[8 * i + 2 * j] = f.x; v[8 * i + 2 * j + 1] = f.y;
                }
            }
        }
    }
}

// Where one accumulator row (TMEM lane) of a tile goes: its output row
// (row groups and offset applied) and its residual row.
struct RowCtx {
    bool live;
    long long orow, res_row;
};

__device__ __forceinline__ RowCtx row_ctx(const Params& p, int grow) {
    RowCtx rc;
    rc.live = grow < p.M;
    rc.orow = grow;
    if (p.out_group_rows > 0)
        rc.orow = grow + static_cast<long long>(grow / p.out_group_rows) * p.out_group_gap;
    rc.orow += p.out_row_offset;
    rc.res_row = p.res_period > 0 ? rc.orow % p.res_period : rc.orow;
    return rc;
}

// The tile's bias and channel-scale columns into shared memory, by the four
// epilogue warps (threads 64..191); the caller synchronises them after.
template <int BN>
__device__ __forceinline__ void stage_vectors(const Params& p, Tail* tail, int n0) {
    static_assert(BN <= kMaxBN, "tile wider than the staged vectors");
    for (int t = static_cast<int>(threadIdx.x) - 64; t >= 0 && t < BN; t += 128) {
        tail->bias[t] = p.bias != nullptr ? __ldg(p.bias + n0 + t) : 0.0f;
        tail->chan[t] = p.chan_scale != nullptr ? __ldg(p.chan_scale + n0 + t) : 1.0f;
    }
}

// The first 32 residual columns of this thread's row, into registers.
__device__ __forceinline__ void prefetch_residual(const Params& p, const RowCtx& rc, int n0,
                                                  float* rv0) {
    if (p.residual == nullptr || !rc.live) return;
    const size_t esz = p.res_dtype == BL_F32 ? 4 : 2;
    const uint8_t* rb = static_cast<const uint8_t*>(p.residual) + esz * (rc.res_row * p.res_ld + n0);
    load16(rb, p.res_dtype, rv0);
    load16(rb + esz * 16, p.res_dtype, rv0 + 16);
}

// The epilogue chain of one accumulator row: TMEM columns 32 at a time, then
// bias, activation, scale, channel scale, residual and the store.
// `tmo` (may be null): the output tensor map. Each warp then writes its
// 32 x 32 block into `buf`, swizzled as the map's 128-byte (4-byte values) or
// 64-byte (2-byte values) swizzle lays it out, so a quarter-warp's 16-byte
// writes hit distinct banks, and one lane stores the block with first output
// row `box_row`; rows past the output are clipped by the map. Without it each
// thread stores its own row.
// EPI: the epilogue fixed at compile time, so a kernel carries only its own
// code (measured: the generic chain's size stalled instruction fetch). -1
// generic (everything decided at run time); 0 plain (bias only, 16-bit out);
// 1 bias + GELU-erf, 16-bit out; 2 bias, LayerScale and f32 residual. The
// host picks a fixed form only where the arguments match it exactly.
// kParts > 0 (stream-K): `parts` is this row's partial sums of the tile's
// other pieces, `nparts` (at most kParts) slots `part_stride` floats apart,
// added to the accumulator in slot order before anything else; a chunk's
// partials and residual are then loaded together while its accumulator
// comes (one round trip a chunk).
template <int BN, int EPI = -1, int kParts = 0>
__device__ __forceinline__ void store_tile(const Params& p, const Tail* tail, uint32_t t_lane,
                                           int n0, const RowCtx& rc, const float* rv0,
                                           const CUtensorMap* tmo = nullptr,
                                           uint8_t* buf = nullptr, int box_row = 0,
                                           float* keep = nullptr, const float* parts = nullptr,
                                           int nparts = 0, size_t part_stride = 0) {
    const bool live = rc.live;
    const long long orow = rc.orow, res_row = rc.res_row;
    const size_t res_esz = p.res_dtype == BL_F32 ? 4 : 2;
    const int lane = lane_id();
    float run_mean = 0.0f, run_m2 = 0.0f;  // row statistics of the stored slice
    float dacc = 0.0f;                     // row reduction (dot_w), in column order
    const bool add_res = (EPI < 0 ? p.residual != nullptr : EPI == 2) && live;
    // stream-K: the chunk's residual, the first chunk's from the caller (so
    // rv0 is not live across the loop), later ones loaded with the partials
    float rvc[kParts > 0 ? 32 : 1];
    if constexpr (kParts > 0) {
        if (add_res) {
#pragma unroll
            for (int i = 0; i < 32; ++i) rvc[i] = rv0[i];
        }
    }
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
        const int col = n0 + c * 32;
        // stream-K: the chunk's other addends, loaded together: the other
        // pieces' partial sums (written by other CTAs in this launch: through
        // L2 only) and, past the first chunk, whose residual the caller
        // loaded, the residual
        float4 pf[kParts > 0 ? kParts : 1][8];
        if constexpr (kParts > 0) {
#pragma unroll
            for (int q = 0; q < kParts; ++q) {
                if (q < nparts) {
                    const float4* src =
                        reinterpret_cast<const float4*>(parts + q * part_stride + c * kSkChunk);
#pragma unroll
                    for (int i = 0; i < 8; ++i) pf[q][i] = __ldcg(src + i * kSkGroup);
                }
            }
        }
        if constexpr (kParts > 0) {
            if (add_res && c > 0) {
                const uint8_t* rb = static_cast<const uint8_t*>(p.residual) +
                                    res_esz * (res_row * p.res_ld + col);
                load16(rb, p.res_dtype, rvc);
                load16(rb + res_esz * 16, p.res_dtype, rvc + 16);
            }
        }
        uint32_t r[32];
        tmem_ld32(t_lane + c * 32, r);
        tmem_wait_ld();
        if (!live && tmo == nullptr) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
        if constexpr (kParts > 0) {
#pragma unroll
            for (int q = 0; q < kParts; ++q) {
                if (q < nparts) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[4 * i] += pf[q][i].x;
                        v[4 * i + 1] += pf[q][i].y;
                        v[4 * i + 2] += pf[q][i].z;
                        v[4 * i + 3] += pf[q][i].w;
                    }
                }
            }
        }
        if (p.bias != nullptr) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const float4 b = *reinterpret_cast<const float4*>(tail->bias + c * 32 + i);
                v[i] += b.x; v[i + 1] += b.y; v[i + 2] += b.z; v[i + 3] += b.w;
            }
        }
        const int act = EPI < 0 ? p.act : EPI == 1 ? 3 : 0;
        if (act == 1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
        } else if (act == 2) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = gelu_tanh(v[i]);
        } else if (act == 3) {
#pragma unroll
            for (int i = 0; i < 32; i += 2) gelu_erf2(v[i], v[i + 1]);
        }
        if (EPI < 0 && p.scale != 1.0f) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= p.scale;
        }
        if (EPI < 0 ? p.chan_scale != nullptr : EPI == 2) {
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
                const float4 s = *reinterpret_cast<const float4*>(tail->chan + c * 32 + i);
                v[i] *= s.x; v[i + 1] *= s.y; v[i + 2] *= s.z; v[i + 3] *= s.w;
            }
        }
        if (add_res) {
            if constexpr (kParts > 0) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += rvc[i];
            } else if (c == 0) {
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += rv0[i];
            } else {
                const uint8_t* rb = static_cast<const uint8_t*>(p.residual) +
                                    res_esz * (res_row * p.res_ld + col);
                float rv[16];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    load16(rb + res_esz * 16 * h, p.res_dtype, rv);
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[16 * h + i] += rv[i];
                }
            }
        }
        if constexpr (EPI < 0 && kParts == 0) {
            if (p.dot_w != nullptr) {
                // the row reduced to one value (the host allows one column
                // tile, no tensor-map store, no statistics): nothing stored
                // but the last chunk's sum
#pragma unroll
                for (int i = 0; i < 32; i += 4) {
                    const float4 w = __ldg(reinterpret_cast<const float4*>(p.dot_w + col + i));
                    dacc = fmaf(v[i], w.x, dacc);
                    dacc = fmaf(v[i + 1], w.y, dacc);
                    dacc = fmaf(v[i + 2], w.z, dacc);
                    dacc = fmaf(v[i + 3], w.w, dacc);
                }
                if (c == BN / 32 - 1 && live) {
                    const float y = dacc + p.dot_bias;
                    static_cast<float*>(p.out)[orow] = p.dot_act ? fmaxf(y, 0.0f) : y;
                }
                continue;
            }
        }
        if (EPI < 0 && p.stats_out != nullptr) {
            // this chunk's mean and M2, merged into the slice's (Chan et al.)
            float cs = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) cs += v[i];
            const float cm = cs * (1.0f / 32.0f);
            float cm2 = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) cm2 += (v[i] - cm) * (v[i] - cm);
            const float na = 32.0f * static_cast<float>(c), nab = na + 32.0f;
            const float delta = cm - run_mean;
            run_mean += delta * (32.0f / nab);
            run_m2 += cm2 + delta * delta * (na * 32.0f / nab);
        }
        if (keep != nullptr && c == 0) {
#pragma unroll
            for (int i = 0; i < 32; ++i) keep[i] = v[i];
        }
        const int dt = EPI == 2 ? BL_F32 : col >= p.split_col ? p.out_dtype_hi : p.out_dtype;
        if (EPI >= 0 || tmo != nullptr) {
            // 4-byte blocks fill `buf`; 2-byte blocks alternate between its
            // halves, so a block is written while the previous one is still
            // being read out (a tile's first block waits for every earlier one)
            const bool wide = dt == BL_F32;
            uint8_t* blk = wide ? buf : buf + (c & 1) * (kEpiBlock / 2);
            if (lane == 0) {
                if (wide || c == 0) bulk_wait_read();
                else bulk_wait_read1();
            }
            __syncwarp();
            if (wide) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<float4*>(blk + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(blk + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
                        make_uint4(pack2(v[8 * j], v[8 * j + 1], dt),
                                   pack2(v[8 * j + 2], v[8 * j + 3], dt),
                                   pack2(v[8 * j + 4], v[8 * j + 5], dt),
                                   pack2(v[8 * j + 6], v[8 * j + 7], dt));
            }
            fence_proxy_async_smem();  // the writes above, seen by the bulk copy
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(tmo, smem_u32(blk), col, box_row);
                bulk_commit();
            }
        } else if (dt == BL_F32) {
            float4* o = reinterpret_cast<float4*>(static_cast<float*>(p.out) +
                                                  orow * p.out_ld + col);
#pragma unroll
            for (int i = 0; i < 8; ++i)
                o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
            uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) +
                                                orow * p.out_ld + col);
#pragma unroll
            for (int i = 0; i < 4; ++i)
                o[i] = make_uint4(pack2(v[8 * i], v[8 * i + 1], dt),
                                  pack2(v[8 * i + 2], v[8 * i + 3], dt),
                                  pack2(v[8 * i + 4], v[8 * i + 5], dt),
                                  pack2(v[8 * i + 6], v[8 * i + 7], dt));
        }
    }
    if (EPI < 0 && p.stats_out != nullptr && live)
        p.stats_out[orow * p.stats_parts + n0 / BN] = make_float2(run_mean, run_m2);
}

template <int BN, bool kLn>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const Params p) {
    using L = Layout<BN>;
    constexpr int STAGES = L::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    Tail* tail = reinterpret_cast<Tail*>(smem + STAGES * L::kStage);
    volatile int* abort = &tail->abort;
    auto sA = [&](int s) { return smem + s * L::kStage; };
    auto sB = [&](int s) { return smem + s * L::kStage + kTileA; };

    const int warp = warp_id();
    const int lane = lane_id();
    const int m0 = (p.m_tile0 + static_cast<int>(blockIdx.x)) * BM;
    const int n0 = blockIdx.y * BN;
    const int nk = p.K / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->full[s]), kLn ? 1 + 4 : 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        mbar_init(smem_u32(&tail->acc_full[0]), 1);
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        // descriptors are launch parameters: fetch them while the previous
        // kernel may still be running
        tma_prefetch_desc(&tm_b);
        if (!kLn) tma_prefetch_desc(&tm_a);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    pdl_trigger();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&tm_b);
            if (!kLn) tma_prefetch_desc(&tm_a);
            int loaded = 0;  // k-blocks whose loads were started
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                if (kb >= STAGES &&
                    !mbar_wait(smem_u32(&tail->empty[s]), ((kb / STAGES) - 1) & 1, abort, p.status,
                               ST_TIMEOUT_TMA, kb))
                    break;
                const uint32_t bar = smem_u32(&tail->full[s]);
                mbar_arrive_expect_tx(bar, (kLn ? 0u : kTileA) + L::kTileB);
                if (!kLn) tma_load_2d(smem_u32(sA(s)), &tm_a, kb * BK, m0, bar);
                tma_load_2d(smem_u32(sB(s)), &tm_b, kb * BK, n0, bar);
                ++loaded;
            }
            if (*abort) {
                // let every started copy land before shared memory is released
                for (int s = 0; s < STAGES && s < loaded; ++s) {
                    const int uses = (loaded - s - 1) / STAGES + 1;
                    mbar_wait(smem_u32(&tail->full[s]), (uses - 1) & 1, nullptr, p.status,
                              ST_TIMEOUT_DRAIN, s);
                }
            }
        }
    } else if (warp == 1) {
        // The whole warp runs the issuer's loop and one elected lane issues,
        // keeping descriptors warp-uniform; that lane alone waits on each
        // barrier and the vote hands its outcome to the warp.
        const bool elected = elect_one();
        const uint32_t idesc = idesc_f16(BM, BN, p.ab_fmt, p.ab_fmt, 0, 0);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            bool r = true;
            if (elected)
                r = mbar_wait(smem_u32(&tail->full[s]), (kb / STAGES) & 1, abort, p.status,
                              ST_TIMEOUT_MMA, kb);
            ok = __all_sync(0xFFFFFFFFu, r);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a = smem_u32(sA(s)), b = smem_u32(sB(s));
            if (elected) {
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    mma_ss(tmem, desc_k(a + 32 * k), desc_k(b + 32 * k), idesc,
                           (kb > 0 || k > 0) ? 1u : 0u);
                // Release the stage only if the producers will refill it, so
                // no arrival lands after the CTA has finished.
                if (kb + STAGES < nk) mma_commit(smem_u32(&tail->empty[s]));
            }
            __syncwarp();
        }
        if (elected) {
            if (ok) {
                mma_commit(smem_u32(&tail->acc_full[0]));
            } else {
                mma_commit(smem_u32(&tail->drain));
                mbar_wait(smem_u32(&tail->drain), 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0xD);
            }
        }
        __syncwarp();
    } else {
        constexpr unsigned kFull = 0xFFFFFFFFu;
        const int sub = warp & 3;
        const int row = sub * 32 + lane;
        const int grow = m0 + row;
        bool ok = true;
        if (kLn) {
            // ---------------------------------------------- LayerNorm prologue
            // Warp w normalises rows [32 w, 32 w + 32) of the tile, the lanes
            // spread along the row so every load is one coalesced segment.
            // Statistics: a one-pass sum and sum of squares of the deviations
            // from the row's first element (so a large mean does not cancel),
            // the biased variance of reference.rs:247-270; lane r keeps row r's.
            const int dt = p.ab_fmt ? BL_BF16 : BL_F16;
            const float inv_k = 1.0f / static_cast<float>(p.K);
            float my_mean = 0.0f, my_rstd = 0.0f;
            if (p.ln_stats != nullptr) {
                // the producing GEMM left (mean, M2) per row slice: combine
                // them (equal counts), lane r for row r
                const int gr = m0 + sub * 32 + lane;
                if (gr < p.M) {
                    const float2* st = p.ln_stats + static_cast<long long>(gr) * p.ln_stats_parts;
                    const float nper = static_cast<float>(p.K / p.ln_stats_parts);
                    float sm = 0.0f;
                    for (int q = 0; q < p.ln_stats_parts; ++q) sm += st[q].x;
                    const float mean = sm / static_cast<float>(p.ln_stats_parts);
                    float m2 = 0.0f;
                    for (int q = 0; q < p.ln_stats_parts; ++q) {
                        const float2 v = st[q];
                        m2 += v.y + (v.x - mean) * (v.x - mean) * nper;
                    }
                    my_mean = mean;
                    my_rstd = rsqrtf(m2 * inv_k + p.eps);
                }
            }
            for (int r = 0; r < 32 && p.ln_stats == nullptr; ++r) {
                const int gr = m0 + sub * 32 + r;
                if (gr >= p.M) break;
                const float* xr = p.x + static_cast<long long>(gr) * p.ldx;
                const float x0 = xr[0];
                float s1 = 0.0f, s2 = 0.0f;
                for (int k = 2 * lane; k < p.K; k += 64) {
                    const float2 v = *reinterpret_cast<const float2*>(xr + k);
                    const float d0 = v.x - x0, d1 = v.y - x0;
                    s1 += d0 + d1;
                    s2 += d0 * d0 + d1 * d1;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    s1 += __shfl_xor_sync(kFull, s1, o);
                    s2 += __shfl_xor_sync(kFull, s2, o);
                }
                if (lane == r) {
                    const float dm = s1 * inv_k;
                    my_mean = x0 + dm;
                    my_rstd = rsqrtf(fmaxf(s2 * inv_k - dm * dm, 0.0f) + p.eps);
                }
            }
            for (int kb = 0; kb < nk; ++kb) {
                const int s = kb % STAGES;
                // this k-block's 32 rows are loaded before the stage is
                // awaited, all at once, so one memory latency covers them
                const int k = kb * BK + 2 * lane;
                float2 xv[32];
#pragma unroll
                for (int r = 0; r < 32; ++r) {
                    const int gr = m0 + sub * 32 + r;
                    xv[r] = gr < p.M ? *reinterpret_cast<const float2*>(
                                           p.x + static_cast<long long>(gr) * p.ldx + k)
                                     : make_float2(0.0f, 0.0f);
                }
                const float2 g = __ldg(reinterpret_cast<const float2*>(p.gamma + k));
                const float2 b = __ldg(reinterpret_cast<const float2*>(p.beta + k));
                if (kb >= STAGES) {
                    ok = mbar_wait(smem_u32(&tail->empty[s]), ((kb / STAGES) - 1) & 1, abort,
                                   p.status, ST_TIMEOUT_SOFTMAX, kb);
                    ok = __all_sync(kFull, ok);
                    if (!ok) break;
                }
                uint8_t* tile = sA(s);
                // lane's 4 bytes: 16-byte chunk lane/4 of the row, XOR row%8
                const int chunk = lane >> 2, off = (lane & 3) * 4;
#pragma unroll
                for (int r = 0; r < 32; ++r) {
                    const int trow = sub * 32 + r;
                    const int gr = m0 + trow;
                    const float mean = __shfl_sync(kFull, my_mean, r);
                    const float rstd = __shfl_sync(kFull, my_rstd, r);
                    const uint32_t w =
                        gr < p.M ? pack2((xv[r].x - mean) * rstd * g.x + b.x,
                                         (xv[r].y - mean) * rstd * g.y + b.y, dt)
                                 : 0u;
                    *reinterpret_cast<uint32_t*>(tile + trow * 128 + ((chunk ^ (trow & 7)) << 4) +
                                                 off) = w;
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tail->full[s]));
            }
        }
        // -------------------------------------------------------- epilogue
        // What the epilogue reads is fetched while the main loop still runs.
        const RowCtx rc = row_ctx(p, grow);
        stage_vectors<BN>(p, tail, n0);
        asm volatile("bar.sync 1, 128;" ::: "memory");
        float rv0[32];
        prefetch_residual(p, rc, n0, rv0);
        if (ok) ok = mbar_wait(smem_u32(&tail->acc_full[0]), 0, abort, p.status, ST_TIMEOUT_SOFTMAX,
                               0xE);
        ok = __all_sync(kFull, ok);
        if (ok) {
            tc_fence_after();
            store_tile<BN>(p, tail, tmem + (static_cast<uint32_t>(sub * 32) << 16), n0, rc, rv0);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, L::kTmemCols);
    }
}

__device__ __forceinline__ bool epilogue_all(bool ok) {
    // AND of `ok` over the four epilogue warps; also their barrier
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, 128, p;\n"
        " selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(ok ? 1u : 0u)
        : "memory");
    return r != 0;
}

constexpr int kMaxNormParts = 16;  // epilogue LayerNorm rows of at most 512 columns

__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The epilogue LayerNorm of one 32-column tile (persistent kernel, every
// tile of the launch resident at once): publish this slice's (mean, M2) of
// each row, wait until the row tile's other column tiles have published
// theirs (a bounded spin on a counter), merge them in column order (Chan et
// al.; every tile of the row gets the same bits), normalise the slice's 32
// values `v` and store them through `tmn`. The last tile of the row tile to
// finish zeroes its counters for the next launch. Returns false when the
// wait ran out.
__device__ bool norm_tile(const Params& p, const CUtensorMap* tmn, const float* v, bool live,
                          int m0, int n0, int row, uint8_t* buf, volatile int* abort) {
    const int parts = p.N / 32;
    const int grow = m0 + row;
    const int lane = lane_id();
    unsigned* ctr = p.norm_ctr + 2 * (m0 / BM);
    if (live) {
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) sum += v[i];
        const float mean = sum * (1.0f / 32.0f);
        float m2 = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) m2 += (v[i] - mean) * (v[i] - mean);
        p.norm_stats[static_cast<size_t>(grow) * parts + n0 / 32] = make_float2(mean, m2);
    }
    epilogue_all(true);  // the tile's rows are written
    bool ok = true;
    if (row == 0) {
        __threadfence();  // ... and published (cumulative over the barrier)
        atomicAdd(ctr, 1u);
        const long long t0 = clock64();
        const long long limit = wait_limit(p.status);
        while (ld_acquire_gpu(ctr) < static_cast<unsigned>(parts)) {
            if (*abort || clock64() - t0 > limit) {
                if (!*abort) record_status(p.status, ST_TIMEOUT_SOFTMAX, 0x300 + m0 / BM);
                *abort = 1;
                ok = false;
                break;
            }
            __nanosleep(32);
        }
    }
    if (!epilogue_all(ok)) return false;
    float mu = 0.0f, m2 = 0.0f;
    if (live) {
        // every partial's load is issued before the merge (one L2 round trip)
        const float2* st = p.norm_stats + static_cast<size_t>(grow) * parts;
        float2 part[kMaxNormParts];
#pragma unroll
        for (int q = 0; q < kMaxNormParts; ++q)
            if (q < parts) part[q] = __ldcg(st + q);
#pragma unroll
        for (int q = 0; q < kMaxNormParts; ++q) {
            if (q < parts) {
                const float na = 32.0f * static_cast<float>(q), nab = na + 32.0f;
                const float delta = part[q].x - mu;
                mu += delta * (32.0f / nab);
                m2 += part[q].y + delta * delta * (na * 32.0f / nab);
            }
        }
    }
    const float rstd = rsqrtf(m2 / static_cast<float>(p.N) + p.norm_eps);
    uint32_t y[16];
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(p.norm_gamma + n0 + i));
        const float4 b = __ldg(reinterpret_cast<const float4*>(p.norm_beta + n0 + i));
        y[i / 2] = pack2((v[i] - mu) * rstd * g.x + b.x, (v[i + 1] - mu) * rstd * g.y + b.y,
                         p.norm_dtype);
        y[i / 2 + 1] = pack2((v[i + 2] - mu) * rstd * g.z + b.z,
                             (v[i + 3] - mu) * rstd * g.w + b.w, p.norm_dtype);
    }
    if (lane == 0) bulk_wait_read();  // the output block has left `buf`
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
            make_uint4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tmn, smem_u32(buf), n0, m0 + (row & ~31));
        bulk_commit();
    }
    epilogue_all(true);  // every reader of this tile is past the statistics
    if (row == 0 && atomicAdd(ctr + 1, 1u) == static_cast<unsigned>(parts) - 1) {
        ctr[0] = 0u;
        ctr[1] = 0u;
    }
    return true;
}

// The persistent form, for A loaded by TMA: one CTA per SM walks tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... of this launch (tile t is row
// tile t % m_tiles, column tile t / m_tiles). Two TMEM accumulators: the
// epilogue warps drain tile j from one while the MMA thread fills tile j + 1
// in the other, and the TMA ring runs on across tiles, so the epilogue and the
// CTA's set-up leave the critical path once a CTA has more than one tile.
// kPair: the CTA-pair form (a cluster of two CTAs, cta_group::2). A tile is
// 256 x BN: each CTA copies its own 128 rows of A and BN / 2 rows of B into
// its shared memory (so it holds the stage of a 128 x BN/2 tile), the even
// CTA's MMA warp issues M = 256 MMAs that read both CTAs' tiles and write
// each CTA's 128 x BN accumulator, and each CTA's epilogue stores its own
// 128 rows. Per MMA each SM then brings in half the B bytes of a 128 x BN
// tile. The stage barriers that the MMA waits on are the even CTA's (both
// CTAs' copies count on them); the MMA's completions arrive on both CTAs'
// barriers; the epilogues of both free an accumulator on the even CTA's
// barrier. No copy is multicast.
template <int BN, int KC, int EPI, bool kPair, bool kSk>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_persistent(const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_o,
                    const __grid_constant__ CUtensorMap tm_n, const Params p) {
    using L = Layout<kPair ? BN / 2 : BN, KC, true>;
    constexpr int STAGES = L::kStages;
    static_assert(STAGES >= 2, "a stage ring needs two stages");
    constexpr uint32_t kAccCols = Layout<BN>::kTmemCols;  // one accumulator
    constexpr uint32_t kCols = 2 * kAccCols;
    constexpr int TM = kPair ? 2 * BM : BM;  // rows of a tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* epi = smem + STAGES * L::kStage;  // output staging, kEpiBytes
    Tail* tail = reinterpret_cast<Tail*>(epi + kEpiBytes);
    volatile int* abort = &tail->abort;
    auto sA = [&](int s) { return smem + s * L::kStage; };
    auto sB = [&](int s) { return smem + s * L::kStage + KC * kTileA; };

    const int warp = warp_id();
    const int lane = lane_id();
    const int nk = p.K / (BK * KC);  // stages per tile (the host makes KC divide K / 64)
    // tiles are walked by CTA (one CTA) or by pair (kPair; p.m_tiles then
    // counts 256-row tiles)
    const int rank = kPair ? static_cast<int>(cluster_rank()) : 0;
    const int unit = kPair ? static_cast<int>(blockIdx.x) / 2 : static_cast<int>(blockIdx.x);
    const int units = kPair ? static_cast<int>(gridDim.x) / 2 : static_cast<int>(gridDim.x);
    const bool leader = rank == 0;
    const int total = p.m_tiles * (p.N / BN);  // tiles of this launch
    // The CTA's segments: stage ranges [s0, s1) of a tile, each accumulated
    // from zero. Without stream-K: tiles unit, unit + units, ... whole. With
    // it (S = p.sk_pieces > 1, one CTA per unit): the launch's total x S
    // pieces (piece i of a tile: stages [i nk / S, (i + 1) nk / S)) dealt in
    // contiguous ranges. The CTA holding a tile's last piece finishes the
    // tile. A CTA takes its tiles from the last to the first and each tile's
    // pieces in order, so a finishing piece comes after the CTA's own
    // earlier pieces of that tile, and the pieces it waits for from other
    // CTAs are the first work of lower-numbered CTAs, which the block
    // scheduler starts no later than this one.
    static_assert(!(kSk && kPair), "stream-K takes one CTA per tile");
    const int S = !kSk || p.sk_pieces <= 1 ? 1 : p.sk_pieces;
    int u0 = 0, u1 = 0, nseg;
    if (S > 1) {
        const long long U = static_cast<long long>(total) * S;
        u0 = static_cast<int>(U * unit / units);
        u1 = static_cast<int>(U * (unit + 1) / units);
        nseg = u1 - u0;
    } else {
        nseg = unit < total ? (total - unit + units - 1) / units : 0;
    }
    struct Seg {
        int t, piece, s0, s1;
    };
    auto seg = [&](int j) {
        Seg q;
        if (S > 1) {
            int t = (u1 - 1) / S, rem = j;
            for (;;) {
                const int lo = u0 > t * S ? u0 : t * S;
                const int hi = u1 < (t + 1) * S ? u1 : (t + 1) * S;
                if (rem < hi - lo) {
                    q.t = t;
                    q.piece = lo + rem - t * S;
                    break;
                }
                rem -= hi - lo;
                --t;
            }
            q.s0 = q.piece * nk / S;
            q.s1 = (q.piece + 1) * nk / S;
        } else {
            q.t = unit + j * units;
            q.piece = 0;
            q.s0 = 0;
            q.s1 = nk;
        }
        return q;
    };
    auto count_stages = [&]() {
        int n = 0;
        for (int j = 0; j < nseg; ++j) {
            const Seg q = seg(j);
            n += q.s1 - q.s0;
        }
        return n;
    };
    auto tile_m0 = [&](int t) {  // this CTA's first row of tile t
        return (p.m_tile0 + t % p.m_tiles) * TM + rank * BM;
    };
    auto tile_n0 = [&](int t) { return (t / p.m_tiles) * BN; };
    // the barrier the MMA waits on for stage s: the even CTA's
    auto full_bar = [&](int s) {
        const uint32_t b = smem_u32(&tail->full[s]);
        return kPair ? dsmem_addr(b, 0) : b;
    };

    if (threadIdx.x == 0) {
        trace_stamp(p.trace, 0);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&tail->acc_full[b]), 1);
            mbar_init(smem_u32(&tail->acc_empty[b]), kPair ? 8 : 4);
        }
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        if (p.tma_store) tma_prefetch_desc(&tm_o);
    }
    if (warp == 1) {
        if constexpr (kPair) {
            tmem_alloc_pair(smem_u32(&tail->tmem_base), kCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(smem_u32(&tail->tmem_base), kCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    // the pair: both CTAs' barriers and tensor memory exist before either
    // CTA's copies or MMAs can signal or write the other's
    if constexpr (kPair) cluster_sync();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    if (threadIdx.x == 0) trace_stamp(p.trace, 1);
    // Programmatic dependent launch: with weights_static, B and the epilogue
    // vectors do not depend on the previous kernel, so the first stages' B
    // copies and the vector staging start before the wait; A, the residual
    // and every store come after it (each role waits before its first
    // dependent access; the MMA warp touches no global memory).
    pdl_trigger();

    if (warp == 0) {
        // The whole warp runs the producer loop in step; lane 0 arms the
        // stage and copies A, lane 1 copies B, so the two copies of a stage
        // are in flight together (each thread's copies are serial). Lane 0
        // alone waits for the stage to be free; the vote hands the outcome
        // to the warp, so both lanes start the same stages.
        // kPair: the even CTA arms its barrier for both CTAs' bytes; B rows
        // of this CTA's half start BN / 2 further in the odd CTA
        constexpr uint32_t kArm = kPair ? 2 * L::kStage : L::kStage;
        const int b_off = kPair ? rank * (BN / 2) : 0;
        auto load = [&](uint32_t dst, const CUtensorMap* map, int y, int z, uint32_t bar) {
            if constexpr (kPair) tma_load_3d_pair(dst, map, 0, y, z, bar);
            else tma_load_3d(dst, map, 0, y, z, bar);
        };
        const int total_g = count_stages();
        const int first = !p.weights_static ? 0 : STAGES < total_g ? STAGES : total_g;
        for (int j = 0, g = 0; j < nseg && g < first; ++j) {  // stages whose B is fetched up front
            const Seg q = seg(j);
            for (int kb = q.s0; kb < q.s1 && g < first; ++kb, ++g) {
                if (lane == 0 && leader) mbar_arrive_expect_tx(smem_u32(&tail->full[g]), kArm);
                if (lane == 1)
                    load(smem_u32(sB(g)), &tm_b, tile_n0(q.t) + b_off, kb * KC, full_bar(g));
            }
        }
        pdl_wait();
        if (lane == 0) trace_stamp(p.trace, 2);
        int g = 0;  // stages whose loads were started, over all tiles
        bool ok = true;
        for (int j = 0; j < nseg && ok; ++j) {
            const Seg q = seg(j);
            const int m0 = tile_m0(q.t), n0 = tile_n0(q.t);
            for (int kb = q.s0; kb < q.s1; ++kb, ++g) {
                const int s = g % STAGES;
                bool r = true;
                if (lane == 0 && g >= STAGES)
                    r = mbar_wait(smem_u32(&tail->empty[s]), ((g / STAGES) - 1) & 1, abort,
                                  p.status, ST_TIMEOUT_TMA, g);
                ok = __all_sync(0xFFFFFFFFu, r);
                if (!ok) break;
                const uint32_t bar = full_bar(s);  // the copies' (kPair: the even CTA's)
                if (lane == 0) {
                    if (g >= first && leader)
                        mbar_arrive_expect_tx(smem_u32(&tail->full[s]), kArm);
                    load(smem_u32(sA(s)), &tm_a, m0, kb * KC, bar);
                } else if (lane == 1 && g >= first) {
                    load(smem_u32(sB(s)), &tm_b, n0 + b_off, kb * KC, bar);
                }
                __syncwarp();
            }
        }
        if (lane == 0 && *abort && leader) {
            // let every started copy land before shared memory is released
            // (the pair's copies, both CTAs', count on the even CTA's
            // barriers, and the pair leaves together after the closing
            // cluster barrier)
            for (int s = 0; s < STAGES && s < g; ++s) {
                const int uses = (g - s - 1) / STAGES + 1;
                mbar_wait(smem_u32(&tail->full[s]), (uses - 1) & 1, nullptr, p.status,
                          ST_TIMEOUT_DRAIN, s);
            }
        }
        __syncwarp();
    } else if (warp == 1 && !(kPair && !leader)) {
        // whole-warp issuer loop, one elected lane issues and waits (see
        // gemm_kernel)
        const bool elected = elect_one();
        auto wait_all = [&](uint32_t bar, uint32_t parity, uint32_t where) -> bool {
            bool r = true;
            if (elected)
                r = kPair ? mbar_wait_cluster(bar, parity, abort, p.status, ST_TIMEOUT_MMA, where)
                          : mbar_wait(bar, parity, abort, p.status, ST_TIMEOUT_MMA, where);
            return __all_sync(0xFFFFFFFFu, r);
        };
        auto commit = [&](uint32_t bar) {
            if constexpr (kPair) mma_commit_pair(bar);
            else mma_commit(bar);
        };
        const uint32_t idesc = idesc_f16(TM, BN, p.ab_fmt, p.ab_fmt, 0, 0);
        const int total_g = count_stages();
        int g = 0;
        bool ok = true;
        for (int j = 0; j < nseg && ok; ++j) {
            const Seg q = seg(j);
            const int b = j & 1, use = j >> 1;
            if (use > 0 && !wait_all(smem_u32(&tail->acc_empty[b]), (use - 1) & 1, 0x100 + j)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t acc = tmem + static_cast<uint32_t>(b) * kAccCols;
            for (int kb = q.s0; kb < q.s1; ++kb, ++g) {
                const int s = g % STAGES;
                ok = wait_all(smem_u32(&tail->full[s]), (g / STAGES) & 1, g);  // the even CTA's own
                if (!ok) break;
                if (g == 0 && elected) trace_stamp(p.trace, 3);
                tc_fence_after();
                const uint32_t a = smem_u32(sA(s)), bb = smem_u32(sB(s));
                if (elected) {
#pragma unroll
                    for (int c = 0; c < KC; ++c)
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k) {
                            const uint64_t da = desc_k(a + c * kTileA + 32 * k);
                            const uint64_t db = desc_k(bb + c * L::kTileB + 32 * k);
                            const uint32_t acc_in = (kb > q.s0 || c > 0 || k > 0) ? 1u : 0u;
                            if constexpr (kPair) mma_ss_pair(acc, da, db, idesc, acc_in);
                            else mma_ss(acc, da, db, idesc, acc_in);
                        }
                    // release the stage only if the producer will refill it,
                    // so no arrival lands after the CTA has finished
                    if (g + STAGES < total_g) commit(smem_u32(&tail->empty[s]));
                }
                __syncwarp();
            }
            if (ok && elected) commit(smem_u32(&tail->acc_full[b]));
            if (j == 0 && elected) trace_stamp(p.trace, 4);
            __syncwarp();
        }
        if (!ok && elected) {
            commit(smem_u32(&tail->drain));
            mbar_wait(smem_u32(&tail->drain), 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0xD);
        }
        __syncwarp();
    } else if (warp >= 2) {
        const int sub = warp & 3;
        const int row = sub * 32 + lane;
        constexpr size_t kSlot = static_cast<size_t>(BN / 32) * kSkChunk;  // floats per slot
        for (int j = 0; j < nseg; ++j) {
            const Seg q = seg(j);
            const int b = j & 1, use = j >> 1;
            const int m0 = tile_m0(q.t), n0 = tile_n0(q.t);
            const RowCtx rc = row_ctx(p, m0 + row);
            epilogue_all(true);  // the previous tile's staged vectors are no longer read
            if (!p.weights_static) pdl_wait();
            stage_vectors<BN>(p, tail, n0);
            epilogue_all(true);
            pdl_wait();  // the residual and the outputs belong to the previous kernels
            const bool finish = q.piece == S - 1;  // this CTA finishes the tile
            const size_t slot0 = static_cast<size_t>(q.t) * S;  // the tile's first slot
            const float* parts = nullptr;
            if (finish && S > 1) {
                // the last piece finishes the tile: wait (bounded) until the
                // earlier pieces are stored (before its own accumulator, so
                // their first chunk loads beside the residual's), clear their
                // flags for the next launch, and add them in piece order
                bool fine = true;
                if (threadIdx.x == 64) {
                    const long long t0 = clock64();
                    const long long limit = wait_limit(p.status);
                    for (int i = 0; i < S - 1 && fine; ++i) {
                        while (ld_acquire_gpu(p.sk_flag + slot0 + i) == 0u) {
                            if (*abort || clock64() - t0 > limit) {
                                if (!*abort)
                                    record_status(p.status, ST_TIMEOUT_SOFTMAX, 0x400 + q.t);
                                *abort = 1;
                                fine = false;
                                break;
                            }
                            __nanosleep(32);
                        }
                    }
                }
                if (!epilogue_all(fine)) break;
                if (threadIdx.x == 64)
                    for (int i = 0; i < S - 1; ++i) p.sk_flag[slot0 + i] = 0u;
                parts = p.sk_part + kSlot * slot0 + sk_row_base(row);
            }
            float rv0[32];
            if (finish) prefetch_residual(p, rc, n0, rv0);
            bool ok = mbar_wait(smem_u32(&tail->acc_full[b]), use & 1, abort, p.status,
                                ST_TIMEOUT_SOFTMAX, 0x200 + j);
            if (j == 0 && threadIdx.x == 64) trace_stamp(p.trace, 5);
            if (!epilogue_all(ok)) break;
            tc_fence_after();
            const uint32_t t_acc = tmem + static_cast<uint32_t>(b) * kAccCols +
                                   (static_cast<uint32_t>(sub * 32) << 16);
            if (!finish) {
                // an earlier piece of a stream-K tile: its partial sums into its
                // slot (a warp's stores of one column group contiguous), then
                // its flag, once every row is stored
                float* dst = p.sk_part + kSlot * (slot0 + q.piece) + sk_row_base(row);
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t r[32];
                    tmem_ld32(t_acc + c * 32, r);
                    tmem_wait_ld();
                    float4* d = reinterpret_cast<float4*>(dst + c * kSkChunk);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        __stcg(d + i * kSkGroup, make_float4(__uint_as_float(r[4 * i]),
                                                  __uint_as_float(r[4 * i + 1]),
                                                  __uint_as_float(r[4 * i + 2]),
                                                  __uint_as_float(r[4 * i + 3])));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tail->acc_empty[b]));
                epilogue_all(true);  // every row of the slot is stored
                if (threadIdx.x == 64) {
                    __threadfence();  // ... and published (cumulative over the barrier)
                    st_release_gpu(p.sk_flag + slot0 + q.piece, 1u);
                }
                continue;
            }
            float keep[32];
            store_tile<BN, EPI, kSk ? kMaxSkParts : 0>(
                p, tail, t_acc, n0, rc, rv0, p.tma_store ? &tm_o : nullptr, epi + sub * kEpiBlock,
                m0 + sub * 32 + p.out_row_offset, p.norm_out != nullptr ? keep : nullptr, parts,
                S - 1, kSlot);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (kPair && !leader)
                    mbar_arrive_remote(dsmem_addr(smem_u32(&tail->acc_empty[b]), 0));
                else
                    mbar_arrive(smem_u32(&tail->acc_empty[b]));
            }
            if (p.norm_out != nullptr &&
                !norm_tile(p, &tm_n, keep, rc.live, m0, n0, row, epi + sub * kEpiBlock, abort))
                break;
        }
        // stores complete before the staging is released and the kernel ends
        if (p.tma_store && lane == 0) bulk_wait_all();
        __syncwarp();
        if (threadIdx.x == 64) trace_stamp(p.trace, 6);
    }

    tc_fence_before();
    __syncthreads();
    // the pair leaves together: no arrival or MMA read of one CTA's memory
    // is outstanding when the other exits
    if constexpr (kPair) cluster_sync();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if constexpr (kPair) tmem_dealloc_pair(tmem, kCols);
        else tmem_dealloc(tmem, kCols);
    }
    if (threadIdx.x == 0) trace_stamp(p.trace, 7);
}

// The K range split over a cluster of two CTAs (one tile per cluster): CTA
// r of the pair accumulates the tile's stages [r S / 2, (r + 1) S / 2) into
// its own tensor memory, then owns columns [r BN / 2, (r + 1) BN / 2) of the
// tile. Each epilogue warp writes the partner's half of its 32 rows' partial
// sums into its block of the output staging (128-byte rows swizzled by
// 16-byte chunk) and one lane copies the block into the partner's receive
// buffer with one bulk copy that completes on the partner's barrier (armed
// at set-up for the four blocks); each warp then waits for the partner's
// blocks, adds them to its own half (two addends, so either order gives the
// same bits), writes the sum back to tensor memory and runs the ordinary
// epilogue on its half. For K-heavy
// launches with few tiles (ViT-S fc2: K = 1536 on 66 tiles of 64 columns),
// which a CTA per tile leaves bound by the operand feed of half the SMs.
template <int BN, int KC>
struct SplitLayout {
    static constexpr uint32_t kTileB = BN * BK * 2;
    static constexpr uint32_t kStage = KC * (kTileA + kTileB);
    static constexpr uint32_t kRecv = BM * (BN / 2) * 4;
    static constexpr int kStages =
        static_cast<int>((kSmemLimit - 4096 - kEpiBytes - kRecv) / kStage) < kMaxStages
            ? static_cast<int>((kSmemLimit - 4096 - kEpiBytes - kRecv) / kStage)
            : kMaxStages;
};

template <int BN, int KC>
constexpr size_t split_smem_bytes() {
    using L = SplitLayout<BN, KC>;
    return 1024 + L::kStages * L::kStage + L::kRecv + kEpiBytes + sizeof(Tail);
}

template <int BN, int KC, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_split2(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                const __grid_constant__ CUtensorMap tm_o, const Params p) {
    using L = SplitLayout<BN, KC>;
    constexpr int STAGES = L::kStages;
    static_assert(STAGES >= 2, "a stage ring needs two stages");
    constexpr int HALF = BN / 2;
    constexpr uint32_t kCols = Layout<BN>::kTmemCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* recv = smem + STAGES * L::kStage;  // the partner's partials of this CTA's half
    uint8_t* epi = recv + L::kRecv;
    Tail* tail = reinterpret_cast<Tail*>(epi + kEpiBytes);
    volatile int* abort = &tail->abort;
    auto sA = [&](int s) { return smem + s * L::kStage; };
    auto sB = [&](int s) { return smem + s * L::kStage + KC * kTileA; };

    const int warp = warp_id();
    const int lane = lane_id();
    const int rank = static_cast<int>(cluster_rank());
    const int t = static_cast<int>(blockIdx.x) / 2;  // the cluster's tile
    const int m0 = (p.m_tile0 + t % p.m_tiles) * BM;
    const int n0 = (t / p.m_tiles) * BN;
    const int all = p.K / (BK * KC);  // stages of the whole K
    const int s0 = all * rank / 2;    // this CTA's stages [s0, s0 + nk)
    const int nk = all * (rank + 1) / 2 - s0;
    // the tail's drain barrier doubles as the receive barrier: armed here for
    // the partner's four 32-row blocks, completed by their bulk copies
    const uint32_t b_recv = smem_u32(&tail->drain);

    if (threadIdx.x == 0) {
        trace_stamp(p.trace, 0);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        mbar_init(smem_u32(&tail->acc_full[0]), 1);
        mbar_init(smem_u32(&tail->acc_full[1]), 1);  // the MMA's unwinding
        mbar_init(b_recv, 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        tma_prefetch_desc(&tm_a);
        tma_prefetch_desc(&tm_b);
        if (p.tma_store) tma_prefetch_desc(&tm_o);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) mbar_arrive_expect_tx(b_recv, L::kRecv);
    cluster_sync();  // the partner's barrier and receive buffer exist before any push
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    if (threadIdx.x == 0) trace_stamp(p.trace, 1);
    pdl_trigger();

    if (warp == 0) {
        const int first = !p.weights_static ? 0 : STAGES < nk ? STAGES : nk;
        for (int g = 0; g < first; ++g) {
            const uint32_t bar = smem_u32(&tail->full[g]);
            if (lane == 0) mbar_arrive_expect_tx(bar, L::kStage);
            if (lane == 1) tma_load_3d(smem_u32(sB(g)), &tm_b, 0, n0, (s0 + g) * KC, bar);
        }
        pdl_wait();
        if (lane == 0) trace_stamp(p.trace, 2);
        int g = 0;
        for (; g < nk; ++g) {
            const int s = g % STAGES;
            bool r = true;
            if (lane == 0 && g >= STAGES)
                r = mbar_wait(smem_u32(&tail->empty[s]), ((g / STAGES) - 1) & 1, abort, p.status,
                              ST_TIMEOUT_TMA, g);
            if (!__all_sync(0xFFFFFFFFu, r)) break;
            const uint32_t bar = smem_u32(&tail->full[s]);
            if (lane == 0) {
                if (g >= first) mbar_arrive_expect_tx(bar, L::kStage);
                tma_load_3d(smem_u32(sA(s)), &tm_a, 0, m0, (s0 + g) * KC, bar);
            } else if (lane == 1 && g >= first) {
                tma_load_3d(smem_u32(sB(s)), &tm_b, 0, n0, (s0 + g) * KC, bar);
            }
            __syncwarp();
        }
        if (lane == 0 && *abort) {
            for (int s = 0; s < STAGES && s < g; ++s) {
                const int uses = (g - s - 1) / STAGES + 1;
                mbar_wait(smem_u32(&tail->full[s]), (uses - 1) & 1, nullptr, p.status,
                          ST_TIMEOUT_DRAIN, s);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        const bool elected = elect_one();
        const uint32_t idesc = idesc_f16(BM, BN, p.ab_fmt, p.ab_fmt, 0, 0);
        bool ok = true;
        for (int g = 0; g < nk && ok; ++g) {
            const int s = g % STAGES;
            bool r = true;
            if (elected)
                r = mbar_wait(smem_u32(&tail->full[s]), (g / STAGES) & 1, abort, p.status,
                              ST_TIMEOUT_MMA, g);
            ok = __all_sync(0xFFFFFFFFu, r);
            if (!ok) break;
            if (g == 0 && elected) trace_stamp(p.trace, 3);
            tc_fence_after();
            const uint32_t a = smem_u32(sA(s)), bb = smem_u32(sB(s));
            if (elected) {
#pragma unroll
                for (int c = 0; c < KC; ++c)
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                        mma_ss(tmem, desc_k(a + c * kTileA + 32 * k),
                               desc_k(bb + c * L::kTileB + 32 * k), idesc,
                               (g > 0 || c > 0 || k > 0) ? 1u : 0u);
                if (g + STAGES < nk) mma_commit(smem_u32(&tail->empty[s]));
            }
            __syncwarp();
        }
        if (elected) {
            if (ok) {
                mma_commit(smem_u32(&tail->acc_full[0]));
                trace_stamp(p.trace, 4);
            } else {
                mma_commit(smem_u32(&tail->acc_full[1]));
                mbar_wait(smem_u32(&tail->acc_full[1]), 0, nullptr, p.status, ST_TIMEOUT_DRAIN,
                          0xD);
            }
        }
        __syncwarp();
    } else {
        const int sub = warp & 3;
        const int row = sub * 32 + lane;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(sub * 32) << 16);
        const int mine = rank * HALF, theirs = (1 - rank) * HALF;  // column offsets
        const RowCtx rc = row_ctx(p, m0 + row);
        if (!p.weights_static) pdl_wait();
        stage_vectors<HALF>(p, tail, n0 + mine);
        epilogue_all(true);
        pdl_wait();  // the residual and the outputs belong to the previous kernels
        float rv0[32];
        prefetch_residual(p, rc, n0 + mine, rv0);
        bool ok = mbar_wait(smem_u32(&tail->acc_full[0]), 0, abort, p.status, ST_TIMEOUT_SOFTMAX,
                            0x200);
        if (threadIdx.x == 64) trace_stamp(p.trace, 5);
        ok = epilogue_all(ok);
        tc_fence_after();
        // the partner's half of this warp's 32 rows, 32 columns at a time,
        // staged in the warp's 4 KiB block and copied into the partner's
        // receive buffer (block c of warp sub at (c * 4 + sub) * 4 KiB)
        const uint32_t peer = static_cast<uint32_t>(1 - rank);
        uint8_t* blk = epi + sub * kEpiBlock;
#pragma unroll 1
        for (int c = 0; c < HALF / 32; ++c) {
            uint32_t r[32];
            if (ok) {
                tmem_ld32(t_lane + theirs + 32 * c, r);
                tmem_wait_ld();
            }
            if (c > 0) {  // the previous block has left the staging
                if (lane == 0) bulk_wait_read();
                __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                *reinterpret_cast<uint4*>(blk + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                    make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                const uint32_t off = static_cast<uint32_t>((c * 4 + sub) * kEpiBlock);
                bulk_copy_to_peer(dsmem_addr(smem_u32(recv) + off, peer), smem_u32(blk),
                                  kEpiBlock, dsmem_addr(b_recv, peer));
                bulk_commit();
            }
        }
        if (lane == 0) bulk_wait_read();  // the staging is free for the output blocks
        __syncwarp();
        // the partner's partials of this CTA's half, added to its own and
        // written back for the ordinary epilogue
        if (ok) ok = mbar_wait_cluster(b_recv, 0, abort, p.status, ST_TIMEOUT_SOFTMAX, 0x210);
        ok = epilogue_all(ok);
        if (ok) {
#pragma unroll 1
            for (int c = 0; c < HALF / 32; ++c) {
                uint32_t r[32];
                tmem_ld32(t_lane + mine + 32 * c, r);
                tmem_wait_ld();
                const uint8_t* src = recv + (c * 4 + sub) * kEpiBlock + lane * 128;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint4 q = *reinterpret_cast<const uint4*>(src + ((j ^ (lane & 7)) << 4));
                    r[4 * j] = __float_as_uint(__uint_as_float(r[4 * j]) + __uint_as_float(q.x));
                    r[4 * j + 1] =
                        __float_as_uint(__uint_as_float(r[4 * j + 1]) + __uint_as_float(q.y));
                    r[4 * j + 2] =
                        __float_as_uint(__uint_as_float(r[4 * j + 2]) + __uint_as_float(q.z));
                    r[4 * j + 3] =
                        __float_as_uint(__uint_as_float(r[4 * j + 3]) + __uint_as_float(q.w));
                }
                tmem_st32(t_lane + mine + 32 * c, r);
            }
            tmem_wait_st();
            store_tile<HALF, EPI>(p, tail, t_lane + mine, n0 + mine, rc, rv0,
                                  p.tma_store ? &tm_o : nullptr, epi + sub * kEpiBlock,
                                  m0 + sub * 32 + p.out_row_offset);
        }
        if (p.tma_store && lane == 0) bulk_wait_all();
        __syncwarp();
        if (threadIdx.x == 64) trace_stamp(p.trace, 6);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
    if (threadIdx.x == 0) trace_stamp(p.trace, 7);
}

// The LayerNorm prologue with its rows brought by TMA (one tile per CTA):
// A = LayerNorm(x) for f32 rows x whose per-row statistics the GEMM that
// wrote x left as (mean, M2) per column slice. A stage holds a k-block of x
// (128 rows x 64 f32, unswizzled, by TMA), the 16-bit A tile the epilogue
// warps normalise from it into the MMA's swizzled layout, and the B tile.
// The epilogue warps are free while the main loop runs, as each CTA has
// one tile; they then run the epilogue. Barriers per stage: full (x and B
// landed), conv (A written), empty (the MMAs are done with the stage).
constexpr uint32_t kTileX = BM * BK * 4;  // 32 KiB

template <int BN>
struct LnLayout {
    static constexpr uint32_t kTileB = BN * BK * 2;
    static constexpr uint32_t kStage = kTileX + kTileA + kTileB;
    static constexpr int kStages =
        static_cast<int>((kSmemLimit - 4096 - kEpiBytes) / kStage) < kMaxStages
            ? static_cast<int>((kSmemLimit - 4096 - kEpiBytes) / kStage)
            : kMaxStages;
};

template <int BN>
constexpr size_t ln_smem_bytes() {
    return 1024 + LnLayout<BN>::kStages * LnLayout<BN>::kStage + kEpiBytes + sizeof(Tail);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_ln_staged(const __grid_constant__ CUtensorMap tm_x,
                   const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_o, const Params p) {
    using L = LnLayout<BN>;
    constexpr int STAGES = L::kStages;
    static_assert(STAGES >= 2, "a stage ring needs two stages");
    constexpr uint32_t kCols = Layout<BN>::kTmemCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* epi = smem + STAGES * L::kStage;
    Tail* tail = reinterpret_cast<Tail*>(epi + kEpiBytes);
    volatile int* abort = &tail->abort;
    auto sX = [&](int s) { return smem + s * L::kStage; };
    auto sA = [&](int s) { return smem + s * L::kStage + kTileX; };
    auto sB = [&](int s) { return smem + s * L::kStage + kTileX + kTileA; };

    const int warp = warp_id();
    const int lane = lane_id();
    const int nk = p.K / BK;
    const int t = static_cast<int>(blockIdx.x);  // the grid has one CTA per tile
    const int m0 = (p.m_tile0 + t % p.m_tiles) * BM;
    const int n0 = (t / p.m_tiles) * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->conv[s]), 4);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        mbar_init(smem_u32(&tail->acc_full[0]), 1);
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_b);
        if (p.tma_store) tma_prefetch_desc(&tm_o);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    pdl_trigger();

    if (warp == 0) {
        // lane 0 arms each stage and copies x, lane 1 copies B (with
        // weights_static the first stages' B before the dependency wait)
        const int first = !p.weights_static ? 0 : (STAGES < nk ? STAGES : nk);
        for (int g = 0; g < first; ++g) {
            const uint32_t bar = smem_u32(&tail->full[g]);
            if (lane == 0) mbar_arrive_expect_tx(bar, kTileX + L::kTileB);
            if (lane == 1) tma_load_3d(smem_u32(sB(g)), &tm_b, 0, n0, g, bar);
        }
        pdl_wait();
        int g = 0;
        for (; g < nk; ++g) {
            const int s = g % STAGES;
            bool r = true;
            if (lane == 0 && g >= STAGES)
                r = mbar_wait(smem_u32(&tail->empty[s]), ((g / STAGES) - 1) & 1, abort, p.status,
                              ST_TIMEOUT_TMA, g);
            if (!__all_sync(0xFFFFFFFFu, r)) break;
            const uint32_t bar = smem_u32(&tail->full[s]);
            if (lane == 0) {
                if (g >= first) mbar_arrive_expect_tx(bar, kTileX + L::kTileB);
                tma_load_2d(smem_u32(sX(s)), &tm_x, g * BK, m0, bar);
            } else if (lane == 1 && g >= first) {
                tma_load_3d(smem_u32(sB(s)), &tm_b, 0, n0, g, bar);
            }
            __syncwarp();
        }
        if (lane == 0 && *abort) {
            for (int s = 0; s < STAGES && s < g; ++s) {
                const int uses = (g - s - 1) / STAGES + 1;
                mbar_wait(smem_u32(&tail->full[s]), (uses - 1) & 1, nullptr, p.status,
                          ST_TIMEOUT_DRAIN, s);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        const bool elected = elect_one();
        const uint32_t idesc = idesc_f16(BM, BN, p.ab_fmt, p.ab_fmt, 0, 0);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            bool r = true;
            if (elected)
                r = mbar_wait(smem_u32(&tail->conv[s]), (kb / STAGES) & 1, abort, p.status,
                              ST_TIMEOUT_MMA, kb);
            ok = __all_sync(0xFFFFFFFFu, r);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a = smem_u32(sA(s)), b = smem_u32(sB(s));
            if (elected) {
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    mma_ss(tmem, desc_k(a + 32 * k), desc_k(b + 32 * k), idesc,
                           (kb > 0 || k > 0) ? 1u : 0u);
                if (kb + STAGES < nk) mma_commit(smem_u32(&tail->empty[s]));
            }
            __syncwarp();
        }
        if (elected) {
            if (ok) {
                mma_commit(smem_u32(&tail->acc_full[0]));
            } else {
                mma_commit(smem_u32(&tail->drain));
                mbar_wait(smem_u32(&tail->drain), 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0xD);
            }
        }
        __syncwarp();
    } else {
        constexpr unsigned kFull = 0xFFFFFFFFu;
        const int sub = warp & 3;
        const int row = sub * 32 + lane;
        const int dt = p.ab_fmt ? BL_BF16 : BL_F16;
        pdl_wait();  // x's statistics come from the previous kernel
        // lane r: mean and 1/std of the warp's row r, from the slices'
        // (mean, M2) (equal counts: the mean of means, then the M2s plus
        // each slice's squared offset times its count)
        float my_mean = 0.0f, my_rstd = 0.0f;
        {
            const int gr = m0 + row;
            if (gr < p.M) {
                const float2* st = p.ln_stats + static_cast<long long>(gr) * p.ln_stats_parts;
                const float nper = static_cast<float>(p.K / p.ln_stats_parts);
                float2 part[kMaxNormParts];
#pragma unroll
                for (int q = 0; q < kMaxNormParts; ++q)
                    if (q < p.ln_stats_parts) part[q] = st[q];
                float sm = 0.0f;
#pragma unroll
                for (int q = 0; q < kMaxNormParts; ++q)
                    if (q < p.ln_stats_parts) sm += part[q].x;
                const float mean = sm / static_cast<float>(p.ln_stats_parts);
                float m2 = 0.0f;
#pragma unroll
                for (int q = 0; q < kMaxNormParts; ++q)
                    if (q < p.ln_stats_parts)
                        m2 += part[q].y + (part[q].x - mean) * (part[q].x - mean) * nper;
                my_mean = mean;
                my_rstd = rsqrtf(m2 / static_cast<float>(p.K) + p.eps);
            }
        }
        // Every lane needs all 32 rows' (1/std, -mean/std): gathered once
        // into registers (rows past M get 0 and 0: their A rows hold beta,
        // and their output rows are never stored).
        float ra[32], rc2[32];
#pragma unroll
        for (int r2 = 0; r2 < 32; ++r2) {
            const float rs = __shfl_sync(kFull, my_rstd, r2);
            ra[r2] = rs;
            rc2[r2] = -__shfl_sync(kFull, my_mean, r2) * rs;
        }
        bool ok = true;
        const int chunk = lane >> 2, off = (lane & 3) * 4;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            const int k = kb * BK + 2 * lane;
            const float2 g = __ldg(reinterpret_cast<const float2*>(p.gamma + k));
            const float2 b = __ldg(reinterpret_cast<const float2*>(p.beta + k));
            const unsigned long long g2 = f2pack(g.x, g.y), b2 = f2pack(b.x, b.y);
            bool r = true;
            if (lane == 0)
                r = mbar_wait(smem_u32(&tail->full[s]), (kb / STAGES) & 1, abort, p.status,
                              ST_TIMEOUT_SOFTMAX, 0x400 + kb);
            ok = __all_sync(kFull, r);
            if (!ok) break;
            const uint8_t* xs = sX(s) + sub * 32 * (BK * 4) + lane * 8;
            uint8_t* tile = sA(s) + sub * 32 * 128 + off;
            // y = (x * rstd - mean * rstd) * gamma + beta, two packed FMAs a
            // pair. Sixteen rows are read before any is written: the stores
            // may alias the loads as far as the compiler knows, so mixing them
            // would serialise every row's latency.
#pragma unroll
            for (int h = 0; h < 32; h += 16) {
                float2 xv[16];
#pragma unroll
                for (int r2 = 0; r2 < 16; ++r2)
                    xv[r2] = *reinterpret_cast<const float2*>(xs + (h + r2) * (BK * 4));
#pragma unroll
                for (int r2 = 0; r2 < 16; ++r2) {
                    const int rr = h + r2;
                    const unsigned long long t2 = ffma2(f2pack(xv[r2].x, xv[r2].y),
                                                        f2pack(ra[rr], ra[rr]),
                                                        f2pack(rc2[rr], rc2[rr]));
                    float y0, y1;
                    f2unpack(ffma2(t2, g2, b2), y0, y1);
                    *reinterpret_cast<uint32_t*>(tile + rr * 128 + ((chunk ^ (rr & 7)) << 4)) =
                        pack2(y0, y1, dt);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tail->conv[s]));
        }
        // ------------------------------------------------------ epilogue
        const RowCtx rc = row_ctx(p, m0 + row);
        stage_vectors<BN>(p, tail, n0);
        epilogue_all(true);
        float rv0[32];
        prefetch_residual(p, rc, n0, rv0);
        if (ok) ok = mbar_wait(smem_u32(&tail->acc_full[0]), 0, abort, p.status,
                               ST_TIMEOUT_SOFTMAX, 0xE);
        if (epilogue_all(ok)) {
            tc_fence_after();
            store_tile<BN>(p, tail, tmem + (static_cast<uint32_t>(sub * 32) << 16), n0, rc, rv0,
                           p.tma_store ? &tm_o : nullptr, epi + sub * kEpiBlock,
                           m0 + sub * 32 + p.out_row_offset);
        }
        if (p.tma_store && lane == 0) bulk_wait_all();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
}

// The 3x3 convolution (stride 1, zero padding 1) of an NHWC f32 image as an
// implicit GEMM: row m of A is output pixel m, and K column (ky 3 + kx) cin +
// ci holds input pixel (y + ky - 1, x + kx - 1), channel ci (the tap-major
// order of the weights). Nothing is gathered in memory. A k-block of 64
// columns is two halves of 32 channels of one tap each (cin a multiple of
// 32); for each half the producer copies, by TMA, the 128 input pixels that
// the tile's rows read through that tap: a 128 x 32 f32 box starting at
// pixel m0 + (ky - 1) w + (kx - 1), rows before the image or past its end
// zero-filled by the copy. The four epilogue warps, idle until the
// accumulator is ready, turn the two halves into the 16-bit A tile in the
// MMA's swizzled layout, applying the optional ReLU and zeroing the pixels
// whose tap column falls outside the image (x + kx - 1 < 0 or >= w, which
// the flat copy wraps into the neighbouring row), then run the epilogue.
// One tile per CTA.
// A stage: the two f32 halves (TMA destinations, 128-byte aligned), the A
// tile (1024-byte aligned for the 128-byte swizzle), the B tile. A warp's
// 8-byte reads of a row are served per half-warp, 128 contiguous bytes of
// one half each, so the halves need no offset against bank conflicts.
constexpr uint32_t kConvHalf = BM * 32 * 4;  // 16 KiB: 128 pixels x 32 f32 channels
constexpr uint32_t kConvX1 = kConvHalf;
constexpr uint32_t kConvA = 2 * kConvHalf;
static_assert(kConvX1 % 128 == 0 && kConvA % 1024 == 0, "TMA and swizzle alignment");

template <int BN>
struct ConvLayout {
    static constexpr uint32_t kTileB = BN * BK * 2;
    static constexpr uint32_t kB = kConvA + kTileA;
    static constexpr uint32_t kStage = (kB + kTileB + 1023) / 1024 * 1024;
    static_assert(kB % 1024 == 0, "B tile alignment");
    static constexpr int kStages =
        static_cast<int>((kSmemLimit - 4096 - kEpiBytes) / kStage) < kMaxStages
            ? static_cast<int>((kSmemLimit - 4096 - kEpiBytes) / kStage)
            : kMaxStages;
};

template <int BN>
constexpr size_t conv_smem_bytes() {
    return 1024 + ConvLayout<BN>::kStages * ConvLayout<BN>::kStage + kEpiBytes + sizeof(Tail);
}

// Half h of k-block kb: K columns [64 kb + 32 h, + 32), or none past conv_k.
struct ConvHalf {
    bool live;
    int kx, x, y;  // tap column; the copy's start (channel, pixel)
};
__device__ __forceinline__ ConvHalf conv_half(const Params& p, int kb, int h, int m0) {
    ConvHalf c{};
    const int kk = kb * BK + 32 * h;
    c.live = kk < p.conv_k;
    if (c.live) {
        const int tap = kk / p.conv_cin;
        const int ky = tap / 3;
        c.kx = tap - 3 * ky;
        c.x = kk - tap * p.conv_cin;
        c.y = m0 + (ky - 1) * p.conv_w + (c.kx - 1);
    }
    return c;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_conv(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_b,
              const __grid_constant__ CUtensorMap tm_o, const Params p) {
    using L = ConvLayout<BN>;
    constexpr int STAGES = L::kStages;
    static_assert(STAGES >= 2, "a stage ring needs two stages");
    constexpr uint32_t kCols = Layout<BN>::kTmemCols;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* epi = smem + STAGES * L::kStage;
    Tail* tail = reinterpret_cast<Tail*>(epi + kEpiBytes);
    volatile int* abort = &tail->abort;
    auto sX = [&](int s, int h) { return smem + s * L::kStage + (h ? kConvX1 : 0u); };
    auto sA = [&](int s) { return smem + s * L::kStage + kConvA; };
    auto sB = [&](int s) { return smem + s * L::kStage + L::kB; };

    const int warp = warp_id();
    const int lane = lane_id();
    const int nk = p.K / BK;
    const int t = static_cast<int>(blockIdx.x);  // the grid has one CTA per tile
    const int m0 = (p.m_tile0 + t % p.m_tiles) * BM;
    const int n0 = (t / p.m_tiles) * BN;
    // bytes a stage's copies bring: B and the live halves
    auto stage_bytes = [&](int kb) {
        return L::kTileB + (conv_half(p, kb, 0, m0).live ? kConvHalf : 0u) +
               (conv_half(p, kb, 1, m0).live ? kConvHalf : 0u);
    };

    if (threadIdx.x == 0) {
        trace_stamp(p.trace, 0);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&tail->full[s]), 1);
            mbar_init(smem_u32(&tail->conv[s]), 4);
            mbar_init(smem_u32(&tail->empty[s]), 1);
        }
        mbar_init(smem_u32(&tail->acc_full[0]), 1);
        mbar_init(smem_u32(&tail->drain), 1);
        tail->abort = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
        tma_prefetch_desc(&tm_x);
        tma_prefetch_desc(&tm_b);
        if (p.tma_store) tma_prefetch_desc(&tm_o);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tail->tmem_base), kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tail->tmem_base;
    if (threadIdx.x == 0) trace_stamp(p.trace, 1);
    pdl_trigger();

    if (warp == 0) {
        // lane 0 arms each stage and copies input half 0, lane 2 copies half
        // 1 and lane 1 copies B (with weights_static the first stages' B
        // before the dependency wait): a thread's bulk copies complete one
        // after another, so the three are issued by three threads
        const int first = !p.weights_static ? 0 : (STAGES < nk ? STAGES : nk);
        for (int g = 0; g < first; ++g) {
            const uint32_t bar = smem_u32(&tail->full[g]);
            if (lane == 0) mbar_arrive_expect_tx(bar, stage_bytes(g));
            if (lane == 1) tma_load_3d(smem_u32(sB(g)), &tm_b, 0, n0, g, bar);
        }
        pdl_wait();
        if (lane == 0) trace_stamp(p.trace, 2);
        int g = 0;
        for (; g < nk; ++g) {
            const int s = g % STAGES;
            bool r = true;
            if (lane == 0 && g >= STAGES)
                r = mbar_wait(smem_u32(&tail->empty[s]), ((g / STAGES) - 1) & 1, abort, p.status,
                              ST_TIMEOUT_TMA, g);
            if (!__all_sync(0xFFFFFFFFu, r)) break;
            const uint32_t bar = smem_u32(&tail->full[s]);
            if (lane == 0 && g >= first) mbar_arrive_expect_tx(bar, stage_bytes(g));
            __syncwarp();  // the stage is armed before any of its copies can land
            if (lane == 0 || lane == 2) {
                const int h = lane >> 1;
                const ConvHalf c = conv_half(p, g, h, m0);
                if (c.live) tma_load_2d(smem_u32(sX(s, h)), &tm_x, c.x, c.y, bar);
            } else if (lane == 1 && g >= first) {
                tma_load_3d(smem_u32(sB(s)), &tm_b, 0, n0, g, bar);
            }
            __syncwarp();
        }
        if (lane == 0 && *abort) {
            for (int s = 0; s < STAGES && s < g; ++s) {
                const int uses = (g - s - 1) / STAGES + 1;
                mbar_wait(smem_u32(&tail->full[s]), (uses - 1) & 1, nullptr, p.status,
                          ST_TIMEOUT_DRAIN, s);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        const bool elected = elect_one();
        const uint32_t idesc = idesc_f16(BM, BN, p.ab_fmt, p.ab_fmt, 0, 0);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            bool r = true;
            if (elected)
                r = mbar_wait(smem_u32(&tail->conv[s]), (kb / STAGES) & 1, abort, p.status,
                              ST_TIMEOUT_MMA, kb);
            ok = __all_sync(0xFFFFFFFFu, r);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a = smem_u32(sA(s)), b = smem_u32(sB(s));
            if (elected) {
#pragma unroll
                for (int k = 0; k < BK / 16; ++k)
                    mma_ss(tmem, desc_k(a + 32 * k), desc_k(b + 32 * k), idesc,
                           (kb > 0 || k > 0) ? 1u : 0u);
                if (kb + STAGES < nk) mma_commit(smem_u32(&tail->empty[s]));
            }
            __syncwarp();
        }
        if (elected) {
            if (ok) {
                mma_commit(smem_u32(&tail->acc_full[0]));
            } else {
                mma_commit(smem_u32(&tail->drain));
                mbar_wait(smem_u32(&tail->drain), 0, nullptr, p.status, ST_TIMEOUT_DRAIN, 0xD);
            }
        }
        __syncwarp();
    } else {
        constexpr unsigned kFull = 0xFFFFFFFFu;
        const int sub = warp & 3;
        const int row = sub * 32 + lane;
        const int dt = p.ab_fmt ? BL_BF16 : BL_F16;
        pdl_wait();  // the residual read by the epilogue comes from the previous kernels
        // Pixels of this warp's 32 rows in the image's first and last column
        // (bit r: row sub * 32 + r): their left / right taps are outside.
        const int col = (m0 + row) % p.conv_w;
        const unsigned left = __ballot_sync(kFull, col == 0);
        const unsigned right = __ballot_sync(kFull, col == p.conv_w - 1);
        // lane L converts K columns 2L and 2L + 1 of each row: half L / 16,
        // channels 2 (L % 16) and the next
        const int h = lane >> 4;
        const int chunk = lane >> 2, off = (lane & 3) * 4;
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
            const int s = kb % STAGES;
            const ConvHalf c = conv_half(p, kb, h, m0);
            const unsigned zero = !c.live ? ~0u : c.kx == 0 ? left : c.kx == 2 ? right : 0u;
            bool r = true;
            if (lane == 0)
                r = mbar_wait(smem_u32(&tail->full[s]), (kb / STAGES) & 1, abort, p.status,
                              ST_TIMEOUT_SOFTMAX, 0x400 + kb);
            ok = __all_sync(kFull, r);
            if (!ok) break;
            if (kb == 0 && threadIdx.x == 64) trace_stamp(p.trace, 3);
            const uint8_t* xs = sX(s, h) + sub * 32 * 128 + (lane & 15) * 8;
            uint8_t* tile = sA(s) + sub * 32 * 128 + off;
            // sixteen rows read before any is written (the stores may alias
            // the loads as far as the compiler knows)
#pragma unroll
            for (int h2 = 0; h2 < 32; h2 += 16) {
                float2 xv[16];
#pragma unroll
                for (int r2 = 0; r2 < 16; ++r2)
                    xv[r2] = *reinterpret_cast<const float2*>(xs + (h2 + r2) * 128);
#pragma unroll
                for (int r2 = 0; r2 < 16; ++r2) {
                    const int rr = h2 + r2;
                    float y0 = xv[r2].x, y1 = xv[r2].y;
                    if (p.conv_relu) y0 = fmaxf(y0, 0.0f), y1 = fmaxf(y1, 0.0f);
                    if ((zero >> rr) & 1u) y0 = 0.0f, y1 = 0.0f;
                    *reinterpret_cast<uint32_t*>(tile + rr * 128 + ((chunk ^ (rr & 7)) << 4)) =
                        pack2(y0, y1, dt);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tail->conv[s]));
        }
        if (threadIdx.x == 64) trace_stamp(p.trace, 4);
        // ------------------------------------------------------ epilogue
        const RowCtx rc = row_ctx(p, m0 + row);
        stage_vectors<BN>(p, tail, n0);
        epilogue_all(true);
        float rv0[32];
        prefetch_residual(p, rc, n0, rv0);
        if (ok) ok = mbar_wait(smem_u32(&tail->acc_full[0]), 0, abort, p.status,
                               ST_TIMEOUT_SOFTMAX, 0xE);
        if (threadIdx.x == 64) trace_stamp(p.trace, 5);
        if (epilogue_all(ok)) {
            tc_fence_after();
            store_tile<BN>(p, tail, tmem + (static_cast<uint32_t>(sub * 32) << 16), n0, rc, rv0,
                           p.tma_store ? &tm_o : nullptr, epi + sub * kEpiBlock,
                           m0 + sub * 32 + p.out_row_offset);
        }
        if (p.tma_store && lane == 0) bulk_wait_all();
        __syncwarp();
        if (threadIdx.x == 64) trace_stamp(p.trace, 6);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kCols);
    }
    if (threadIdx.x == 0) trace_stamp(p.trace, 7);
}

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
    }
    return n;
}

// How many clusters of two persistent CTAs (this kernel's shared memory)
// the device runs at once, queried once per kernel.
template <typename K>
int pair_clusters(K kern, size_t smem) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

template <int BN, int KC, int EPI, bool kPair, bool kSk>
int prepare_persistent(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                       const CUtensorMap& tn, const Params& p, Launch* out) {
    constexpr size_t smem = smem_bytes<kPair ? BN / 2 : BN, KC, true>();
    out->op = 2;
    auto kern = gemm_persistent<BN, KC, EPI, kPair, kSk>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    const int tiles = p.m_tiles * (p.N / BN);
    if constexpr (kPair) {
        static int clusters = 0;  // per kernel; the same on every B200
        if (clusters == 0) clusters = pair_clusters(kern, smem);
        if (clusters <= 0) return fail(BL_ERR_UNSUPPORTED, "gemm: no CTA pair fits an SM pair");
        const dim3 grid(2 * std::min(tiles, clusters));
        out->run = [=](cudaStream_t s) {
            return launch_k_cluster(kern, grid, dim3(kThreads), dim3(2, 1, 1), smem, s, ta, tb, to,
                                    tn, p);
        };
    } else {
        // stream-K: one CTA per piece up to one per SM
        const int work = p.sk_pieces > 1 ? tiles * p.sk_pieces : tiles;
        const dim3 grid(std::min(work, sm_count()));
        out->run = [=](cudaStream_t s) {
            return launch_k(kern, grid, dim3(kThreads), smem, s, ta, tb, to, tn, p);
        };
    }
    return BL_OK;
}

template <int BN, int EPI, bool kPair, bool kSk>
int prepare_persistent(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                       const CUtensorMap& tn, const Params& p, int kc, Launch* out) {
    // only the depths whose ring holds two stages are built
    constexpr int SB = kPair ? BN / 2 : BN;  // B rows a CTA holds
    if constexpr (Layout<SB, 4, true>::kStages >= 2)
        if (kc == 4) return prepare_persistent<BN, 4, EPI, kPair, kSk>(ta, tb, to, tn, p, out);
    if constexpr (Layout<SB, 2, true>::kStages >= 2)
        if (kc == 2) return prepare_persistent<BN, 2, EPI, kPair, kSk>(ta, tb, to, tn, p, out);
    if (kc != 1) return fail(BL_ERR_UNSUPPORTED, "gemm: no kernel for %d k-blocks per stage", kc);
    return prepare_persistent<BN, 1, EPI, kPair, kSk>(ta, tb, to, tn, p, out);
}

template <int BN, int KC, int EPI>
int prepare_split2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                   const Params& p, Launch* out) {
    constexpr size_t smem = split_smem_bytes<BN, KC>();
    out->op = 2;
    auto kern = gemm_split2<BN, KC, EPI>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    const dim3 grid(2 * p.m_tiles * (p.N / BN));
    out->run = [=](cudaStream_t s) {
        return launch_k_cluster(kern, grid, dim3(kThreads), dim3(2, 1, 1), smem, s, ta, tb, to, p);
    };
    return BL_OK;
}

// The epilogue form (store_tile's EPI) these arguments match exactly, or -1.
int epilogue_form(const Params& p) {
    if (!p.tma_store || p.scale != 1.0f || p.stats_out != nullptr || p.norm_out != nullptr)
        return -1;
    const bool wide = p.out_dtype == BL_F32, one_type = p.out_dtype_hi == p.out_dtype;
    const bool plain_tail = p.chan_scale == nullptr && p.residual == nullptr && !wide;
    if (plain_tail && p.act == 0) return 0;
    if (plain_tail && p.act == 3) return 1;
    if (p.act == 0 && p.chan_scale != nullptr && p.residual != nullptr && wide && one_type)
        return 2;
    return -1;
}

// The split form's stages: the most k-blocks (4, 2, 1) that divide K / 64
// and leave a ring of two stages beside the receive buffer and the staging.
int pick_kc_split(int bn, uint32_t k) {
    const uint32_t nk = k / BK;
    for (int kc : {4, 2}) {
        const uint32_t stage = kc * (kTileA + bn * BK * 2);
        if (nk % kc == 0 && (kSmemLimit - 4096 - kEpiBytes - BM * (bn / 2) * 4) / stage >= 2)
            return kc;
    }
    return 1;
}

template <int BN, int KC>
int prepare_split2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                   const Params& p, Launch* out) {
    switch (epilogue_form(p)) {
        case 0: return prepare_split2<BN, KC, 0>(ta, tb, to, p, out);
        case 1: return prepare_split2<BN, KC, 1>(ta, tb, to, p, out);
        case 2: return prepare_split2<BN, KC, 2>(ta, tb, to, p, out);
        default: return prepare_split2<BN, KC, -1>(ta, tb, to, p, out);
    }
}

template <int BN, bool kPair = false, bool kSk = false>
int prepare_persistent(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                       const CUtensorMap& tn, const Params& p, int kc, Launch* out) {
    switch (epilogue_form(p)) {
        case 0: return prepare_persistent<BN, 0, kPair, kSk>(ta, tb, to, tn, p, kc, out);
        case 1: return prepare_persistent<BN, 1, kPair, kSk>(ta, tb, to, tn, p, kc, out);
        case 2: return prepare_persistent<BN, 2, kPair, kSk>(ta, tb, to, tn, p, kc, out);
        default: return prepare_persistent<BN, -1, kPair, kSk>(ta, tb, to, tn, p, kc, out);
    }
}

// k-blocks per stage of the persistent kernel: the most (4, 2, 1) that divide
// K / 64 and still leave a ring of two stages beside the output staging.
int pick_kc(int bn, uint32_t k) {
    const uint32_t nk = k / BK;
    for (int kc : {4, 2}) {
        const uint32_t stage = kc * (kTileA + bn * BK * 2);
        if (nk % kc == 0 && (kSmemLimit - 4096 - kEpiBytes) / stage >= 2) return kc;
    }
    return 1;
}

// Stream-K pieces per tile for `tiles` tiles (the whole launch's) of `nk`
// stages of kc k-blocks, bn columns wide, on `sms` SMs: the count S (1 =
// whole tiles) that minimises an estimate of the busiest CTA's time in SM
// clocks: its pieces' stages (operand bytes at about 45 bytes per clock, as
// for the tile width), one slot's partial sums stored or loaded per piece at
// the same rate, and half of the finishing piece's S - 1 loads exposed. A
// split must beat whole tiles by a tenth.
int sk_pieces(long long tiles, int nk, int bn, int kc, int sms) {
    const double stage = kc * (kTileA + bn * BK * 2.0) / 45.0;
    const double slot = BM * bn * 4.0 / 45.0;
    auto cost = [&](int S) {
        const long long units = tiles * S;
        const long long grid = std::min<long long>(units, sms);
        const long long per = (units + grid - 1) / grid;
        const long long piece = (nk + S - 1) / S;
        return static_cast<double>(per * piece) * stage +
               (S > 1 ? static_cast<double>(per) * slot + 0.5 * (S - 1) * slot : 0.0);
    };
    const double whole = cost(1);
    int best = 1;
    double best_cost = whole;
    for (int S = 2; S <= std::min(nk, kMaxSkPieces); ++S)
        if (cost(S) < best_cost) best = S, best_cost = cost(S);
    return best_cost < 0.9 * whole ? best : 1;
}

// The workspace of a stream-K launch: a flag per (tile, piece) slot, padded
// to 256 bytes, then the slots' partial sums (128 x bn f32 each).
uint64_t sk_flag_bytes(long long slots) { return (4ull * slots + 255) / 256 * 256; }
uint64_t sk_workspace_bytes(long long tiles, int pieces, int bn) {
    const long long slots = tiles * pieces;
    return sk_flag_bytes(slots) + 4ull * BM * bn * slots;
}

int pick_bn(const bl_gemm_args& g);

// The form a launch takes when it can take stream-K: A by TMA into the
// one-CTA persistent kernel, no LayerNorm, epilogue LayerNorm, statistics,
// CTA pairs or K split. Returns the piece count from the whole launch's
// shape (1: whole tiles) and the tile width and stage depth.
int sk_form(const bl_gemm_args& g, int* bn_out, int* kc_out) {
    if (g.stream_k != 2 || g.ln_x != nullptr || g.norm_out != nullptr || g.stats_out != nullptr ||
        g.pair_tiles == 2 || g.k % BK != 0 || g.m == 0 || g.n == 0)
        return 1;
    const int bn = pick_bn(g);
    if ((bn != 128 && bn != 256) || g.n % bn != 0) return 1;
    const bool split_ok = g.n % 64 == 0 && (g.tile_n == 0 || g.tile_n == 64) && g.k / BK >= 4;
    const bool ksplit =
        g.split_k == 2 ||
        (g.split_k == 0 && split_ok && g.k >= 1024 && g.n <= 512 &&
         2ull * ((g.m + BM - 1) / BM) * (g.n / 64) <= static_cast<uint64_t>(sm_count()));
    if (ksplit) return 1;
    const int kc = pick_kc(bn, g.k);
    const int nk = static_cast<int>(g.k / (BK * kc));
    const long long tiles = static_cast<long long>((g.m + BM - 1) / BM) * (g.n / bn);
    int pieces = sk_pieces(tiles, nk, bn, kc, sm_count());
    if (pieces <= 1 && nk >= 2) pieces = 2;
    *bn_out = bn;
    *kc_out = kc;
    return pieces;
}

uint64_t sk_bytes(const bl_gemm_args& g) {
    int bn = 0, kc = 0;
    const int pieces = sk_form(g, &bn, &kc);
    if (pieces <= 1) return 0;
    return sk_workspace_bytes(static_cast<long long>((g.m + BM - 1) / BM) * (g.n / bn), pieces, bn);
}

template <int BN>
int prepare_ln_staged(const CUtensorMap& tx, const CUtensorMap& tb, const CUtensorMap& to,
                      const Params& p, Launch* out) {
    constexpr size_t smem = ln_smem_bytes<BN>();
    out->op = 2;
    auto kern = gemm_ln_staged<BN>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    const dim3 grid(p.m_tiles * (p.N / BN));
    out->run = [=](cudaStream_t s) {
        return launch_k(kern, grid, dim3(kThreads), smem, s, tx, tb, to, p);
    };
    return BL_OK;
}

template <int BN>
int prepare_conv(const CUtensorMap& tx, const CUtensorMap& tb, const CUtensorMap& to,
                 const Params& p, Launch* out) {
    constexpr size_t smem = conv_smem_bytes<BN>();
    out->op = 2;
    auto kern = gemm_conv<BN>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    const dim3 grid(p.m_tiles * (p.N / BN));
    out->run = [=](cudaStream_t s) {
        return launch_k(kern, grid, dim3(kThreads), smem, s, tx, tb, to, p);
    };
    return BL_OK;
}

template <int BN, bool kLn>
int prepare_t(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, Launch* out) {
    constexpr size_t smem = smem_bytes<BN>();
    out->op = 2;
    auto kern = gemm_kernel<BN, kLn>;
    BL_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    const dim3 grid(p.m_tiles, p.N / BN);
    out->run = [=](cudaStream_t s) {
        return launch_k(kern, grid, dim3(kThreads), smem, s, ta, tb, p);
    };
    return BL_OK;
}

// norm_sync: the counters (two per row tile), then float2 [m][n / 32]
uint64_t norm_ctr_bytes(uint32_t m) { return ((8ull * ((m + BM - 1) / BM)) + 15) & ~15ull; }
uint64_t norm_sync_bytes(uint32_t m, uint32_t n) {
    return norm_ctr_bytes(m) + 8ull * m * (n / 32);
}

int pick_bn(const bl_gemm_args& g) {
    if (g.tile_n) return static_cast<int>(g.tile_n);
    const int mt = static_cast<int>((g.m + BM - 1) / BM);
    const int cands[4] = {128, 96, 64, 32};
    if (g.ln_x == nullptr) {
        const int wide[5] = {256, 128, 96, 64, 32};  // the persistent kernel's widths
        // Persistent grid: the busiest CTA's tiles times a tile's cost. A
        // k-block is bound by its operand bytes arriving (measured about 45
        // bytes per SM clock from L2); the epilogue costs about 600 clocks
        // per 32 columns. Ties go to the wider tile. (Adding the L2's total
        // delivery as a bound picked 64 columns for ViT-S fc2, measured 10 %
        // slower than 32.)
        const long long nk = g.k / BK, sms = sm_count();
        int best = 0;
        long long best_cost = 0;
        for (int bn : wide) {
            if (g.n % bn != 0) continue;
            const long long tiles = static_cast<long long>(mt) * (g.n / bn);
            const long long per_cta = (tiles + sms - 1) / sms;
            const long long tile = nk * (kTileA + bn * BK * 2) / 45 + 600LL * (bn / 32);
            const long long cost = per_cta * tile;
            if (best == 0 || cost < best_cost) best = bn, best_cost = cost;
        }
        return best;
    }
    // One tile per CTA: the widest tile whose grid still fills the SMs.
    for (int bn : cands)
        if (g.n % bn == 0 && mt * static_cast<int>(g.n / bn) >= 120) return bn;
    for (int i = 3; i >= 0; --i)
        if (g.n % cands[i] == 0) return cands[i];
    return 0;
}

int prepare(const bl_gemm_args& g, uint32_t row_begin, uint32_t row_end, Launch* out,
            const bl_conv3x3_args* conv = nullptr) {
    if (g.m == 0 || g.n == 0 || g.k == 0) return fail(BL_ERR_INVALID, "gemm: zero dimension");
    if (g.k % BK != 0) return fail(BL_ERR_UNSUPPORTED, "gemm: K=%u is not a multiple of 64", g.k);
    if (g.ab_dtype != BL_F16 && g.ab_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "gemm: operand dtype %d (f16 or bf16)", g.ab_dtype);
    int bn = pick_bn(g);
    if (conv != nullptr) {
        // implicit 3x3 convolution: A is the image, tiles of at most 128 columns
        if (conv->input == nullptr || conv->h == 0 || conv->w == 0 || conv->cin == 0)
            return fail(BL_ERR_INVALID, "conv3x3: empty image or null input");
        if (conv->cin % 32 != 0)
            return fail(BL_ERR_UNSUPPORTED, "conv3x3: %u channels (a multiple of 32)", conv->cin);
        if (1ull * conv->h * conv->w != g.m)
            return fail(BL_ERR_INVALID, "conv3x3: m=%u is not h * w = %u x %u", g.m, conv->h,
                        conv->w);
        if (g.k != (9 * conv->cin + BK - 1) / BK * BK)
            return fail(BL_ERR_INVALID, "conv3x3: k=%u is not 9 x %u channels rounded up to 64",
                        g.k, conv->cin);
        if (reinterpret_cast<uintptr_t>(conv->input) & 15)
            return fail(BL_ERR_INVALID, "conv3x3: input must be 16-byte aligned");
        if (g.a != nullptr || g.ln_x != nullptr || g.norm_out != nullptr || g.stats_out != nullptr)
            return fail(BL_ERR_INVALID, "conv3x3: the image is A (no a, LayerNorm or statistics)");
        if (1ull * g.m + conv->w + 1 >= (1ull << 31))
            return fail(BL_ERR_UNSUPPORTED, "conv3x3: %u pixels exceed 32-bit coordinates", g.m);
        bn = g.tile_n ? static_cast<int>(g.tile_n)
                      : g.n % 128 == 0 ? 128 : g.n % 96 == 0 ? 96 : g.n % 64 == 0 ? 64 : 32;
        if (bn > 128)
            return fail(BL_ERR_UNSUPPORTED, "conv3x3: tile width %d (at most 128)", bn);
    }
    if (g.stats_out != nullptr) {
        // one stats slice per column tile
        if (g.stats_parts == 0 || g.n % g.stats_parts != 0)
            return fail(BL_ERR_INVALID, "gemm: %u stats parts do not divide N=%u", g.stats_parts, g.n);
        const uint32_t w = g.n / g.stats_parts;
        if (g.tile_n && g.tile_n != w)
            return fail(BL_ERR_INVALID, "gemm: tile width %u differs from the stats slice %u",
                        g.tile_n, w);
        if (g.out_dtype != BL_F32 || (g.split_col > 0 && g.split_col < g.n))
            return fail(BL_ERR_INVALID, "gemm: row statistics need an f32 output of one type");
        if (reinterpret_cast<uintptr_t>(g.stats_out) & 7)
            return fail(BL_ERR_INVALID, "gemm: stats output must be 8-byte aligned");
        bn = static_cast<int>(w);
    }
    const bool norm = g.norm_out != nullptr;
    if (norm) {
        if (g.tile_n && g.tile_n != 32)
            return fail(BL_ERR_UNSUPPORTED, "gemm: the epilogue LayerNorm needs 32-column tiles");
        bn = 32;
    }
    const bool dot = g.dot_w != nullptr;
    if (dot) {
        if (g.n > 128 || (g.tile_n && g.tile_n != g.n))
            return fail(BL_ERR_UNSUPPORTED, "gemm: a row reduction takes one column tile (N=%u, "
                                            "at most 128)", g.n);
        if (g.out_dtype != BL_F32 || (g.split_col > 0 && g.split_col < g.n) ||
            g.out_group_rows != 0 || g.out_row_offset != 0 || g.stats_out != nullptr || norm ||
            g.ln_x != nullptr || g.pair_tiles == 2 || g.split_k == 2 || g.stream_k == 2)
            return fail(BL_ERR_UNSUPPORTED,
                        "gemm: a row reduction needs an f32 output of one type without row groups "
                        "or offset, and no statistics, LayerNorm, CTA pairs, K split or stream-K");
        if (g.dot_act != 0 && g.dot_act != 1)
            return fail(BL_ERR_INVALID, "gemm: row reduction activation %d (0 or 1)", g.dot_act);
        if (reinterpret_cast<uintptr_t>(g.dot_w) & 15)
            return fail(BL_ERR_INVALID, "gemm: row reduction weights must be 16-byte aligned");
        bn = static_cast<int>(g.n);
    }
    if (bn == 0 || g.n % bn != 0 ||
        (bn != 32 && bn != 64 && bn != 96 && bn != 128 && bn != 256))
        return fail(BL_ERR_UNSUPPORTED, "gemm: N=%u has no tile width (32/64/96/128/256)", g.n);
    const bool ln = g.ln_x != nullptr;
    if (bn == 256 && ln)
        return fail(BL_ERR_UNSUPPORTED, "gemm: 256-column tiles take A loaded by TMA, not a "
                                        "LayerNorm prologue");
    if (norm) {
        const uint64_t tiles = ((static_cast<uint64_t>(g.m) + BM - 1) / BM) * (g.n / 32);
        if (ln || g.out_dtype != BL_F32 || (g.split_col > 0 && g.split_col < g.n) ||
            g.out_group_rows != 0 || g.stats_out != nullptr)
            return fail(BL_ERR_UNSUPPORTED,
                        "gemm: the epilogue LayerNorm needs an f32 output of one type, no row "
                        "groups, no LayerNorm prologue and no statistics output");
        if (g.n > 32 * kMaxNormParts)
            return fail(BL_ERR_UNSUPPORTED, "gemm: the epilogue LayerNorm takes rows of at most %d "
                        "columns", 32 * kMaxNormParts);
        if (tiles > static_cast<uint64_t>(sm_count()))
            return fail(BL_ERR_UNSUPPORTED,
                        "gemm: the epilogue LayerNorm needs every tile resident (%llu tiles, %d "
                        "SMs)", (unsigned long long)tiles, sm_count());
        if (row_begin != 0 || row_end < g.m)
            return fail(BL_ERR_UNSUPPORTED, "gemm: the epilogue LayerNorm covers whole launches");
        if (g.norm_out_dtype != BL_F16 && g.norm_out_dtype != BL_BF16)
            return fail(BL_ERR_INVALID, "gemm: LayerNorm output dtype %d (f16 or bf16)",
                        g.norm_out_dtype);
        const uint64_t nld = g.norm_out_ld ? g.norm_out_ld : g.n;
        if ((reinterpret_cast<uintptr_t>(g.norm_out) & 15) || (nld * 2) % 16 ||
            g.norm_gamma == nullptr || g.norm_beta == nullptr ||
            (reinterpret_cast<uintptr_t>(g.norm_gamma) & 15) ||
            (reinterpret_cast<uintptr_t>(g.norm_beta) & 15))
            return fail(BL_ERR_INVALID,
                        "gemm: LayerNorm output rows and gamma / beta must be 16-byte aligned");
        if (g.norm_sync == nullptr || (reinterpret_cast<uintptr_t>(g.norm_sync) & 15) ||
            g.norm_sync_bytes < norm_sync_bytes(g.m, g.n))
            return fail(BL_ERR_INVALID, "gemm: norm_sync must be 16-byte aligned and hold %llu bytes",
                        (unsigned long long)norm_sync_bytes(g.m, g.n));
    }
    if (g.ln_stats != nullptr &&
        (!ln || g.ln_stats_parts == 0 || g.k % g.ln_stats_parts != 0 ||
         (reinterpret_cast<uintptr_t>(g.ln_stats) & 7)))
        return fail(BL_ERR_INVALID,
                    "gemm: LayerNorm statistics need the LayerNorm prologue, parts dividing K=%u "
                    "and 8-byte alignment", g.k);
    if (!ln && g.a == nullptr && conv == nullptr) return fail(BL_ERR_INVALID, "gemm: no A operand");
    if (ln && (g.ln_gamma == nullptr || g.ln_beta == nullptr || !(g.ln_eps > 0.0f)))
        return fail(BL_ERR_INVALID, "gemm: LayerNorm prologue needs gamma, beta and eps > 0");
    if (ln && ((reinterpret_cast<uintptr_t>(g.ln_x) & 15) || (g.ln_ldx % 4) || g.ln_ldx < g.k))
        return fail(BL_ERR_INVALID, "gemm: LayerNorm input must be 16-byte aligned rows");
    if (g.out == nullptr) return fail(BL_ERR_INVALID, "gemm: null output");
    const bool split = g.split_col > 0 && g.split_col < g.n;
    const int dts[2] = {g.out_dtype, split ? g.out_dtype_hi : g.out_dtype};
    for (int dt : dts)
        if (dt != BL_F32 && dt != BL_F16 && dt != BL_BF16)
            return fail(BL_ERR_INVALID, "gemm: output dtype %d", dt);
    const uint64_t out_ld = g.out_ld ? g.out_ld : g.n;
    if ((reinterpret_cast<uintptr_t>(g.out) & 15) || (out_ld * 2) % 16 ||
        (g.out_dtype == BL_F32 && (out_ld * 4) % 16))
        return fail(BL_ERR_INVALID, "gemm: output must be 16-byte aligned rows");
    if (split && g.split_col % 32)
        return fail(BL_ERR_INVALID, "gemm: split column must be a multiple of 32");
    if ((g.bias && (reinterpret_cast<uintptr_t>(g.bias) & 15)) ||
        (g.chan_scale && (reinterpret_cast<uintptr_t>(g.chan_scale) & 15)))
        return fail(BL_ERR_INVALID, "gemm: bias/scale vectors must be 16-byte aligned");
    if (g.act < 0 || g.act > 3) return fail(BL_ERR_INVALID, "gemm: activation %d", g.act);
    if (ln && ((reinterpret_cast<uintptr_t>(g.ln_gamma) & 15) ||
               (reinterpret_cast<uintptr_t>(g.ln_beta) & 15)))
        return fail(BL_ERR_INVALID, "gemm: LayerNorm gamma/beta must be 16-byte aligned");
    if (g.residual != nullptr) {
        const uint64_t rld = g.res_ld ? g.res_ld : g.n;
        const uint64_t esz = g.res_dtype == BL_F32 ? 4 : 2;
        if ((reinterpret_cast<uintptr_t>(g.residual) & 15) || (rld * esz) % 16 ||
            (g.res_dtype != BL_F32 && g.res_dtype != BL_F16 && g.res_dtype != BL_BF16))
            return fail(BL_ERR_INVALID, "gemm: residual must be 16-byte aligned rows");
    }

    CUtensorMap ta{}, tb{};
    int rc;
    // A LayerNorm prologue whose statistics were left by the GEMM that wrote
    // x runs with its rows brought by TMA when every tile fits one CTA per SM
    // (gemm_ln_staged); otherwise, or without statistics, the epilogue warps
    // load the rows (gemm_kernel).
    const uint64_t ldx = g.ln_ldx ? g.ln_ldx : g.k;
    const uint64_t row_tiles = (std::min(row_end, g.m) + BM - 1) / BM - row_begin / BM;
    const bool staged = ln && g.ln_stats != nullptr && g.ln_stats_parts <= kMaxNormParts &&
                        row_tiles * (g.n / bn) <= static_cast<uint64_t>(sm_count()) &&
                        (ldx * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(g.ln_x) & 15) == 0;
    // 256-row tiles over CTA pairs (pair_tiles 2): whole launches with A
    // loaded by TMA, tiles 128 or 256 columns wide; 0 and 1 keep one CTA
    // per tile.
    if (g.pair_tiles > 2) return fail(BL_ERR_INVALID, "gemm: pair_tiles %u (0, 1 or 2)", g.pair_tiles);
    const bool pair = g.pair_tiles == 2;
    if (pair) {
        if (ln || norm || conv != nullptr || g.a == nullptr)
            return fail(BL_ERR_UNSUPPORTED, "gemm: CTA pairs take A loaded by TMA (no LayerNorm "
                                            "prologue, epilogue LayerNorm or convolution)");
        if (row_begin != 0 || row_end < g.m)
            return fail(BL_ERR_UNSUPPORTED, "gemm: CTA pairs cover whole launches");
        if (!g.tile_n) bn = g.n % 256 == 0 ? 256 : 128;
        if ((bn != 128 && bn != 256) || g.n % bn != 0)
            return fail(BL_ERR_UNSUPPORTED, "gemm: CTA pairs take 128- or 256-column tiles (N=%u)",
                        g.n);
    }
    // The K range split over a cluster of two CTAs (split_k 2, or 0 for
    // K >= 1024 with N <= 512 in 64-column tiles, a rule of the shape alone so
    // row parts split exactly as their whole launch): 64-column tiles.
    if (g.split_k > 2) return fail(BL_ERR_INVALID, "gemm: split_k %u (0, 1 or 2)", g.split_k);
    const bool split_ok = !ln && !norm && !dot && conv == nullptr && g.a != nullptr &&
                          g.stats_out == nullptr && !pair && g.n % 64 == 0 &&
                          (g.tile_n == 0 || g.tile_n == 64) && g.k / BK >= 4;
    // (the automatic rule also asks that both CTAs of every tile of the whole
    // launch, m rows, fit one wave; m is the whole launch's for a row part)
    const bool ksplit =
        g.split_k == 2 ||
        (g.split_k == 0 && split_ok && g.k >= 1024 && g.n <= 512 &&
         2ull * ((g.m + BM - 1) / BM) * (g.n / 64) <= static_cast<uint64_t>(sm_count()));
    if (ksplit) {
        if (!split_ok)
            return fail(BL_ERR_UNSUPPORTED, "gemm: the K split takes A loaded by TMA, N a multiple "
                                            "of 64, 64-column tiles, K >= 256, no LayerNorm, "
                                            "statistics, CTA pairs or convolution");
        bn = 64;
    }
    const int kc = ln ? 1 : ksplit ? pick_kc_split(bn, g.k) : pick_kc(pair ? bn / 2 : bn, g.k);
    // Stream-K on request (sk_form: pieces from the whole launch's shape) on
    // the persistent path
    if (g.stream_k > 2) return fail(BL_ERR_INVALID, "gemm: stream_k %u (0, 1 or 2)", g.stream_k);
    int pieces = 1;
    const long long whole_tiles = static_cast<long long>((g.m + BM - 1) / BM) * (g.n / bn);
    {
        const bool sk_path = !ln && !norm && conv == nullptr && !pair && !ksplit && !staged &&
                             g.a != nullptr && g.stats_out == nullptr;
        int sbn = 0, skc = 0;
        int want = sk_path ? sk_form(g, &sbn, &skc) : 1;
        if (want > 1 && (sbn != bn || skc != kc)) want = 1;
        if (g.stream_k == 2 && want <= 1)
            return fail(BL_ERR_UNSUPPORTED,
                        "gemm: stream-K takes A loaded by TMA into one CTA per 128- or "
                        "256-column tile (no LayerNorm, statistics, CTA pairs, K split or "
                        "convolution) and at least two stages of K");
        if (want > 1) {
            const uint64_t need = sk_workspace_bytes(whole_tiles, want, bn);
            if (g.workspace == nullptr || g.workspace_bytes < need ||
                (reinterpret_cast<uintptr_t>(g.workspace) & 15) != 0)
                return fail(BL_ERR_INVALID,
                            "gemm: stream-K needs a 16-byte aligned workspace of %llu bytes",
                            (unsigned long long)need);
            pieces = want;
        }
    }
    const uint64_t ldb = g.ldb ? g.ldb : g.k;
    if (conv != nullptr) {
        // the image as [pixels][channels] f32 rows, boxes of 32 channels x 128 pixels
        const uint64_t dx[2] = {conv->cin, g.m};
        const uint32_t bx[2] = {32, BM};
        if ((rc = make_tmap_2d(&ta, conv->input, 4, dx, 4ull * conv->cin, bx, 0)) != BL_OK)
            return rc;
        const uint64_t db[3] = {BK, g.n, g.k / BK}, sb[2] = {ldb * 2, BK * 2};
        const uint32_t bb[3] = {BK, static_cast<uint32_t>(bn), 1};
        if ((rc = make_tmap_16bit_3d(&tb, g.b, db, sb, bb)) != BL_OK) return rc;
    } else if (staged) {
        const uint64_t dx[2] = {g.k, g.m};
        const uint32_t bx[2] = {BK, BM};
        if ((rc = make_tmap_2d(&ta, g.ln_x, 4, dx, ldx * 4, bx, 0)) != BL_OK) return rc;
        const uint64_t db[3] = {BK, g.n, g.k / BK}, sb[2] = {ldb * 2, BK * 2};
        const uint32_t bb[3] = {BK, static_cast<uint32_t>(bn), 1};
        if ((rc = make_tmap_16bit_3d(&tb, g.b, db, sb, bb)) != BL_OK) return rc;
    } else if (!ln) {
        // Persistent kernel: 3-D views (64 columns, rows, 64-column block)
        // so one copy brings kc consecutive k-blocks of 128 (A) or bn (B)
        // rows.
        const uint64_t lda = g.lda ? g.lda : g.k;
        const uint64_t da[3] = {BK, g.m, g.k / BK}, sa[2] = {lda * 2, BK * 2};
        const uint32_t ba[3] = {BK, BM, static_cast<uint32_t>(kc)};
        if ((rc = make_tmap_16bit_3d(&ta, g.a, da, sa, ba)) != BL_OK) return rc;
        const uint64_t db[3] = {BK, g.n, g.k / BK}, sb[2] = {ldb * 2, BK * 2};
        const uint32_t bb[3] = {BK, static_cast<uint32_t>(pair ? bn / 2 : bn),
                                static_cast<uint32_t>(kc)};
        if ((rc = make_tmap_16bit_3d(&tb, g.b, db, sb, bb)) != BL_OK) return rc;
    } else {
        const uint64_t dims[2] = {g.k, g.n};
        const uint32_t box[2] = {BK, static_cast<uint32_t>(bn)};
        if ((rc = make_tmap_16bit_2d(&tb, g.b, dims, ldb * 2, box)) != BL_OK) return rc;
    }
    Params p{};
    p.M = static_cast<int>(g.m);
    p.N = static_cast<int>(g.n);
    p.K = static_cast<int>(g.k);
    p.ab_fmt = g.ab_dtype == BL_BF16 ? 1 : 0;
    p.x = static_cast<const float*>(g.ln_x);
    p.ldx = static_cast<long long>(g.ln_ldx ? g.ln_ldx : g.k);
    p.gamma = g.ln_gamma;
    p.beta = g.ln_beta;
    p.eps = g.ln_eps;
    p.bias = g.bias;
    p.act = g.act;
    p.scale = g.scale == 0.0f ? 1.0f : g.scale;
    p.chan_scale = g.chan_scale;
    p.residual = g.residual;
    p.res_dtype = g.res_dtype;
    p.res_ld = static_cast<long long>(g.res_ld ? g.res_ld : g.n);
    p.res_period = static_cast<int>(g.res_period);
    p.out = g.out;
    p.out_dtype = g.out_dtype;
    p.out_dtype_hi = split ? g.out_dtype_hi : g.out_dtype;
    p.split_col = split ? static_cast<int>(g.split_col) : static_cast<int>(g.n);
    p.out_ld = static_cast<long long>(out_ld);
    p.out_row_offset = static_cast<int>(g.out_row_offset);
    p.out_group_rows = static_cast<int>(g.out_group_rows);
    p.out_group_gap = static_cast<int>(g.out_group_gap);
    p.stats_out = static_cast<float2*>(g.stats_out);
    p.stats_parts = static_cast<int>(g.stats_parts);
    p.ln_stats = static_cast<const float2*>(g.ln_stats);
    p.ln_stats_parts = static_cast<int>(g.ln_stats_parts);
    p.weights_static = g.weights_static ? 1 : 0;
    p.m_tile0 = static_cast<int>(row_begin / BM);
    p.m_tiles = static_cast<int>((std::min(row_end, g.m) + BM - 1) / BM) - p.m_tile0;
    if (pair) p.m_tiles = static_cast<int>((g.m + 2 * BM - 1) / (2 * BM));  // 256-row tiles
    if (row_begin % BM != 0 || row_begin >= row_end || p.m_tiles <= 0)
        return fail(BL_ERR_INVALID, "gemm: row part [%u, %u) is not whole 128-row tiles", row_begin, row_end);
    p.status = status_ptr();
    p.trace = reinterpret_cast<unsigned long long*>(g.trace);
    if (dot) {
        p.dot_w = g.dot_w;
        p.dot_bias = g.dot_bias;
        p.dot_act = g.dot_act;
    }
    if (pieces > 1) {
        p.sk_pieces = pieces;
        p.sk_flag = static_cast<unsigned*>(g.workspace);
        p.sk_part = reinterpret_cast<float*>(static_cast<uint8_t*>(g.workspace) +
                                             sk_flag_bytes(whole_tiles * pieces));
    }
    if (conv != nullptr) {
        p.conv_w = static_cast<int>(conv->w);
        p.conv_pix = static_cast<int>(g.m);
        p.conv_cin = static_cast<int>(conv->cin);
        p.conv_k = static_cast<int>(9 * conv->cin);
        p.conv_relu = conv->relu ? 1 : 0;
    }
    if (ln && !staged) {
        switch (bn) {
            case 32: return prepare_t<32, true>(ta, tb, p, out);
            case 64: return prepare_t<64, true>(ta, tb, p, out);
            case 96: return prepare_t<96, true>(ta, tb, p, out);
            default: return prepare_t<128, true>(ta, tb, p, out);
        }
    }
    CUtensorMap tn{};
    if (norm) {
        const uint64_t nld = g.norm_out_ld ? g.norm_out_ld : g.n;
        const uint64_t dims[2] = {g.n, g.m};
        const uint32_t box[2] = {32, 32};
        if ((rc = make_tmap_2d(&tn, g.norm_out, 2, dims, nld * 2, box, 64)) != BL_OK)
            return rc;
        p.norm_out = g.norm_out;
        p.norm_dtype = g.norm_out_dtype;
        p.norm_gamma = g.norm_gamma;
        p.norm_beta = g.norm_beta;
        p.norm_eps = g.norm_eps;
        p.norm_ctr = static_cast<unsigned*>(g.norm_sync);
        p.norm_stats = reinterpret_cast<float2*>(static_cast<uint8_t*>(g.norm_sync) +
                                                 norm_ctr_bytes(g.m));
    }
    // Output rows leave through a tensor map when they form one strided 2-D
    // array of a single element size (no row groups).
    CUtensorMap to{};
    const int esz = static_cast<int>(dtype_size(dts[0]));
    if (!dot && g.out_group_rows == 0 && dtype_size(dts[1]) == dtype_size(dts[0])) {
        const uint64_t dims[2] = {g.n, static_cast<uint64_t>(g.m) + g.out_row_offset};
        const uint32_t box[2] = {32, 32};
        if ((rc = make_tmap_2d(&to, g.out, esz, dims, out_ld * esz, box,
                                     esz == 4 ? 128 : 64)) != BL_OK)
            return rc;
        p.tma_store = 1;
    }
    if (conv != nullptr) {
        switch (bn) {
            case 32: return prepare_conv<32>(ta, tb, to, p, out);
            case 64: return prepare_conv<64>(ta, tb, to, p, out);
            case 96: return prepare_conv<96>(ta, tb, to, p, out);
            default: return prepare_conv<128>(ta, tb, to, p, out);
        }
    }
    if (staged) {
        switch (bn) {
            case 32: return prepare_ln_staged<32>(ta, tb, to, p, out);
            case 64: return prepare_ln_staged<64>(ta, tb, to, p, out);
            case 96: return prepare_ln_staged<96>(ta, tb, to, p, out);
            default: return prepare_ln_staged<128>(ta, tb, to, p, out);
        }
    }
    if (pair)
        return bn == 256 ? prepare_persistent<256, true>(ta, tb, to, tn, p, kc, out)
                         : prepare_persistent<128, true>(ta, tb, to, tn, p, kc, out);
    if (ksplit) {
        // pick_kc_split keeps two stages: only those depths are built
        if constexpr (SplitLayout<64, 4>::kStages >= 2)
            if (kc == 4) return prepare_split2<64, 4>(ta, tb, to, p, out);
        if (kc == 2) return prepare_split2<64, 2>(ta, tb, to, p, out);
        return prepare_split2<64, 1>(ta, tb, to, p, out);
    }
    if (pieces > 1)  // sk_form takes stream-K for 128- and 256-column tiles only
        return bn == 256 ? prepare_persistent<256, false, true>(ta, tb, to, tn, p, kc, out)
                         : prepare_persistent<128, false, true>(ta, tb, to, tn, p, kc, out);
    switch (bn) {
        case 32: return prepare_persistent<32>(ta, tb, to, tn, p, kc, out);
        case 64: return prepare_persistent<64>(ta, tb, to, tn, p, kc, out);
        case 96: return prepare_persistent<96>(ta, tb, to, tn, p, kc, out);
        case 256: return prepare_persistent<256>(ta, tb, to, tn, p, kc, out);
        default: return prepare_persistent<128>(ta, tb, to, tn, p, kc, out);
    }
}

}  // namespace gemm

int prepare_gemm(const bl_gemm_args& g, Launch* out) { return gemm::prepare(g, 0, g.m, out); }
int prepare_gemm_rows(const bl_gemm_args& g, uint32_t row_begin, uint32_t row_end, Launch* out) {
    return gemm::prepare(g, row_begin, row_end, out);
}

}  // namespace bl

extern "C" size_t bl_gemm_workspace_bytes(const bl_gemm_args* args) {
    return args == nullptr ? 0 : static_cast<size_t>(bl::gemm::sk_bytes(*args));
}

extern "C" size_t bl_gemm_norm_sync_bytes(const bl_gemm_args* args) {
    return args == nullptr ? 0 : static_cast<size_t>(bl::gemm::norm_sync_bytes(args->m, args->n));
}

extern "C" int bl_conv3x3(const bl_gemm_args* args, const bl_conv3x3_args* conv, void* stream) {
    if (args == nullptr || conv == nullptr) return bl::fail(BL_ERR_INVALID, "conv3x3: null args");
    bl::Launch l;
    int rc = bl::gemm::prepare(*args, 0, args->m, &l, conv);
    return rc != BL_OK ? rc : bl::enqueue(l, static_cast<cudaStream_t>(stream));
}

extern "C" int bl_gemm(const bl_gemm_args* args, void* stream) {
    if (args == nullptr) return bl::fail(BL_ERR_INVALID, "gemm: null args");
    bl::Launch l;
    int rc = bl::prepare_gemm(*args, &l);
    return rc != BL_OK ? rc : bl::enqueue(l, static_cast<cudaStream_t>(stream));
}
