// Memory-bound helpers of the encoder: the standalone LayerNorm (the final
// norm, with TokensToMap folded in) and the embedding front (patch matrix for
// the patch-embedding GEMM, class token + position embedding).
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "host.h"

namespace bl {
namespace misc {

__device__ __forceinline__ uint16_t to16(float v, int dt) {
    if (dt == BL_BF16) {
        __nv_bfloat16 h = __float2bfloat16_rn(v);
        return *reinterpret_cast<uint16_t*>(&h);
    }
    __half h = __float2half_rn(v);
    return *reinterpret_cast<uint16_t*>(&h);
}

// One warp per output row. Two passes over the row held in registers
// (mean, then the biased variance of the deviations), as reference.rs:247-270
// defines the layer norm; f32 arithmetic.
template <int kPerLane>
__global__ void __launch_bounds__(256) layernorm_kernel(bl_layernorm_args a, int row_begin, int row_end) {
    pdl_trigger();
    pdl_wait();
    const int row = row_begin + static_cast<int>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= row_end) return;
    long long in_row = row;
    if (a.in_group_rows > 0) in_row += static_cast<long long>(row / a.in_group_rows) * a.in_group_gap;
    in_row += a.in_row_offset;
    const float* x = a.x + in_row * static_cast<long long>(a.ldx);
    const int cols = static_cast<int>(a.cols);
    // All loads (row, gamma, beta) before the first store: see layernorm_vec_kernel.
    float v[kPerLane], g[kPerLane], b[kPerLane];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < cols ? __ldg(x + c) : 0.0f;
        g[i] = c < cols ? __ldg(a.gamma + c) : 0.0f;
        b[i] = c < cols ? __ldg(a.beta + c) : 0.0f;
        s += v[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    const float mean = s / static_cast<float>(cols);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int c = lane + 32 * i;
        const float d = c < cols ? v[i] - mean : 0.0f;
        q += d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
    const float rstd = rsqrtf(q / static_cast<float>(cols) + a.eps);
    const long long orow = static_cast<long long>(row) * static_cast<long long>(a.ldo);
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int c = lane + 32 * i;
        if (c >= cols) break;
        const float y = (v[i] - mean) * rstd * g[i] + b[i];
        if (a.out_dtype == BL_F32)
            static_cast<float*>(a.out)[orow + c] = y;
        else
            static_cast<uint16_t*>(a.out)[orow + c] = to16(y, a.out_dtype);
    }
}

// The same LayerNorm with 16-byte accesses: lane l holds columns
// [4(l + 32i), 4(l + 32i) + 4) for i < kVec, so each warp load or store of
// a row moves 512 contiguous bytes (f32 in) or 256 bytes (16-bit out). For
// rows whose column count, strides and bases are multiples of 4 elements and
// 16 / 8 bytes; four rows (warps) per 128-thread block.
template <int kVec>
__global__ void __launch_bounds__(128) layernorm_vec_kernel(bl_layernorm_args a, int row_begin,
                                                            int row_end) {
    pdl_trigger();
    pdl_wait();
    const int row = row_begin + static_cast<int>(blockIdx.x) * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= row_end) return;
    long long in_row = row;
    if (a.in_group_rows > 0) in_row += static_cast<long long>(row / a.in_group_rows) * a.in_group_gap;
    in_row += a.in_row_offset;
    const float4* x = reinterpret_cast<const float4*>(a.x + in_row * static_cast<long long>(a.ldx));
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    const float4* b4 = reinterpret_cast<const float4*>(a.beta);
    const int quads = static_cast<int>(a.cols) >> 2;
    // Every load is issued before the first store: the output may alias
    // gamma and beta as far as the compiler knows, so loads left between
    // stores would each wait for the one before.
    float4 v[kVec], g[kVec], b[kVec];
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
        const int q = lane + 32 * i;
        v[i] = q < quads ? __ldg(x + q) : zero;
        g[i] = q < quads ? __ldg(g4 + q) : zero;
        b[i] = q < quads ? __ldg(b4 + q) : zero;
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kVec; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    const float mean = s / static_cast<float>(a.cols);
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
        if (lane + 32 * i < quads) {
            const float d0 = v[i].x - mean, d1 = v[i].y - mean, d2 = v[i].z - mean,
                        d3 = v[i].w - mean;
            sq += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xFFFFFFFFu, sq, o);
    const float rstd = rsqrtf(sq / static_cast<float>(a.cols) + a.eps);
    const long long orow = static_cast<long long>(row) * static_cast<long long>(a.ldo);
#pragma unroll
    for (int i = 0; i < kVec; ++i) {
        const int q = lane + 32 * i;
        if (q >= quads) break;
        float4 y;
        y.x = (v[i].x - mean) * rstd * g[i].x + b[i].x;
        y.y = (v[i].y - mean) * rstd * g[i].y + b[i].y;
        y.z = (v[i].z - mean) * rstd * g[i].z + b[i].z;
        y.w = (v[i].w - mean) * rstd * g[i].w + b[i].w;
        if (a.out_dtype == BL_F32) {
            reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow)[q] = y;
        } else {
            uint2 w;
            w.x = to16(y.x, a.out_dtype) | (static_cast<uint32_t>(to16(y.y, a.out_dtype)) << 16);
            w.y = to16(y.z, a.out_dtype) | (static_cast<uint32_t>(to16(y.w, a.out_dtype)) << 16);
            reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.out) + orow)[q] = w;
        }
    }
}

// Patch matrix: one thread per (patch, 8 consecutive taps). Tap t of a patch
// is (ky, kx, ci) = (t / (p*cin), (t / cin) % p, t % cin), the HWIO order of
// the reference's patch weights, so row . weight[cout][t] is its patch_embed.
// Index arithmetic in 32 bits (the host checks that every index fits): the
// divisions happen once per thread, and the 8 taps step (ky, kx, ci) by
// increments, since run-time integer divisions dominated the kernel.
// Blocks past `patch_blocks` (one per frame, when a.x is set) write the
// frame's class-token row: x[f][0][c] = cls[c] + pos[0][c] (an f32 add, as a
// fused epilogue Add would do), so the rows need no launch of their own.
__global__ void patchify_kernel(bl_patchify_args a, int grid_side, int taps,
                                unsigned patch_blocks) {
    pdl_trigger();
    pdl_wait();
    if (blockIdx.x >= patch_blocks) {
        const long long f = blockIdx.x - patch_blocks;
        const long long tokens = static_cast<long long>(grid_side) * grid_side + 1;
        for (int c = threadIdx.x; c < static_cast<int>(a.dim); c += blockDim.x)
            a.x[f * tokens * a.dim + c] = a.cls[c] + a.pos[c];
        return;
    }
    const unsigned idx = blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned groups = a.k_pad / 8;
    const unsigned per_frame = static_cast<unsigned>(grid_side * grid_side);
    if (idx >= a.frames * per_frame * groups) return;
    const unsigned patch = idx / groups;
    const int g = static_cast<int>(idx - patch * groups);
    const unsigned f = patch / per_frame;
    const int pp = static_cast<int>(patch - f * per_frame);
    const int gy = pp / grid_side, gx = pp - (pp / grid_side) * grid_side;
    const int P = static_cast<int>(a.patch), C = static_cast<int>(a.cin);
    const int side = static_cast<int>(a.side);
    const float* img = a.image + static_cast<size_t>(f) * side * side * C;
    int t = g * 8;
    int ky = t / (P * C);
    int kx = (t - ky * P * C) / C;
    int ci = t - ky * P * C - kx * C;
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j, ++t) {
        float v = 0.0f;
        if (t < taps) v = img[((gy * P + ky) * side + gx * P + kx) * C + ci];
        h[j] = to16(v, a.a_dtype);
        if (++ci == C) {
            ci = 0;
            if (++kx == P) kx = 0, ++ky;
        }
    }
    uint4 w;
    w.x = h[0] | (static_cast<uint32_t>(h[1]) << 16);
    w.y = h[2] | (static_cast<uint32_t>(h[3]) << 16);
    w.z = h[4] | (static_cast<uint32_t>(h[5]) << 16);
    w.w = h[6] | (static_cast<uint32_t>(h[7]) << 16);
    reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.a) + patch * a.k_pad)[g] = w;
}

}  // namespace misc
}  // namespace bl

namespace bl {

int prepare_layernorm_rows(const bl_layernorm_args& a, uint32_t row_begin, uint32_t row_end,
                           Launch* out) {
    if (a.rows == 0 || a.cols == 0 || a.x == nullptr || a.out == nullptr || a.gamma == nullptr ||
        a.beta == nullptr)
        return fail(BL_ERR_INVALID, "layernorm: empty shape or null pointer");
    if (!(a.eps > 0.0f)) return fail(BL_ERR_INVALID, "layernorm: epsilon must be positive");
    if (a.cols > 1024) return fail(BL_ERR_UNSUPPORTED, "layernorm: %u columns (max 1024)", a.cols);
    if (a.out_dtype != BL_F32 && a.out_dtype != BL_F16 && a.out_dtype != BL_BF16)
        return fail(BL_ERR_INVALID, "layernorm: output dtype %d", a.out_dtype);
    bl_layernorm_args b = a;
    if (b.ldx == 0) b.ldx = b.cols;
    if (b.ldo == 0) b.ldo = b.cols;
    if (row_begin >= row_end || row_end > a.rows)
        return fail(BL_ERR_INVALID, "layernorm: row part [%u, %u) outside [0, %u)", row_begin, row_end, a.rows);
    const int r0 = static_cast<int>(row_begin), r1 = static_cast<int>(row_end);
    auto aligned = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; };
    const bool vec = b.cols % 4 == 0 && b.ldx % 4 == 0 && b.ldo % 4 == 0 && aligned(b.x, 16) &&
                     aligned(b.gamma, 16) && aligned(b.beta, 16) &&
                     aligned(b.out, b.out_dtype == BL_F32 ? 16 : 8);
    out->op = 3;
    if (vec) {
        const int kvec = static_cast<int>((b.cols + 127) / 128);
        void (*kern)(bl_layernorm_args, int, int) = kvec <= 1   ? misc::layernorm_vec_kernel<1>
                                                  : kvec <= 2 ? misc::layernorm_vec_kernel<2>
                                                  : kvec <= 3 ? misc::layernorm_vec_kernel<3>
                                                  : kvec <= 4 ? misc::layernorm_vec_kernel<4>
                                                  : kvec <= 6 ? misc::layernorm_vec_kernel<6>
                                                              : misc::layernorm_vec_kernel<8>;
        const dim3 grid((row_end - row_begin + 3) / 4);
        out->run = [=](cudaStream_t s) { return launch_k(kern, grid, dim3(128), 0, s, b, r0, r1); };
        return BL_OK;
    }
    const dim3 grid((row_end - row_begin + 7) / 8);
    void (*kern)(bl_layernorm_args, int, int) = a.cols <= 128   ? misc::layernorm_kernel<4>
                                      : a.cols <= 384 ? misc::layernorm_kernel<12>
                                      : a.cols <= 512 ? misc::layernorm_kernel<16>
                                                      : misc::layernorm_kernel<32>;
    out->run = [=](cudaStream_t s) {
        return launch_k(kern, grid, dim3(256), 0, s, b, r0, r1);
    };
    return BL_OK;
}

int prepare_layernorm(const bl_layernorm_args& a, Launch* out) {
    return prepare_layernorm_rows(a, 0, a.rows, out);
}

int prepare_patchify(const bl_patchify_args& a, Launch* out) {
    if (a.frames == 0 || a.patch == 0 || a.cin == 0 || a.side == 0 || a.side % a.patch != 0)
        return fail(BL_ERR_INVALID, "patchify: side %u is not whole patches of %u", a.side, a.patch);
    const uint32_t taps = a.patch * a.patch * a.cin;
    if (a.k_pad < taps || a.k_pad % 64 != 0)
        return fail(BL_ERR_INVALID, "patchify: k_pad %u must cover %u taps and be a multiple of 64",
                    a.k_pad, taps);
    if (a.image == nullptr || a.a == nullptr || (reinterpret_cast<uintptr_t>(a.a) & 15))
        return fail(BL_ERR_INVALID, "patchify: null or misaligned buffers");
    if (a.a_dtype != BL_F16 && a.a_dtype != BL_BF16)
        return fail(BL_ERR_INVALID, "patchify: A dtype %d", a.a_dtype);
    if (a.x != nullptr && (a.cls == nullptr || a.pos == nullptr || a.dim == 0))
        return fail(BL_ERR_INVALID, "patchify: class-token rows need cls, pos and dim");
    const int g = static_cast<int>(a.side / a.patch);
    const long long work = static_cast<long long>(a.frames) * g * g * (a.k_pad / 8);
    if (work >= (1ll << 31) || 1ll * a.side * a.side * a.cin >= (1ll << 31))
        return fail(BL_ERR_UNSUPPORTED, "patchify: %u frames of %u px exceed 32-bit indexing",
                    a.frames, a.side);
    const unsigned blocks = static_cast<unsigned>((work + 255) / 256);
    out->op = 4;
    out->run = [=](cudaStream_t s) {
        // the patch matrix, and one block per frame for its class-token row
        return launch_k(misc::patchify_kernel, dim3(blocks + (a.x != nullptr ? a.frames : 0)),
                        dim3(256), 0, s, a, g, static_cast<int>(taps), blocks);
    };
    return BL_OK;
}

}  // namespace bl

extern "C" int bl_layernorm(const bl_layernorm_args* args, void* stream) {
    if (args == nullptr) return bl::fail(BL_ERR_INVALID, "layernorm: null args");
    bl::Launch l;
    int rc = bl::prepare_layernorm(*args, &l);
    return rc != BL_OK ? rc : bl::enqueue(l, static_cast<cudaStream_t>(stream));
}

extern "C" int bl_patchify(const bl_patchify_args* args, void* stream) {
    if (args == nullptr) return bl::fail(BL_ERR_INVALID, "patchify: null args");
    bl::Launch l;
    int rc = bl::prepare_patchify(*args, &l);
    return rc != BL_OK ? rc : bl::enqueue(l, static_cast<cudaStream_t>(stream));
}
