// The DPT decoder's data-movement kernels; its convolutions run on the
// tcgen05 GEMM (csrc/gemm.cu). A 3x3 (or 1x1) convolution is an im2col
// gather of NHWC f32 pixels into 16-bit rows of K = taps x cin (zero padding
// at the image border, an optional ReLU on the way in: the residual units'
// pre-activation, the reference's ReLU prologue, crates/beatlm-core/src/
// kernel.rs:265-319) followed by one GEMM with the HWIO weights as [cout][K].
// A transposed convolution of kernel = stride = f is one GEMM per pixel into
// [pixels][f*f*cout] and a scatter of each pixel's f x f block. The bilinear
// resampling (corners aligned) is its own kernel. All HBM-bound byte moves:
// coalesced 16-byte stores, grid-stride loops over a multiple of the SMs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "host.h"

namespace bl {
namespace gemm {
int sm_count();  // csrc/gemm.cu
}
namespace dec {

template <typename T>
__device__ __forceinline__ uint16_t to16(float v);
template <>
__device__ __forceinline__ uint16_t to16<__half>(float v) {
    return __half_as_ushort(__float2half_rn(v));
}
template <>
__device__ __forceinline__ uint16_t to16<__nv_bfloat16>(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// One thread writes 8 consecutive columns (16 bytes) of one output row:
// column k = (ky * ks + kx) * cin + ci, zero past ks * ks * cin.
template <typename T>
__global__ void im2col_kernel(const float* __restrict__ in, uint4* __restrict__ out, int h,
                              int w, int cin, int ks, int stride, int relu, int oh, int ow,
                              int k_pad) {
    const int vecs = k_pad / 8;
    const long long total = static_cast<long long>(oh) * ow * vecs;
    const int taps = ks * cin * ks;
    const int pad = ks / 2;
    for (long long v = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < total;
         v += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long pix = v / vecs;
        const int k0 = static_cast<int>(v % vecs) * 8;
        const int y = static_cast<int>(pix / ow), x = static_cast<int>(pix % ow);
        uint16_t r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k = k0 + j;
            float val = 0.0f;
            if (k < taps) {
                const int tap = k / cin, ci = k - tap * cin;
                const int iy = y * stride + tap / ks - pad, ix = x * stride + tap % ks - pad;
                if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
                    val = __ldg(in + (static_cast<long long>(iy) * w + ix) * cin + ci);
                    if (relu) val = fmaxf(val, 0.0f);
                }
            }
            r[j] = to16<T>(val);
        }
        out[v] = make_uint4(r[0] | (uint32_t(r[1]) << 16), r[2] | (uint32_t(r[3]) << 16),
                            r[4] | (uint32_t(r[5]) << 16), r[6] | (uint32_t(r[7]) << 16));
    }
}

// out[(y f + ky) * (w f) + x f + kx][co] = blocks[y * w + x][(ky f + kx) cout + co] + bias[co]
__global__ void blocks_to_map_kernel(const float* __restrict__ blocks, const float* __restrict__ bias,
                                     float* __restrict__ out, int h, int w, int f, int cout) {
    const long long total = static_cast<long long>(h) * f * w * f * cout;
    const int ow = w * f;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int co = static_cast<int>(i % cout);
        const long long opix = i / cout;
        const int oy = static_cast<int>(opix / ow), ox = static_cast<int>(opix % ow);
        const int y = oy / f, ky = oy % f, x = ox / f, kx = ox % f;
        float v = __ldg(blocks + (static_cast<long long>(y) * w + x) * (f * f * cout) +
                        (ky * f + kx) * cout + co);
        if (bias) v += __ldg(bias + co);
        out[i] = v;
    }
}

// cout a multiple of 4 (every DPT width) and every index below 2^31: a thread
// moves 4 consecutive channels of one output pixel with 16-byte loads and
// stores and 32-bit index arithmetic (the 64-bit per-element divisions of the
// kernel above bound it, not its memory traffic).
__global__ void blocks_to_map_vec4_kernel(const float4* __restrict__ blocks,
                                          const float4* __restrict__ bias, float4* __restrict__ out,
                                          int w, int f, int c4, unsigned total) {
    const int ow = w * f;
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const unsigned p = i / static_cast<unsigned>(c4);
        const int ch = static_cast<int>(i - p * static_cast<unsigned>(c4));
        const int oy = static_cast<int>(p / static_cast<unsigned>(ow));
        const int ox = static_cast<int>(p - static_cast<unsigned>(oy) * static_cast<unsigned>(ow));
        const int y = oy / f, ky = oy - y * f, x = ox / f, kx = ox - x * f;
        float4 v = __ldg(blocks + ((y * w + x) * f * f + ky * f + kx) * c4 + ch);
        if (bias != nullptr) {
            const float4 b = __ldg(bias + ch);
            v.x += b.x, v.y += b.y, v.z += b.z, v.w += b.w;
        }
        out[i] = v;
    }
}

// Corners aligned: output row oy reads position oy (ih-1)/(oh-1) (0 for one
// row) between its floor and the next row, clamped; columns likewise.
__device__ __forceinline__ void axis(int o, int in, int outn, int* i0, int* i1, float* l) {
    const float pos = outn > 1 ? static_cast<float>(o) * static_cast<float>(in - 1) /
                                     static_cast<float>(outn - 1)
                               : 0.0f;
    int a = static_cast<int>(floorf(pos));
    a = a > in - 1 ? in - 1 : a;
    *i0 = a;
    *i1 = a + 1 < in ? a + 1 : in - 1;
    *l = pos - static_cast<float>(a);
}

// The four corners mixed along x, then y, each product and sum rounded as
// written (no contraction left to the compiler), so every resampling kernel
// below gives the same f32 bits for the same pixel.
__device__ __forceinline__ float bilerp(float v00, float v01, float v10, float v11, float lx,
                                        float ly) {
    const float top = __fadd_rn(__fmul_rn(1.0f - lx, v00), __fmul_rn(lx, v01));
    const float bottom = __fadd_rn(__fmul_rn(1.0f - lx, v10), __fmul_rn(lx, v11));
    return __fadd_rn(__fmul_rn(1.0f - ly, top), __fmul_rn(ly, bottom));
}

__global__ void resize_bilinear_kernel(const float* __restrict__ in, float* __restrict__ out, int ih,
                                       int iw, int oh, int ow, int c) {
    const long long total = static_cast<long long>(oh) * ow * c;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int ch = static_cast<int>(i % c);
        const long long p = i / c;
        const int oy = static_cast<int>(p / ow), ox = static_cast<int>(p % ow);
        int y0, y1, x0, x1;
        float ly, lx;
        axis(oy, ih, oh, &y0, &y1, &ly);
        axis(ox, iw, ow, &x0, &x1, &lx);
        const float a00 = __ldg(in + (static_cast<long long>(y0) * iw + x0) * c + ch);
        const float a01 = __ldg(in + (static_cast<long long>(y0) * iw + x1) * c + ch);
        const float a10 = __ldg(in + (static_cast<long long>(y1) * iw + x0) * c + ch);
        const float a11 = __ldg(in + (static_cast<long long>(y1) * iw + x1) * c + ch);
        out[i] = bilerp(a00, a01, a10, a11, lx, ly);
    }
}

// c a multiple of 4 (every DPT width) and every index below 2^31: a thread
// resamples 4 consecutive channels of one output pixel with 16-byte loads
// and stores and 32-bit index arithmetic (one set of weights per 4 values).
__global__ void resize_bilinear_vec4_kernel(const float4* __restrict__ in, float4* __restrict__ out,
                                            int ih, int iw, int oh, int ow, int c4) {
    const unsigned total = static_cast<unsigned>(oh) * static_cast<unsigned>(ow) * static_cast<unsigned>(c4);
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const unsigned p = i / static_cast<unsigned>(c4);
        const int ch = static_cast<int>(i - p * static_cast<unsigned>(c4));
        const int oy = static_cast<int>(p / static_cast<unsigned>(ow));
        const int ox = static_cast<int>(p - static_cast<unsigned>(oy) * static_cast<unsigned>(ow));
        int y0, y1, x0, x1;
        float ly, lx;
        axis(oy, ih, oh, &y0, &y1, &ly);
        axis(ox, iw, ow, &x0, &x1, &lx);
        const float4 a00 = __ldg(in + (y0 * iw + x0) * c4 + ch), a01 = __ldg(in + (y0 * iw + x1) * c4 + ch);
        const float4 a10 = __ldg(in + (y1 * iw + x0) * c4 + ch), a11 = __ldg(in + (y1 * iw + x1) * c4 + ch);
        out[i] = make_float4(bilerp(a00.x, a01.x, a10.x, a11.x, lx, ly),
                             bilerp(a00.y, a01.y, a10.y, a11.y, lx, ly),
                             bilerp(a00.z, a01.z, a10.z, a11.z, lx, ly),
                             bilerp(a00.w, a01.w, a10.w, a11.w, lx, ly));
    }
}

// The same resampling written as 16-bit rows of ld8 * 8 values, the A operand
// of a 1x1 convolution's GEMM (what a gather of the f32 map would store, with
// no f32 map in between): a thread makes 8 consecutive channels of one output
// pixel from two float4 loads at each corner and stores them as one 16-byte
// vector; vectors past the c4 * 4 channels are zeros. c4 even; 32-bit index
// arithmetic (the host launches it only when every index fits).
template <typename T>
__global__ void resize_bilinear_rows16_kernel(const float4* __restrict__ in, uint4* __restrict__ out,
                                              int ih, int iw, int oh, int ow, int c4, int ld8) {
    const unsigned total = static_cast<unsigned>(oh) * static_cast<unsigned>(ow) * static_cast<unsigned>(ld8);
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const unsigned p = i / static_cast<unsigned>(ld8);
        const int v = static_cast<int>(i - p * static_cast<unsigned>(ld8));
        uint4 r = make_uint4(0u, 0u, 0u, 0u);
        if (2 * v < c4) {
            const int oy = static_cast<int>(p / static_cast<unsigned>(ow));
            const int ox = static_cast<int>(p - static_cast<unsigned>(oy) * static_cast<unsigned>(ow));
            int y0, y1, x0, x1;
            float ly, lx;
            axis(oy, ih, oh, &y0, &y1, &ly);
            axis(ox, iw, ow, &x0, &x1, &lx);
            const float4* c00 = in + (y0 * iw + x0) * c4 + 2 * v;
            const float4* c01 = in + (y0 * iw + x1) * c4 + 2 * v;
            const float4* c10 = in + (y1 * iw + x0) * c4 + 2 * v;
            const float4* c11 = in + (y1 * iw + x1) * c4 + 2 * v;
            float f[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float4 a00 = __ldg(c00 + h), a01 = __ldg(c01 + h);
                const float4 a10 = __ldg(c10 + h), a11 = __ldg(c11 + h);
                f[4 * h + 0] = bilerp(a00.x, a01.x, a10.x, a11.x, lx, ly);
                f[4 * h + 1] = bilerp(a00.y, a01.y, a10.y, a11.y, lx, ly);
                f[4 * h + 2] = bilerp(a00.z, a01.z, a10.z, a11.z, lx, ly);
                f[4 * h + 3] = bilerp(a00.w, a01.w, a10.w, a11.w, lx, ly);
            }
            r = make_uint4(to16<T>(f[0]) | (uint32_t(to16<T>(f[1])) << 16),
                           to16<T>(f[2]) | (uint32_t(to16<T>(f[3])) << 16),
                           to16<T>(f[4]) | (uint32_t(to16<T>(f[5])) << 16),
                           to16<T>(f[6]) | (uint32_t(to16<T>(f[7])) << 16));
        }
        out[i] = r;
    }
}

// cin a multiple of 8 (every DPT width): a thread's 8 columns are 8
// consecutive channels of one tap, read as two 16-byte loads. No division in
// the loop: each block first tabulates, per 8-column vector j of an output
// row, its tap (ky, kx) and first channel (or -1 past the taps) in shared
// memory (k_pad / 8 words), and each thread steps its (pixel, vector) pair
// and the pixel's (y, x) by the grid stride with carries. Consecutive
// threads still write consecutive 16-byte vectors.
// Index arithmetic in 32 bits (the host launches it only when every index
// fits). kIn16: the map is already 16-bit of the output's type, and each
// vector is one 16-byte load copied as it is (ReLU clears the values whose
// sign bit is set: the bits the f32 path stores for the same rounded map).
template <typename T, bool kIn16>
__global__ void im2col_vec8_kernel(const void* __restrict__ in_, uint4* __restrict__ out, int h,
                                   int w, int cin, int ks, int stride, int relu, int oh, int ow,
                                   int k_pad) {
    extern __shared__ int vec_tap[];
    const unsigned vecs = static_cast<unsigned>(k_pad) / 8u;
    const unsigned total = static_cast<unsigned>(oh) * static_cast<unsigned>(ow) * vecs;
    const int taps = ks * ks * cin;
    const int pad = ks / 2;
    for (unsigned j = threadIdx.x; j < vecs; j += blockDim.x) {
        const int k0 = static_cast<int>(j) * 8;
        int e = -1;
        if (k0 < taps) {
            const int tap = k0 / cin, ci = k0 - tap * cin;
            const int ky = tap / ks, kx = tap - ky * ks;
            e = (ky << 28) | (kx << 24) | ci;
        }
        vec_tap[j] = e;
    }
    __syncthreads();
    const unsigned step = gridDim.x * blockDim.x;
    const unsigned step_p = step / vecs, step_j = step - step_p * vecs;
    const unsigned step_y = step_p / static_cast<unsigned>(ow);
    const unsigned step_x = step_p - step_y * static_cast<unsigned>(ow);
    unsigned v = blockIdx.x * blockDim.x + threadIdx.x;
    unsigned pix = v / vecs, j = v - pix * vecs;
    unsigned y = pix / static_cast<unsigned>(ow), x = pix - y * static_cast<unsigned>(ow);
    for (; v < total; v += step) {
        uint4 r = make_uint4(0u, 0u, 0u, 0u);  // the zero border and the padded columns
        const int e = vec_tap[j];
        if (e >= 0) {
            const int ky = e >> 28, kx = (e >> 24) & 15, ci = e & 0xFFFFFF;
            const int iy = static_cast<int>(y) * stride + ky - pad;
            const int ix = static_cast<int>(x) * stride + kx - pad;
            if (iy >= 0 && iy < h && ix >= 0 && ix < w) {
                const long long off = (static_cast<long long>(iy) * w + ix) * cin + ci;
                if constexpr (kIn16) {
                    r = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(in_) + off));
                    if (relu) {
                        // a 0xFFFF mask on each 16-bit half whose sign bit is set
                        auto clear = [](uint32_t u) { return u & ~(((u >> 15) & 0x00010001u) * 0xFFFFu); };
                        r = make_uint4(clear(r.x), clear(r.y), clear(r.z), clear(r.w));
                    }
                } else {
                    const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(in_) + off);
                    float4 lo = __ldg(src), hi = __ldg(src + 1);
                    if (relu) {
                        lo = make_float4(fmaxf(lo.x, 0.f), fmaxf(lo.y, 0.f), fmaxf(lo.z, 0.f), fmaxf(lo.w, 0.f));
                        hi = make_float4(fmaxf(hi.x, 0.f), fmaxf(hi.y, 0.f), fmaxf(hi.z, 0.f), fmaxf(hi.w, 0.f));
                    }
                    r = make_uint4(to16<T>(lo.x) | (uint32_t(to16<T>(lo.y)) << 16),
                                   to16<T>(lo.z) | (uint32_t(to16<T>(lo.w)) << 16),
                                   to16<T>(hi.x) | (uint32_t(to16<T>(hi.y)) << 16),
                                   to16<T>(hi.z) | (uint32_t(to16<T>(hi.w)) << 16));
                }
            }
        }
        out[v] = r;
        // the next (pixel, vector) and the pixel's (y, x), with carries
        j += step_j;
        unsigned carry = 0;
        if (j >= vecs) {
            j -= vecs;
            carry = 1;
        }
        x += step_x + carry;
        y += step_y;
        if (x >= static_cast<unsigned>(ow)) {
            x -= static_cast<unsigned>(ow);
            y += 1;
        }
    }
}

// One output channel of a 1x1 convolution over NHWC f32 rows of 4 * c4
// values: out[p] = act(sum_i in[p][i] w[i] + b). A warp step covers 16
// pixels as four 4-pixel loads (lane l: pixel 4 k + l / 8, float4 l % 8 of
// each 32 channels, so a load is 512 contiguous bytes at 32 channels); each
// lane sums its float4s in channel order, an xor-shuffle tree within the
// pixel's 8 lanes completes the sum (the same bits whichever lane reads it),
// and the group's first lane stores the pixel.
__global__ void conv1x1_one_kernel(const float4* __restrict__ in, const float4* __restrict__ w,
                                   float b, float* __restrict__ out, unsigned pixels, int c4,
                                   int relu) {
    const int lane = threadIdx.x & 31, sub = lane & 7, grp = lane >> 3;
    const unsigned warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned warps = (gridDim.x * blockDim.x) >> 5;
    for (unsigned p0 = warp * 16u; p0 < pixels; p0 += warps * 16u) {  // warp-uniform
        float acc[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const unsigned p = p0 + 4u * k + grp;
            acc[k] = 0.0f;
            if (p < pixels) {
                const float4* row = in + static_cast<size_t>(p) * c4;
                for (int i = sub; i < c4; i += 8) {
                    const float4 v = __ldg(row + i), q = __ldg(w + i);
                    acc[k] = fmaf(v.x, q.x, acc[k]);
                    acc[k] = fmaf(v.y, q.y, acc[k]);
                    acc[k] = fmaf(v.z, q.z, acc[k]);
                    acc[k] = fmaf(v.w, q.w, acc[k]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float a = acc[k];
            a += __shfl_xor_sync(0xFFFFFFFFu, a, 1);
            a += __shfl_xor_sync(0xFFFFFFFFu, a, 2);
            a += __shfl_xor_sync(0xFFFFFFFFu, a, 4);
            const unsigned p = p0 + 4u * k + grp;
            if (sub == 0 && p < pixels) {
                const float y = a + b;
                out[p] = relu ? fmaxf(y, 0.0f) : y;
            }
        }
    }
}

// blocks of 256 threads, up to 8 per SM, never more than the work needs
unsigned grid_for(long long work) {
    const long long blocks = (work + 255) / 256;
    const long long cap = 8ll * gemm::sm_count();
    return static_cast<unsigned>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

}  // namespace dec
}  // namespace bl

extern "C" {

int bl_im2col(const bl_im2col_args* a, void* stream) {
    using namespace bl;
    if (a == nullptr || a->input == nullptr || a->out == nullptr)
        return fail(BL_ERR_INVALID, "im2col: null argument");
    if (a->ksize != 1 && a->ksize != 3) return fail(BL_ERR_UNSUPPORTED, "im2col: kernel %u (1 or 3)", a->ksize);
    if (a->stride < 1 || a->h == 0 || a->w == 0 || a->cin == 0)
        return fail(BL_ERR_INVALID, "im2col: zero dimension or stride");
    const uint64_t taps = 1ull * a->ksize * a->ksize * a->cin;
    if (a->k_pad % 64 != 0 || a->k_pad < taps)
        return fail(BL_ERR_INVALID, "im2col: k_pad %u must be a multiple of 64 and at least %llu",
                    a->k_pad, (unsigned long long)taps);
    if (a->out_dtype != BL_F16 && a->out_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "im2col: out dtype %d (f16 or bf16)", a->out_dtype);
    if (reinterpret_cast<uintptr_t>(a->out) & 15u) return fail(BL_ERR_INVALID, "im2col: out must be 16-byte aligned");
    const bool in16 = a->in_dtype != BL_F32;
    if (in16 && a->in_dtype != a->out_dtype)
        return fail(BL_ERR_UNSUPPORTED, "im2col: in dtype %d (f32 or the out dtype %d)", a->in_dtype,
                    a->out_dtype);
    const int pad = static_cast<int>(a->ksize / 2);
    const int oh = static_cast<int>((a->h + 2 * pad - a->ksize) / a->stride + 1);
    const int ow = static_cast<int>((a->w + 2 * pad - a->ksize) / a->stride + 1);
    const long long work = 1ll * oh * ow * (a->k_pad / 8);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // the vector path indexes in 32 bits: outputs and inputs below 2^31 elements
    // (and its tap table, k_pad / 8 words, fits the default 48 KiB of shared memory)
    const bool vec = a->cin % 8 == 0 && (reinterpret_cast<uintptr_t>(a->input) & 15u) == 0 &&
                     a->k_pad / 8 * sizeof(int) <= 48u * 1024u &&
                     work < (1ll << 31) - 2ll * 256 * 8 * 148 &&
                     1ll * a->h * a->w * a->cin < (1ll << 31);
    if (in16 && !vec)
        return fail(BL_ERR_UNSUPPORTED,
                    "im2col: a 16-bit map needs cin a multiple of 8, a 16-byte aligned input and "
                    "32-bit indices");
    // the vector path's tap table: one word per 8 columns of an output row
    const size_t table = vec ? sizeof(int) * (a->k_pad / 8) : 0;
    const unsigned grid = dec::grid_for(work);
    const int relu = a->relu ? 1 : 0;
    uint4* out = static_cast<uint4*>(a->out);
    if (!vec) {
        auto kern = a->out_dtype == BL_F16 ? dec::im2col_kernel<__half>
                                           : dec::im2col_kernel<__nv_bfloat16>;
        kern<<<grid, 256, 0, s>>>(static_cast<const float*>(a->input), out, a->h, a->w, a->cin,
                                  a->ksize, a->stride, relu, oh, ow, a->k_pad);
    } else {
        auto kern = a->out_dtype == BL_F16
                        ? (in16 ? dec::im2col_vec8_kernel<__half, true>
                                : dec::im2col_vec8_kernel<__half, false>)
                        : (in16 ? dec::im2col_vec8_kernel<__nv_bfloat16, true>
                                : dec::im2col_vec8_kernel<__nv_bfloat16, false>);
        kern<<<grid, 256, table, s>>>(a->input, out, a->h, a->w, a->cin, a->ksize, a->stride,
                                      relu, oh, ow, a->k_pad);
    }
    BL_CUDA_TRY(cudaGetLastError());
    return BL_OK;
}

int bl_blocks_to_map(const float* blocks, const float* bias, float* out, uint32_t h, uint32_t w,
                     uint32_t f, uint32_t cout, void* stream) {
    using namespace bl;
    if (blocks == nullptr || out == nullptr) return fail(BL_ERR_INVALID, "blocks_to_map: null argument");
    if (h == 0 || w == 0 || f == 0 || cout == 0) return fail(BL_ERR_INVALID, "blocks_to_map: zero dimension");
    const long long work = 1ll * h * f * w * f * cout;
    const bool vec = cout % 4 == 0 &&
                     ((reinterpret_cast<uintptr_t>(blocks) | reinterpret_cast<uintptr_t>(bias) |
                       reinterpret_cast<uintptr_t>(out)) & 15u) == 0 &&
                     work < (1ll << 31) - 2ll * 256 * 8 * 148;
    if (vec)
        dec::blocks_to_map_vec4_kernel<<<dec::grid_for(work / 4), 256, 0,
                                         static_cast<cudaStream_t>(stream)>>>(
            reinterpret_cast<const float4*>(blocks), reinterpret_cast<const float4*>(bias),
            reinterpret_cast<float4*>(out), static_cast<int>(w), static_cast<int>(f),
            static_cast<int>(cout / 4), static_cast<unsigned>(work / 4));
    else
        dec::blocks_to_map_kernel<<<dec::grid_for(work), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            blocks, bias, out, h, w, f, cout);
    BL_CUDA_TRY(cudaGetLastError());
    return BL_OK;
}

int bl_conv1x1_one(const float* in, const float* w, float bias, float* out, uint32_t pixels,
                   uint32_t c, int32_t relu, void* stream) {
    using namespace bl;
    if (in == nullptr || w == nullptr || out == nullptr)
        return fail(BL_ERR_INVALID, "conv1x1_one: null argument");
    if (pixels == 0 || c == 0) return fail(BL_ERR_INVALID, "conv1x1_one: zero dimension");
    if (c % 4 != 0 || c > 1024)
        return fail(BL_ERR_UNSUPPORTED, "conv1x1_one: %u channels (a multiple of 4, at most 1024)", c);
    if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(w)) & 15u) ||
        (reinterpret_cast<uintptr_t>(out) & 3u))
        return fail(BL_ERR_INVALID, "conv1x1_one: in and w must be 16-byte aligned, out 4-byte");
    if (1ull * pixels + 16ull * 8 * 256 * 8 * 148 >= (1ull << 32))
        return fail(BL_ERR_UNSUPPORTED, "conv1x1_one: %u pixels exceed 32-bit indexing", pixels);
    // one warp step per 16 pixels, 8 warps a block
    const long long steps = (static_cast<long long>(pixels) + 15) / 16;
    const unsigned blocks = dec::grid_for(steps * 32);
    dec::conv1x1_one_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const float4*>(in), reinterpret_cast<const float4*>(w), bias, out, pixels,
        static_cast<int>(c / 4), relu ? 1 : 0);
    BL_CUDA_TRY(cudaGetLastError());
    return BL_OK;
}

int bl_resize_bilinear(const float* in, float* out, uint32_t ih, uint32_t iw, uint32_t oh,
                       uint32_t ow, uint32_t c, void* stream) {
    using namespace bl;
    if (in == nullptr || out == nullptr) return fail(BL_ERR_INVALID, "resize: null argument");
    if (ih == 0 || iw == 0 || oh == 0 || ow == 0 || c == 0)
        return fail(BL_ERR_INVALID, "resize: zero dimension");
    const long long work = 1ll * oh * ow * c;
    const bool vec = c % 4 == 0 && ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0 &&
                     work < (1ll << 31) - 2ll * 256 * 8 * 148 && 1ll * ih * iw * c < (1ll << 31);
    if (vec)
        dec::resize_bilinear_vec4_kernel<<<dec::grid_for(work / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            reinterpret_cast<const float4*>(in), reinterpret_cast<float4*>(out), ih, iw, oh, ow, c / 4);
    else
        dec::resize_bilinear_kernel<<<dec::grid_for(work), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            in, out, ih, iw, oh, ow, c);
    BL_CUDA_TRY(cudaGetLastError());
    return BL_OK;
}

int bl_resize_bilinear_rows16(const float* in, void* out, uint32_t ih, uint32_t iw, uint32_t oh,
                              uint32_t ow, uint32_t c, uint32_t ld, int32_t out_dtype,
                              void* stream) {
    using namespace bl;
    if (in == nullptr || out == nullptr) return fail(BL_ERR_INVALID, "resize rows16: null argument");
    if (ih == 0 || iw == 0 || oh == 0 || ow == 0 || c == 0)
        return fail(BL_ERR_INVALID, "resize rows16: zero dimension");
    if (c % 8 != 0 || ld % 8 != 0 || ld < c)
        return fail(BL_ERR_UNSUPPORTED,
                    "resize rows16: %u channels into rows of %u (both multiples of 8, rows >= channels)",
                    c, ld);
    if (out_dtype != BL_F16 && out_dtype != BL_BF16)
        return fail(BL_ERR_UNSUPPORTED, "resize rows16: out dtype %d (f16 or bf16)", out_dtype);
    if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) != 0)
        return fail(BL_ERR_INVALID, "resize rows16: in and out must be 16-byte aligned");
    const long long work = 1ll * oh * ow * (ld / 8);
    if (work >= (1ll << 31) - 2ll * 256 * 8 * 148 || 1ll * ih * iw * c >= (1ll << 31))
        return fail(BL_ERR_UNSUPPORTED, "resize rows16: sizes exceed 32-bit indexing");
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned grid = dec::grid_for(work);
    if (out_dtype == BL_F16)
        dec::resize_bilinear_rows16_kernel<__half><<<grid, 256, 0, st>>>(
            reinterpret_cast<const float4*>(in), static_cast<uint4*>(out), ih, iw, oh, ow, c / 4, ld / 8);
    else
        dec::resize_bilinear_rows16_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
            reinterpret_cast<const float4*>(in), static_cast<uint4*>(out), ih, iw, oh, ow, c / 4, ld / 8);
    BL_CUDA_TRY(cudaGetLastError());
    return BL_OK;
}

}  // extern "C"
