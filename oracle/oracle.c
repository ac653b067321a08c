/*
 * CPU oracle for the ViT attention hot path: TEST INFRASTRUCTURE ONLY (see
 * oracle.h). Each function states the reference function it restates, by file
 * and line within ynishi/beatlm. Built with -ffp-contract=off so no multiply
 * and add are fused: the reference (Rust) never contracts them either.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- data */

/* crates/beatlm-bench/src/net.rs:183-195: state = state * 6364136223846793005
 * + 1442695040888963407 (wrapping); the top 24 bits over 2^24 give [0, 1). */
static float lcg_next(uint64_t* state) {
    *state = *state * 6364136223846793005ULL + 1442695040888963407ULL;
    return (float)(*state >> 40) / (float)(1u << 24);
}

/* net.rs:198-203: low + (high - low) * next, in f32. */
void orc_uniform(uint64_t seed, size_t count, float low, float high, float* out) {
    uint64_t s = seed;
    const float span = high - low;
    for (size_t i = 0; i < count; ++i) {
        float r = lcg_next(&s);
        float scaled = span * r;
        out[i] = low + scaled;
    }
}

void orc_normal(uint64_t seed, size_t count, float mean, float std, float* out) {
    uint64_t s = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < count; i += 2) {
        double u1 = (double)lcg_next(&s);
        double u2 = (double)lcg_next(&s);
        double r = sqrt(-2.0 * log(1.0 - u1));
        double z0 = r * cos(two_pi * u2);
        double z1 = r * sin(two_pi * u2);
        out[i] = (float)((double)mean + (double)std * z0);
        if (i + 1 < count) out[i + 1] = (float)((double)mean + (double)std * z1);
    }
}

/* ---------------------------------------------------------------- ops */

/* reference.rs:247-270: biased variance, f64 throughout, f32 result. */
void orc_layernorm(const float* x, const float* gamma, const float* beta, size_t rows,
                   size_t c, float eps, int threads, float* out) {
    long long n = (long long)rows;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long p = 0; p < n; ++p) {
        const float* row = x + (size_t)p * c;
        double sum = 0.0;
        for (size_t i = 0; i < c; ++i) sum += (double)row[i];
        double mean = sum / (double)c;
        double var = 0.0;
        for (size_t i = 0; i < c; ++i) {
            double dv = (double)row[i] - mean;
            var += dv * dv;
        }
        var /= (double)c;
        double inv = 1.0 / sqrt(var + (double)eps);
        for (size_t i = 0; i < c; ++i) {
            double y = ((double)row[i] - mean) * inv * (double)gamma[i] + (double)beta[i];
            out[(size_t)p * c + i] = (float)y;
        }
    }
}

/* reference.rs:273-298: accumulator starts at the bias; sum over l in
 * increasing order in f64; rounded once. */
void orc_matmul(const float* a, const float* b, const float* bias, size_t m, size_t k,
                size_t n, int threads, float* out) {
    long long rows = (long long)m;
#pragma omp parallel num_threads(threads)
    {
        double* acc = (double*)malloc(n * sizeof(double));
#pragma omp for schedule(static)
        for (long long i = 0; i < rows; ++i) {
            for (size_t j = 0; j < n; ++j) acc[j] = bias ? (double)bias[j] : 0.0;
            for (size_t l = 0; l < k; ++l) {
                double xv = (double)a[(size_t)i * k + l];
                const float* w = b + l * n;
                for (size_t j = 0; j < n; ++j) acc[j] += xv * (double)w[j];
            }
            for (size_t j = 0; j < n; ++j) out[(size_t)i * n + j] = (float)acc[j];
        }
        free(acc);
    }
}

/* reference.rs:301-306 */
void orc_add(const float* a, const float* b, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = (float)((double)a[i] + (double)b[i]);
}

/* reference.rs:325-330 */
void orc_scale(const float* x, size_t n, float factor, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = (float)((double)x[i] * (double)factor);
}

/* reference.rs:337-360: Maclaurin series below 3, the continued fraction of
 * erfc (60 levels, from the tail) from 3. */
double orc_erf(double x) {
    const double pi = 3.141592653589793238462643383279;
    double z = fabs(x);
    double value;
    if (z < 3.0) {
        double term = z, sum = z, nn = 0.0;
        while (fabs(term) > 1e-17 * fabs(sum)) {
            nn += 1.0;
            term *= -z * z / nn;
            sum += term / (2.0 * nn + 1.0);
        }
        value = sum * 2.0 / sqrt(pi);
    } else {
        double tail = z;
        for (int k = 60; k >= 1; --k) tail = z + (double)k / 2.0 / tail;
        value = 1.0 - exp(-z * z) / sqrt(pi) / tail;
    }
    return copysign(value, x);
}

/* reference.rs:369-376: 0.5 x (1 + erf(x / sqrt 2)) in f64. */
void orc_gelu_erf(const float* x, size_t n, float* out) {
    const double sqrt2 = 1.4142135623730950488016887242097;
    for (size_t i = 0; i < n; ++i) {
        double v = (double)x[i];
        out[i] = (float)(0.5 * v * (1.0 + orc_erf(v / sqrt2)));
    }
}

/* reference.rs:379-384: element i times scale[i % channels]. */
void orc_channel_scale(const float* x, const float* scale, size_t n, size_t channels,
                       float* out) {
    for (size_t i = 0; i < n; ++i)
        out[i] = (float)((double)x[i] * (double)scale[i % channels]);
}

/* reference.rs:388-420: image [gh*p][gw*p][cin], weights [p][p][cin][cout]
 * (HWIO), accumulator from the bias, taps in (ky, kx, ci) order. */
void orc_patch_embed(const float* image, const float* w, const float* bias, size_t gh,
                     size_t gw, size_t p, size_t cin, size_t cout, int threads, float* out) {
    size_t width = gw * p;
    long long patches = (long long)(gh * gw);
#pragma omp parallel num_threads(threads)
    {
        double* acc = (double*)malloc(cout * sizeof(double));
#pragma omp for schedule(static)
        for (long long g = 0; g < patches; ++g) {
            size_t gy = (size_t)g / gw, gx = (size_t)g % gw;
            for (size_t co = 0; co < cout; ++co) acc[co] = bias ? (double)bias[co] : 0.0;
            for (size_t ky = 0; ky < p; ++ky)
                for (size_t kx = 0; kx < p; ++kx) {
                    size_t pixel = ((gy * p + ky) * width + gx * p + kx) * cin;
                    for (size_t ci = 0; ci < cin; ++ci) {
                        double xv = (double)image[pixel + ci];
                        const float* row = w + ((ky * p + kx) * cin + ci) * cout;
                        for (size_t co = 0; co < cout; ++co) acc[co] += xv * (double)row[co];
                    }
                }
            for (size_t co = 0; co < cout; ++co) out[(size_t)g * cout + co] = (float)acc[co];
        }
        free(acc);
    }
}

/* reference.rs:423-425 */
void orc_prepend_token(const float* token, const float* tokens, size_t rows, size_t c,
                       float* out) {
    memcpy(out, token, c * sizeof(float));
    memcpy(out + c, tokens, rows * c * sizeof(float));
}

/* reference.rs:428-430: drops the first token. */
void orc_tokens_to_map(const float* input, size_t tokens, size_t c, float* out) {
    memcpy(out, input + c, (tokens - 1) * c * sizeof(float));
}

/* reference.rs:437-455 */
void orc_attention_scores(const float* qkv, size_t t, size_t h, size_t d, int threads,
                          float* out) {
    size_t row = 3 * h * d;
    long long n = (long long)t;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long i = 0; i < n; ++i)
        for (size_t head = 0; head < h; ++head) {
            const float* q = qkv + (size_t)i * row + head * d;
            for (size_t j = 0; j < t; ++j) {
                const float* k = qkv + j * row + h * d + head * d;
                double dot = 0.0;
                for (size_t c = 0; c < d; ++c) dot += (double)q[c] * (double)k[c];
                out[((size_t)i * h + head) * t + j] = (float)dot;
            }
        }
}

/* One softmax row (reference.rs:459-470): f64 max, exp, sum; rounded once. */
static void softmax_row(const float* x, size_t cols, double* exps, float* out) {
    double mx = -INFINITY;
    for (size_t c = 0; c < cols; ++c) {
        double v = (double)x[c];
        if (v > mx) mx = v;
    }
    double sum = 0.0;
    for (size_t c = 0; c < cols; ++c) {
        exps[c] = exp((double)x[c] - mx);
        sum += exps[c];
    }
    for (size_t c = 0; c < cols; ++c) out[c] = (float)(exps[c] / sum);
}

void orc_softmax(const float* x, size_t rows, size_t cols, int threads, float* out) {
    long long n = (long long)rows;
#pragma omp parallel num_threads(threads)
    {
        double* exps = (double*)malloc(cols * sizeof(double));
#pragma omp for schedule(static)
        for (long long r = 0; r < n; ++r)
            softmax_row(x + (size_t)r * cols, cols, exps, out + (size_t)r * cols);
        free(exps);
    }
}

/* reference.rs:474-494: f64 accumulator over j in increasing order. */
void orc_attention_values(const float* probs, const float* qkv, size_t t, size_t h,
                          size_t d, int threads, float* out) {
    size_t row = 3 * h * d;
    long long n = (long long)t;
#pragma omp parallel num_threads(threads)
    {
        double* acc = (double*)malloc(d * sizeof(double));
#pragma omp for schedule(static)
        for (long long i = 0; i < n; ++i)
            for (size_t head = 0; head < h; ++head) {
                for (size_t c = 0; c < d; ++c) acc[c] = 0.0;
                const float* p = probs + ((size_t)i * h + head) * t;
                for (size_t j = 0; j < t; ++j) {
                    const float* v = qkv + j * row + 2 * h * d + head * d;
                    double wgt = (double)p[j];
                    for (size_t c = 0; c < d; ++c) acc[c] += wgt * (double)v[c];
                }
                for (size_t c = 0; c < d; ++c) out[(size_t)i * h * d + head * d + c] = (float)acc[c];
            }
        free(acc);
    }
}

void orc_attention_rows(const float* qkv, size_t t, size_t h, size_t d, float scale,
                        size_t row_begin, size_t row_end, size_t head_begin,
                        size_t head_end, int threads, float* out) {
    size_t row = 3 * h * d;
    long long units = (long long)((row_end - row_begin) * (head_end - head_begin));
    size_t nh = head_end - head_begin;
#pragma omp parallel num_threads(threads)
    {
        float* scores = (float*)malloc(t * sizeof(float));
        float* probs = (float*)malloc(t * sizeof(float));
        double* exps = (double*)malloc(t * sizeof(double));
        double* acc = (double*)malloc(d * sizeof(double));
#pragma omp for schedule(dynamic, 4)
        for (long long u = 0; u < units; ++u) {
            size_t i = row_begin + (size_t)u / nh;
            size_t head = head_begin + (size_t)u % nh;
            const float* q = qkv + i * row + head * d;
            /* attention_scores (437-455), then Scale (325-330) */
            for (size_t j = 0; j < t; ++j) {
                const float* k = qkv + j * row + h * d + head * d;
                double dot = 0.0;
                for (size_t c = 0; c < d; ++c) dot += (double)q[c] * (double)k[c];
                float s = (float)dot;
                scores[j] = (float)((double)s * (double)scale);
            }
            softmax_row(scores, t, exps, probs);          /* 459-470 */
            for (size_t c = 0; c < d; ++c) acc[c] = 0.0;  /* 474-494 */
            for (size_t j = 0; j < t; ++j) {
                const float* v = qkv + j * row + 2 * h * d + head * d;
                double wgt = (double)probs[j];
                for (size_t c = 0; c < d; ++c) acc[c] += wgt * (double)v[c];
            }
            float* o = out + (i - row_begin) * h * d + head * d;
            for (size_t c = 0; c < d; ++c) o[c] = (float)acc[c];
        }
        free(scores); free(probs); free(exps); free(acc);
    }
}

/* ---------------------------------------------------------------- block */

/* reference.rs:520-544:
 *   x1 = x + ls1 * proj(attention(norm1(x)))
 *   out = x1 + ls2 * fc2(gelu_erf(fc1(norm2(x1))))
 * add(x, channel_scale(projected)) adds in the order x + scaled; f64 addition
 * is commutative, so operand order does not change the result. */
void orc_vit_block(const float* x, const orc_block_weights* w, size_t t, size_t h, size_t d,
                   size_t mlp, float eps, int threads, orc_round_fn qkv_round, void* ctx,
                   float* out) {
    size_t width = h * d;
    size_t tw = t * width;
    float* n1 = (float*)malloc(tw * sizeof(float));
    float* qkv = (float*)malloc(t * 3 * width * sizeof(float));
    float* values = (float*)malloc(tw * sizeof(float));
    float* projected = (float*)malloc(tw * sizeof(float));
    float* x1 = (float*)malloc(tw * sizeof(float));
    float* hidden = (float*)malloc(t * mlp * sizeof(float));
    float scale = 1.0f / sqrtf((float)d);

    orc_layernorm(x, w->norm1_g, w->norm1_b, t, width, eps, threads, n1);
    orc_matmul(n1, w->qkv_w, w->qkv_b, t, width, 3 * width, threads, qkv);
    if (qkv_round) qkv_round(qkv, t * 3 * width, ctx);
    orc_attention_rows(qkv, t, h, d, scale, 0, t, 0, h, threads, values);
    orc_matmul(values, w->proj_w, w->proj_b, t, width, width, threads, projected);
    orc_channel_scale(projected, w->ls1, tw, width, projected);
    orc_add(x, projected, tw, x1);
    orc_layernorm(x1, w->norm2_g, w->norm2_b, t, width, eps, threads, n1);
    orc_matmul(n1, w->fc1_w, w->fc1_b, t, width, mlp, threads, hidden);
    orc_gelu_erf(hidden, t * mlp, hidden);
    orc_matmul(hidden, w->fc2_w, w->fc2_b, t, mlp, width, threads, projected);
    orc_channel_scale(projected, w->ls2, tw, width, projected);
    orc_add(x1, projected, tw, out);

    free(n1); free(qkv); free(values); free(projected); free(x1); free(hidden);
}

/* ---------------------------------------------------------------- rounding */

void orc_round_f16(float* values, size_t count, void* ctx) {
    (void)ctx;
    for (size_t i = 0; i < count; ++i) values[i] = (float)(_Float16)values[i];
}

void orc_round_bf16(float* values, size_t count, void* ctx) {
    (void)ctx;
    for (size_t i = 0; i < count; ++i) {
        uint32_t bits;
        memcpy(&bits, &values[i], 4);
        if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu)) {
            bits |= 0x00400000u; /* quiet NaN stays NaN */
        } else {
            bits += 0x7FFFu + ((bits >> 16) & 1u);
        }
        bits &= 0xFFFF0000u;
        memcpy(&values[i], &bits, 4);
    }
}

/* Models the backend's packed Q|K|V storage: in every row of 3 * width
 * values, Q and K rounded to bf16 (ctx != NULL: *(size_t*)ctx = width) or
 * f16, V always to f16. */
static void round_qkv(float* values, size_t count, size_t width, int qk_bf16) {
    size_t row = 3 * width;
    for (size_t r = 0; r < count / row; ++r) {
        float* v = values + r * row;
        if (qk_bf16) orc_round_bf16(v, 2 * width, NULL); else orc_round_f16(v, 2 * width, NULL);
        orc_round_f16(v + 2 * width, width, NULL);
    }
}

void orc_round_qkv_bf16(float* values, size_t count, void* ctx) {
    round_qkv(values, count, *(const size_t*)ctx, 1);
}

void orc_round_qkv_f16(float* values, size_t count, void* ctx) {
    round_qkv(values, count, *(const size_t*)ctx, 0);
}

/* ------------------------------------------------------------- DPT decoder */

/* crates/beatlm-bench/src/reference.rs:31-77 (conv3x3, conv3x3_strided):
 * zero padding 1, output (y, x) centred on input (y s, x s), oh = (h-1)/s+1;
 * per output value the bias, then taps ky, kx, then ci in increasing order,
 * accumulated in f64 and rounded once. HWIO weights [3][3][cin][cout]. */
void orc_conv3x3(const float* input, const float* w, const float* bias, size_t h, size_t wd,
                 size_t cin, size_t cout, size_t stride, int threads, float* out) {
    const size_t oh = (h - 1) / stride + 1, ow = (wd - 1) / stride + 1;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long yy = 0; yy < (long long)oh; ++yy) {
        const size_t y = (size_t)yy;
        for (size_t x = 0; x < ow; ++x)
            for (size_t co = 0; co < cout; ++co) {
                double acc = bias ? (double)bias[co] : 0.0;
                for (size_t ky = 0; ky < 3; ++ky)
                    for (size_t kx = 0; kx < 3; ++kx) {
                        const long long iy = (long long)(y * stride + ky) - 1;
                        const long long ix = (long long)(x * stride + kx) - 1;
                        if (iy < 0 || ix < 0 || iy >= (long long)h || ix >= (long long)wd) continue;
                        const float* a = input + ((size_t)iy * wd + (size_t)ix) * cin;
                        const float* b = w + (ky * 3 + kx) * cin * cout + co;
                        for (size_t ci = 0; ci < cin; ++ci) acc += (double)a[ci] * (double)b[ci * cout];
                    }
                out[(y * ow + x) * cout + co] = (float)acc;
            }
    }
}

/* reference.rs:79-101 (conv1x1): [pixels][cin] x [cin][cout] + bias, f64. */
void orc_conv1x1(const float* input, const float* w, const float* bias, size_t pixels,
                 size_t cin, size_t cout, int threads, float* out) {
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long pp = 0; pp < (long long)pixels; ++pp) {
        const size_t p = (size_t)pp;
        for (size_t co = 0; co < cout; ++co) {
            double acc = bias ? (double)bias[co] : 0.0;
            for (size_t ci = 0; ci < cin; ++ci)
                acc += (double)input[p * cin + ci] * (double)w[ci * cout + co];
            out[p * cout + co] = (float)acc;
        }
    }
}

/* reference.rs:103-140 (conv_transpose): kernel = stride = f, no padding;
 * input pixel (y, x) adds its channels times tap (ky, kx) of the HWIO weights
 * [f][f][cin][cout] into output pixel (y f + ky, x f + kx), in f64; the bias
 * is added last and the sum rounded once. */
void orc_conv_transpose(const float* input, const float* w, const float* bias, size_t h,
                        size_t wd, size_t cin, size_t cout, size_t f, int threads, float* out) {
    const size_t ow = wd * f;
#pragma omp parallel for num_threads(threads) schedule(static)
    for (long long yy = 0; yy < (long long)h; ++yy) {
        const size_t y = (size_t)yy;
        double* acc = (double*)malloc(sizeof(double) * cout);
        for (size_t x = 0; x < wd; ++x)
            for (size_t ky = 0; ky < f; ++ky)
                for (size_t kx = 0; kx < f; ++kx) {
                    for (size_t co = 0; co < cout; ++co) acc[co] = 0.0;
                    const float* px = input + (y * wd + x) * cin;
                    for (size_t ci = 0; ci < cin; ++ci) {
                        const float* taps = w + ((ky * f + kx) * cin + ci) * cout;
                        for (size_t co = 0; co < cout; ++co) acc[co] += (double)px[ci] * (double)taps[co];
                    }
                    float* o = out + ((y * f + ky) * ow + x * f + kx) * cout;
                    for (size_t co = 0; co < cout; ++co)
                        o[co] = (float)(acc[co] + (bias ? (double)bias[co] : 0.0));
                }
        free(acc);
    }
}

/* reference.rs:142-175 (resize_bilinear): corners aligned, f64; output row
 * oy reads position oy (ih-1)/(oh-1) (0 for one output row), between its
 * floor and the next row, clamped to the last; columns likewise. */
static void bilinear_axis(size_t o, size_t in, size_t outn, size_t* i0, size_t* i1, double* l) {
    const double pos = outn > 1 ? (double)o * (double)(in - 1) / (double)(outn - 1) : 0.0;
    size_t a = (size_t)floor(pos);
    if (a > in - 1) a = in - 1;
    *i0 = a;
    *i1 = a + 1 < in ? a + 1 : in - 1;
    *l = pos - (double)a;
}

void orc_resize_bilinear(const float* input, size_t ih, size_t iw, size_t oh, size_t ow,
                         size_t c, float* out) {
    for (size_t oy = 0; oy < oh; ++oy) {
        size_t y0, y1;
        double ly;
        bilinear_axis(oy, ih, oh, &y0, &y1, &ly);
        for (size_t ox = 0; ox < ow; ++ox) {
            size_t x0, x1;
            double lx;
            bilinear_axis(ox, iw, ow, &x0, &x1, &lx);
            for (size_t ch = 0; ch < c; ++ch) {
                const double a00 = input[(y0 * iw + x0) * c + ch], a01 = input[(y0 * iw + x1) * c + ch];
                const double a10 = input[(y1 * iw + x0) * c + ch], a11 = input[(y1 * iw + x1) * c + ch];
                const double top = (1.0 - lx) * a00 + lx * a01;
                const double bottom = (1.0 - lx) * a10 + lx * a11;
                out[(oy * ow + ox) * c + ch] = (float)((1.0 - ly) * top + ly * bottom);
            }
        }
    }
}
