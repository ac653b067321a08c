/*
 * CPU oracle for the ViT attention hot path: TEST INFRASTRUCTURE ONLY.
 *
 * A C restatement of the reference's f64-accumulating CPU operations
 * (crates/beatlm-bench/src/reference.rs), with every operation's result
 * rounded to f32 before the next reads it, exactly as that file does. The
 * product library never links, loads or calls this code; only tests/,
 * __graft_entry__.smoke() and bench.py (its cpu_baseline leg and its
 * `--impl reference` arm) may.
 *
 * Parity pinning: the reference is Rust (no toolchain here), so it cannot be
 * run. This restatement is pinned by the reference's own known-answer tests
 * (reference.rs:723-837), transcribed into tests/golden/reference_kats.json
 * and checked by tests/test_oracle.py.
 *
 * Threads: every function taking `threads` parallelises over independent
 * output rows only, so the arithmetic of each element (and therefore the
 * result, bit for bit) is the same for any thread count. threads = 1 is the
 * faithful single-threaded reference.
 */
#ifndef BEATLM_ORACLE_H
#define BEATLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Seeded data: the LCG of crates/beatlm-bench/src/net.rs:183-203. */
void orc_uniform(uint64_t seed, size_t count, float low, float high, float* out);
/* N(mean, std) by Box-Muller over pairs of the LCG's draws (this build's own
 * convention; the reference draws only uniforms). */
void orc_normal(uint64_t seed, size_t count, float mean, float std, float* out);

/* reference.rs:247-270 */
void orc_layernorm(const float* x, const float* gamma, const float* beta, size_t rows,
                   size_t c, float eps, int threads, float* out);
/* reference.rs:273-298; bias may be NULL */
void orc_matmul(const float* a, const float* b, const float* bias, size_t m, size_t k,
                size_t n, int threads, float* out);
/* reference.rs:301-306 */
void orc_add(const float* a, const float* b, size_t n, float* out);
/* reference.rs:325-330 */
void orc_scale(const float* x, size_t n, float factor, float* out);
/* reference.rs:337-360 */
double orc_erf(double x);
/* reference.rs:369-376 */
void orc_gelu_erf(const float* x, size_t n, float* out);
/* reference.rs:379-384 */
void orc_channel_scale(const float* x, const float* scale, size_t n, size_t channels,
                       float* out);
/* reference.rs:388-420; bias may be NULL */
void orc_patch_embed(const float* image, const float* w, const float* bias, size_t gh,
                     size_t gw, size_t p, size_t cin, size_t cout, int threads, float* out);
/* reference.rs:423-425 */
void orc_prepend_token(const float* token, const float* tokens, size_t rows, size_t c,
                       float* out);
/* reference.rs:428-430 */
void orc_tokens_to_map(const float* input, size_t tokens, size_t c, float* out);

/* reference.rs:437-455: S[i][h][j] from qkv [t][3][h][d] -> [t][h][t] */
void orc_attention_scores(const float* qkv, size_t t, size_t h, size_t d, int threads,
                          float* out);
/* reference.rs:459-470 */
void orc_softmax(const float* x, size_t rows, size_t cols, int threads, float* out);
/* reference.rs:474-494: O[i][h*d] from probs [t][h][t] and qkv */
void orc_attention_values(const float* probs, const float* qkv, size_t t, size_t h,
                          size_t d, int threads, float* out);

/* The scores -> scale -> softmax -> values chain of the reference
 * (depth_anything_v2.rs:340-367 built from reference.rs:437-494), evaluated
 * one (query, head) row at a time so no [t][h][t] tensor is materialised.
 * Every element goes through the same roundings in the same order as the
 * materialised chain, so the two agree bit for bit. Computes query rows
 * [row_begin, row_end) and heads [head_begin, head_end) of `qkv`
 * ([batch-less] [t][3][h][d]); writes out[(i - row_begin)][head * d + c] with
 * row stride h * d. */
void orc_attention_rows(const float* qkv, size_t t, size_t h, size_t d, float scale,
                        size_t row_begin, size_t row_end, size_t head_begin,
                        size_t head_end, int threads, float* out);

/* The weights of one pre-norm ViT block in the IR's layouts
 * (reference.rs:496-517): linear weights [in][out]. */
typedef struct orc_block_weights {
    const float* norm1_g; const float* norm1_b;
    const float* qkv_w;   const float* qkv_b;      /* [w][3w], [3w] */
    const float* proj_w;  const float* proj_b;     /* [w][w],  [w]  */
    const float* ls1;
    const float* norm2_g; const float* norm2_b;
    const float* fc1_w;   const float* fc1_b;      /* [w][mlp], [mlp] */
    const float* fc2_w;   const float* fc2_b;      /* [mlp][w], [w] */
    const float* ls2;
} orc_block_weights;

/* reference.rs:520-544. When qkv_round is non-NULL it is called on the packed
 * [t][3w] projection before attention reads it, so a test can model storage of
 * Q/K/V in 16-bit formats; NULL keeps the reference's f32 values. */
typedef void (*orc_round_fn)(float* values, size_t count, void* ctx);
void orc_vit_block(const float* x, const orc_block_weights* w, size_t t, size_t h, size_t d,
                   size_t mlp, float eps, int threads, orc_round_fn qkv_round, void* ctx,
                   float* out);

/* Rounding helpers that model 16-bit storage: round-to-nearest-even to
 * binary16 / bfloat16 and back to f32. */
void orc_round_f16(float* values, size_t count, void* ctx);
void orc_round_bf16(float* values, size_t count, void* ctx);
/* Packed Q|K|V rows of 3 * width values (ctx points to a size_t width):
 * Q and K rounded to bf16 (resp. f16), V to f16. */
void orc_round_qkv_bf16(float* values, size_t count, void* ctx);
void orc_round_qkv_f16(float* values, size_t count, void* ctx);

/* DPT decoder operations (crates/beatlm-bench/src/reference.rs:25-175), NHWC
 * f32 maps, HWIO weights, f64 accumulation rounded once; bias may be NULL. */
void orc_conv3x3(const float* input, const float* w, const float* bias, size_t h, size_t wd,
                 size_t cin, size_t cout, size_t stride, int threads, float* out);
void orc_conv1x1(const float* input, const float* w, const float* bias, size_t pixels,
                 size_t cin, size_t cout, int threads, float* out);
void orc_conv_transpose(const float* input, const float* w, const float* bias, size_t h,
                        size_t wd, size_t cin, size_t cout, size_t f, int threads, float* out);
void orc_resize_bilinear(const float* input, size_t ih, size_t iw, size_t oh, size_t ow,
                         size_t c, float* out);

#ifdef __cplusplus
}
#endif
#endif
