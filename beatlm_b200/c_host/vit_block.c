/*
 * A host of the C ABI alone (no Python, no PyTorch, no CUDA calls of its
 * own): one pre-norm ViT block of f16 weights on the residual stream x, the
 * way the reference's host runs a program (crates/beatlm/src/model/mod.rs and
 * crates/beatlm-host/src/slots.rs: plan, arenas, kernels, encode, timer,
 * read back):
 *
 *   plan   bl_plan_create over every weight and activation with lifetimes in
 *          program order (MemoryPlan::new), on the CUDA device's profile;
 *   arenas bl_arenas_create (one device allocation), weights and x written
 *          into their placements (bl_arenas_write);
 *   kernels the block's seven launches as specs (LayerNorm, QKV GEMM with
 *          packed Q|K|V and f16 V, attention, out-projection with LayerScale
 *          and residual, LayerNorm, fc1 with GELU-erf, fc2 with LayerScale and
 *          residual), built once (bl_kernels_create);
 *   encode bl_kernels_encode_range on the legacy default stream under the
 *          slice timer (bl_timer_*), collected without blocking;
 *   read   bl_status, then bl_arenas_read of x.
 *
 *   vit_block <input> <output>
 *
 * <input>: int32 tokens, dim, heads, mlp; then f32 arrays: x [tokens][dim] and
 * the block's weights in the reference's layouts (linear weights [in][out]),
 * in the order norm1_g, norm1_b, qkv_w, qkv_b, proj_w, proj_b, ls1, norm2_g,
 * norm2_b, fc1_w, fc1_b, fc2_w, fc2_b, ls2. <output>: x after the block,
 * f32 [tokens][dim]. Prints the plan's size and each kernel's time.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "beatlm_b200.h"

#define CHECK(call)                                                             \
    do {                                                                        \
        int rc_ = (call);                                                       \
        if (rc_ != BL_OK) {                                                     \
            char msg_[1024];                                                    \
            bl_last_error(msg_, sizeof msg_);                                   \
            fprintf(stderr, "%s:%d: %s -> %d: %s\n", __FILE__, __LINE__, #call, \
                    rc_, msg_);                                                 \
            exit(2);                                                            \
        }                                                                       \
    } while (0)

/* IEEE binary32 -> binary16, round to nearest even (the standard
 * conversion; subnormals and overflow to infinity included). */
static uint16_t f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) /* inf or nan */
        return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds past the largest */
    if (absx < 0x38800000u) {                                   /* subnormal or zero in f16 */
        if (absx < 0x33000000u) return (uint16_t)sign;
        const uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
        const int shift = 126 - (int)(absx >> 23); /* 14..24 */
        const uint32_t half = 1u << (shift - 1), rest = m & ((1u << shift) - 1);
        uint32_t v = m >> shift;
        if (rest > half || (rest == half && (v & 1u))) v += 1;
        return (uint16_t)(sign | v);
    }
    uint32_t v = ((absx >> 13) - (112u << 10));
    const uint32_t rest = absx & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (v & 1u))) v += 1;
    return (uint16_t)(sign | v);
}

static void* read_all(const char* path, size_t* n) {
    FILE* f = fopen(path, "rb");
    if (!f) { perror(path); exit(2); }
    fseek(f, 0, SEEK_END);
    *n = (size_t)ftell(f);
    fseek(f, 0, SEEK_SET);
    void* p = malloc(*n);
    if (fread(p, 1, *n, f) != *n) { fprintf(stderr, "short read\n"); exit(2); }
    fclose(f);
    return p;
}

/* [in][out] f32 -> [out][in] f16 (the tensor cores' K-major B operand). */
static uint16_t* linear_f16(const float* w, uint32_t in, uint32_t out) {
    uint16_t* t = malloc((size_t)in * out * 2);
    for (uint32_t i = 0; i < in; ++i)
        for (uint32_t o = 0; o < out; ++o) t[(size_t)o * in + i] = f32_to_f16(w[(size_t)i * out + o]);
    return t;
}

enum { N1G, N1B, QKVW, QKVB, PROJW, PROJB, LS1, N2G, N2B, FC1W, FC1B, FC2W, FC2B, LS2,
       X, XN, QKV, O, H, NTENSORS };

int main(int argc, char** argv) {
    if (argc != 3) { fprintf(stderr, "usage: vit_block <input> <output>\n"); return 2; }
    size_t nbytes = 0;
    char* in = read_all(argv[1], &nbytes);
    int32_t dims[4];
    memcpy(dims, in, sizeof dims);
    const uint32_t T = (uint32_t)dims[0], D = (uint32_t)dims[1], HEADS = (uint32_t)dims[2],
                   M = (uint32_t)dims[3];
    const float* src = (const float*)(in + sizeof dims);
    const size_t count[14] = {D, D, (size_t)D * 3 * D, 3 * D, (size_t)D * D, D, D, D, D,
                              (size_t)D * M, M, (size_t)M * D, D, D};
    const float* x = src;
    const float* w[14];
    const float* p = src + (size_t)T * D;
    for (int i = 0; i < 14; ++i) { w[i] = p; p += count[i]; }
    if ((size_t)((const char*)p - in) != nbytes) { fprintf(stderr, "input size\n"); return 2; }

    /* plan: every tensor with its lifetime over ops 0..6 (norm1, qkv,
     * attention, proj, norm2, fc1, fc2) */
    bl_tensor_desc t[NTENSORS];
    for (int i = 0; i < 14; ++i) {
        const int lin = i == QKVW || i == PROJW || i == FC1W || i == FC2W;
        t[i] = (bl_tensor_desc){(uint32_t)i, lin ? 2u : 4u, count[i], 0, 6};
    }
    t[X] = (bl_tensor_desc){X, 4, (uint64_t)T * D, 0, 6};
    t[XN] = (bl_tensor_desc){XN, 2, (uint64_t)T * D, 0, 5};
    t[QKV] = (bl_tensor_desc){QKV, 2, (uint64_t)T * 3 * D, 1, 2};
    t[O] = (bl_tensor_desc){O, 2, (uint64_t)T * D, 2, 3};
    t[H] = (bl_tensor_desc){H, 2, (uint64_t)T * M, 5, 6};
    bl_device_profile prof;
    CHECK(bl_device_profile_cuda(0, &prof));
    bl_plan* plan = NULL;
    bl_plan_error perr;
    CHECK(bl_plan_create(t, NTENSORS, &prof, &plan, &perr));
    bl_arenas* ar = NULL;
    CHECK(bl_arenas_create(plan, 0, &ar));
    bl_placement pl[NTENSORS];
    void* dev[NTENSORS];
    for (int i = 0; i < NTENSORS; ++i) {
        CHECK(bl_plan_placement(plan, (uint32_t)i, &pl[i]));
        CHECK(bl_arenas_binding(ar, &pl[i], &dev[i]));
    }
    printf("plan: %llu bytes in one allocation of %llu (peak live %llu)\n",
           (unsigned long long)bl_plan_total_bytes(plan), (unsigned long long)bl_arenas_bytes(ar),
           (unsigned long long)bl_plan_peak_live_bytes(plan));

    /* weights and input into their placements (synchronous host buffers) */
    uint16_t* lin[14] = {0};
    lin[QKVW] = linear_f16(w[QKVW], D, 3 * D);
    lin[PROJW] = linear_f16(w[PROJW], D, D);
    lin[FC1W] = linear_f16(w[FC1W], D, M);
    lin[FC2W] = linear_f16(w[FC2W], M, D);
    for (int i = 0; i < 14; ++i) {
        const void* data = lin[i] ? (const void*)lin[i] : (const void*)w[i];
        CHECK(bl_arenas_write(ar, &pl[i], 0, data, count[i] * (lin[i] ? 2 : 4), NULL));
    }
    CHECK(bl_arenas_write(ar, &pl[X], 0, x, (uint64_t)T * D * 4, NULL));

    /* the seven kernels */
    const float eps = 1e-6f;
    bl_layernorm_args ln1 = {0}, ln2 = {0};
    ln1.rows = T, ln1.cols = D, ln1.x = dev[X], ln1.ldx = D, ln1.gamma = dev[N1G];
    ln1.beta = dev[N1B], ln1.eps = eps, ln1.out = dev[XN], ln1.out_dtype = BL_F16, ln1.ldo = D;
    ln2 = ln1;
    ln2.gamma = dev[N2G], ln2.beta = dev[N2B];
    bl_gemm_args qkv = {0}, proj = {0}, fc1 = {0}, fc2 = {0};
    qkv.m = T, qkv.n = 3 * D, qkv.k = D, qkv.ab_dtype = BL_F16, qkv.a = dev[XN], qkv.lda = D;
    qkv.b = dev[QKVW], qkv.ldb = D, qkv.bias = dev[QKVB], qkv.out = dev[QKV];
    qkv.out_dtype = BL_F16, qkv.out_ld = 3 * D, qkv.split_col = 2 * D, qkv.out_dtype_hi = BL_F16;
    qkv.weights_static = 1;
    proj.m = T, proj.n = D, proj.k = D, proj.ab_dtype = BL_F16, proj.a = dev[O], proj.lda = D;
    proj.b = dev[PROJW], proj.ldb = D, proj.bias = dev[PROJB], proj.chan_scale = dev[LS1];
    proj.residual = dev[X], proj.res_dtype = BL_F32, proj.res_ld = D, proj.out = dev[X];
    proj.out_dtype = BL_F32, proj.out_ld = D, proj.weights_static = 1;
    fc1.m = T, fc1.n = M, fc1.k = D, fc1.ab_dtype = BL_F16, fc1.a = dev[XN], fc1.lda = D;
    fc1.b = dev[FC1W], fc1.ldb = D, fc1.bias = dev[FC1B], fc1.act = BL_ACT_GELU_ERF;
    fc1.out = dev[H], fc1.out_dtype = BL_F16, fc1.out_ld = M, fc1.weights_static = 1;
    fc2 = proj;
    fc2.k = M, fc2.a = dev[H], fc2.lda = M, fc2.b = dev[FC2W], fc2.ldb = M, fc2.bias = dev[FC2B];
    fc2.chan_scale = dev[LS2];
    bl_attention_args att = {0};
    att.batch = 1, att.tokens = T, att.heads = HEADS, att.head_dim = D / HEADS;
    att.head_begin = 0, att.head_end = HEADS, att.row_begin = 0, att.row_end = T;
    att.scale = 1.0f / sqrtf((float)(D / HEADS)), att.qk_dtype = BL_F16, att.v_dtype = BL_F16;
    att.out_dtype = BL_F16, att.qkv = dev[QKV], att.out = dev[O];
    const bl_kernel_spec specs[7] = {
        {BL_OP_LAYERNORM, &ln1, "norm1", 1}, {BL_OP_GEMM, &qkv, "qkv", 1},
        {BL_OP_ATTENTION, &att, "attention", 1}, {BL_OP_GEMM, &proj, "proj", 1},
        {BL_OP_LAYERNORM, &ln2, "norm2", 1}, {BL_OP_GEMM, &fc1, "fc1", 1},
        {BL_OP_GEMM, &fc2, "fc2", 1}};
    bl_kernels* k = NULL;
    CHECK(bl_kernels_create(specs, 7, NULL, 0, &k));

    /* encode under the slice timer, collect without blocking */
    bl_timer* timer = NULL;
    CHECK(bl_timer_create(7, &timer));
    int32_t h = -1;
    CHECK(bl_timer_begin_frame(timer, 0, &h));
    CHECK(bl_kernels_encode_range(k, 0, bl_kernels_len(k), 0, NULL, timer, h));
    CHECK(bl_timer_submitted(timer, h));
    bl_slice_time times[7];
    size_t n = 0, frames = 0;
    for (int polls = 0; frames == 0 && polls < 10000; ++polls) {
        CHECK(bl_timer_collect_ready(timer, times, 7, &n, &frames));
        if (frames == 0) {
            struct timespec ts = {0, 1000000};
            nanosleep(&ts, NULL);
        }
    }
    if (frames != 1 || n != 7) { fprintf(stderr, "timer: %zu frames, %zu passes\n", frames, n); return 3; }
    for (size_t i = 0; i < n; ++i)
        printf("%-10s %8.2f us\n", bl_kernels_label(k, times[i].kernel), times[i].micros);

    bl_status_t st;
    CHECK(bl_status(&st, 1));
    if (st.code != 0) { fprintf(stderr, "device status 0x%x\n", st.code); return 4; }
    float* out = malloc((size_t)T * D * 4);
    CHECK(bl_arenas_read(ar, &pl[X], 0, out, (uint64_t)T * D * 4, NULL));
    FILE* f = fopen(argv[2], "wb");
    if (!f || fwrite(out, 4, (size_t)T * D, f) != (size_t)T * D) { perror(argv[2]); return 2; }
    fclose(f);

    bl_timer_destroy(timer);
    bl_kernels_destroy(k);
    bl_arenas_destroy(ar);
    bl_plan_destroy(plan);
    for (int i = 0; i < 14; ++i) free(lin[i]);
    free(out);
    free(in);
    printf("ok\n");
    return 0;
}
