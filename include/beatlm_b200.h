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
    BL_ERR_CAPACITY = 5     /* a plan or buffer does not fit (reference: PlanError, memory.rs:220) */
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
} bl_attention_args;

int bl_attention(const bl_attention_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif
