"""Host-side calls of the fused kernels, on device buffers (torch tensors are
used only as device memory and for the current stream)."""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import _native as N

_TORCH_DTYPE_CODE = {}


def _dtype_code(name: str) -> int:
    return {"f32": N.BL_F32, "f16": N.BL_F16, "bf16": N.BL_BF16}[name]


def _stream_ptr(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def pack_qkv(qkv, qk_dtype: str = "f16", device="cuda"):
    """Packs f32 ``[..., tokens, 3, heads, head_dim]`` values into one 16-bit
    device buffer: the Q and K sections in ``qk_dtype`` ("f16" or "bf16"), the
    V section in f16, the layout the attention kernel reads."""
    import torch
    a = torch.as_tensor(np.ascontiguousarray(qkv, dtype=np.float32))
    qk = a[..., :2, :, :].to(torch.bfloat16 if qk_dtype == "bf16" else torch.float16)
    v = a[..., 2:, :, :].to(torch.float16)
    out = torch.empty(a.shape, dtype=torch.int16)
    out[..., :2, :, :] = qk.view(torch.int16)
    out[..., 2:, :, :] = v.view(torch.int16)
    return out.to(device)


def attention(qkv, *, tokens: int, heads: int, head_dim: int = 64, batch: int = 1,
              qk_dtype: str = "f16", out=None, out_dtype: str = "f32", scale: float | None = None,
              rows: tuple[int, int] | None = None, head_range: tuple[int, int] | None = None,
              out_head_base: int = 0, stream=None):
    """The fused scores -> scale -> softmax -> values chain of one layer
    (reference kernel.rs:722-777) on packed ``[batch][tokens][3][heads][64]``
    16-bit ``qkv``; returns ``out`` ``[batch][tokens][heads * 64]``."""
    import torch
    if scale is None:
        scale = 1.0 / math.sqrt(head_dim)
    r0, r1 = rows or (0, tokens)
    h0, h1 = head_range or (0, heads)
    width = (h1 - out_head_base) * head_dim if head_range else heads * head_dim
    if out is None:
        tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[out_dtype]
        out = torch.zeros((batch, tokens, width), dtype=tdt, device=qkv.device)
    a = N.AttentionArgs(batch=batch, tokens=tokens, heads=heads, head_dim=head_dim,
                        head_begin=h0, head_end=h1, row_begin=r0, row_end=r1, scale=scale,
                        qk_dtype=_dtype_code(qk_dtype), v_dtype=N.BL_F16,
                        out_dtype=_dtype_code(out_dtype), qkv=qkv.data_ptr(), qkv_row_stride=0,
                        out=out.data_ptr(), out_row_stride=out.shape[-1],
                        out_head_base=out_head_base)
    N.check(N.lib().bl_attention(ctypes.byref(a), _stream_ptr(stream)))
    return out
