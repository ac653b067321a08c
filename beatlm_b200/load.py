"""Real weights for the encoder: a safetensors reader, the backbone part of
Depth Anything V2's tensor inventory, and the conversions from the stored
layouts to the encoder's. The host side of the reference's loader
(``crates/beatlm/src/load/reader.rs``, ``load/inventory.rs``,
``load/depth_anything_v2.rs:470-590``) and of its layout conversions
(``crates/beatlm/src/model/mod.rs:272-353``, ``model/positions.rs``).

Only the transformer (the path this package runs) is taken from a file; the
DPT neck and head tensors a checkpoint also holds are left unread.

    w = load.encoder_weights("model.safetensors", cfg)   # -> Encoder(cfg, w, "bf16")
"""
from __future__ import annotations

import dataclasses
import json
import math
import struct

import numpy as np

# stored element types (reader.rs StoredType): numpy types of those with a name
_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": None, "F64": np.float64,
           "U8": np.uint8, "I32": np.int32, "I64": np.int64}
_SIZES = {"F32": 4, "F16": 2, "BF16": 2, "F64": 8, "U8": 1, "I32": 4, "I64": 8, "BOOL": 1,
          "I8": 1, "I16": 2, "U16": 2, "U32": 4, "U64": 8, "F8_E4M3": 1, "F8_E5M2": 1}


class LoadError(ValueError):
    """A file or a tensor that does not fit (load/error.rs): ``kind`` is
    "Format", "Missing", "Shape", "Type" or "Size"."""

    def __init__(self, kind: str, message: str):
        super().__init__("%s: %s" % (kind, message))
        self.kind = kind


@dataclasses.dataclass
class Tensor:
    dtype: str          # the stored type's name, e.g. "F32"
    shape: tuple
    data: memoryview    # the stored bytes, row-major, little endian

    def to_f32(self) -> np.ndarray:
        """The values as float32 (F32, F16 and BF16 only)."""
        if self.dtype == "F32":
            a = np.frombuffer(self.data, dtype="<f4")
        elif self.dtype == "F16":
            a = np.frombuffer(self.data, dtype="<f2").astype(np.float32)
        elif self.dtype == "BF16":
            u = np.frombuffer(self.data, dtype="<u2").astype(np.uint32) << 16
            a = u.view(np.float32)
        else:
            raise LoadError("Type", "%s is not a float type the encoder reads" % self.dtype)
        return a.reshape(self.shape).astype(np.float32, copy=False)


def parse(buf) -> dict:
    """Every tensor of a safetensors buffer, by name (Archive::parse,
    reader.rs): an 8-byte little-endian header length, a JSON header of
    {name: {dtype, shape, data_offsets}} (and an optional __metadata__), then
    the data, which the offsets must cover exactly, in order, each span the
    size of its shape. Anything else is LoadError("Format")."""
    mv = memoryview(buf).cast("B")
    if len(mv) < 8:
        raise LoadError("Format", "shorter than the 8-byte header length")
    (n,) = struct.unpack_from("<Q", mv, 0)
    if n > len(mv) - 8:
        raise LoadError("Format", "header of %d bytes past the end of a %d-byte file" % (n, len(mv)))
    try:
        header = json.loads(bytes(mv[8:8 + n]).decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise LoadError("Format", "header is not JSON: %s" % e) from None
    if not isinstance(header, dict):
        raise LoadError("Format", "header is not an object")
    data = mv[8 + n:]
    spans, out = [], {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        try:
            dtype, shape, (b, e) = info["dtype"], tuple(int(s) for s in info["shape"]), \
                info["data_offsets"]
        except (KeyError, TypeError, ValueError):
            raise LoadError("Format", "tensor %r: malformed entry" % name) from None
        if dtype not in _SIZES:
            raise LoadError("Format", "tensor %r: unknown dtype %r" % (name, dtype))
        if any(s < 0 for s in shape) or not 0 <= b <= e <= len(data):
            raise LoadError("Format", "tensor %r: offsets [%d, %d) outside the data" % (name, b, e))
        if math.prod(shape) * _SIZES[dtype] != e - b:
            raise LoadError("Format", "tensor %r: %d bytes for shape %s of %s"
                            % (name, e - b, shape, dtype))
        spans.append((b, e, name))
        out[name] = Tensor(dtype, shape, data[b:e])
    spans.sort()
    at = 0
    for b, e, name in spans:
        if b != at:
            raise LoadError("Format", "tensor %r starts at %d, not %d (gap or overlap)"
                            % (name, b, at))
        at = e
    if at != len(data):
        raise LoadError("Format", "the tensors cover %d of %d data bytes" % (at, len(data)))
    return out


def read_file(path: str) -> dict:
    """``parse`` of the whole file, read in one go (read_file, reader.rs)."""
    with open(path, "rb") as f:
        return parse(f.read())


def write(tensors: dict, metadata: dict | None = None) -> bytes:
    """A safetensors buffer of float32 numpy arrays (tests and tools)."""
    header, blobs, at = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name, a in tensors.items():
        a = np.ascontiguousarray(a, dtype=np.float32)
        header[name] = {"dtype": "F32", "shape": list(a.shape),
                        "data_offsets": [at, at + a.nbytes]}
        blobs.append(a.astype("<f4").tobytes())
        at += a.nbytes
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    return struct.pack("<Q", len(h)) + h + b"".join(blobs)


# ------------------------------------------------------------------ inventory

def inventory(cfg, mask_token: bool = True, stored_side: int = 518) -> list:
    """The transformer's tensors of Depth Anything V2 (depth_anything_v2.rs:
    470-590): (name, shape, role) in the checkpoint's names, for a ViTConfig
    ``cfg`` whose position embedding is stored for ``stored_side`` pixels."""
    d, m = cfg.dim, cfg.mlp
    tokens = (stored_side // cfg.patch) ** 2 + 1
    inv = [("backbone.embeddings.cls_token", (1, 1, d), "cls")]
    if mask_token:
        inv.append(("backbone.embeddings.mask_token", (1, d), "mask"))
    inv += [("backbone.embeddings.position_embeddings", (1, tokens, d), "pos"),
            ("backbone.embeddings.patch_embeddings.projection.weight",
             (d, cfg.cin, cfg.patch, cfg.patch), "patch_w"),
            ("backbone.embeddings.patch_embeddings.projection.bias", (d,), "patch_b")]
    parts = [("norm1.weight", (d,), "norm1_g"), ("norm1.bias", (d,), "norm1_b"),
             ("attention.attention.query.weight", (d, d), "q_w"),
             ("attention.attention.query.bias", (d,), "q_b"),
             ("attention.attention.key.weight", (d, d), "k_w"),
             ("attention.attention.key.bias", (d,), "k_b"),
             ("attention.attention.value.weight", (d, d), "v_w"),
             ("attention.attention.value.bias", (d,), "v_b"),
             ("attention.output.dense.weight", (d, d), "proj_w"),
             ("attention.output.dense.bias", (d,), "proj_b"),
             ("layer_scale1.lambda1", (d,), "ls1"),
             ("norm2.weight", (d,), "norm2_g"), ("norm2.bias", (d,), "norm2_b"),
             ("mlp.fc1.weight", (m, d), "fc1_w"), ("mlp.fc1.bias", (m,), "fc1_b"),
             ("mlp.fc2.weight", (d, m), "fc2_w"), ("mlp.fc2.bias", (d,), "fc2_b"),
             ("layer_scale2.lambda1", (d,), "ls2")]
    for layer in range(cfg.layers):
        for suffix, shape, role in parts:
            inv.append(("backbone.encoder.layer.%d.%s" % (layer, suffix), shape,
                        (layer, role)))
    inv += [("backbone.layernorm.weight", (d,), "norm_g"),
            ("backbone.layernorm.bias", (d,), "norm_b")]
    return inv


def check(tensors: dict, inv: list):
    """Inventory::check: every listed tensor present, with its shape and a
    float type; tensors the list does not name are left alone."""
    for name, shape, _ in inv:
        t = tensors.get(name)
        if t is None:
            raise LoadError("Missing", name)
        if tuple(t.shape) != tuple(shape):
            raise LoadError("Shape", "%s is %s, want %s" % (name, tuple(t.shape), tuple(shape)))
        if t.dtype not in ("F32", "F16", "BF16"):
            raise LoadError("Type", "%s is stored as %s" % (name, t.dtype))


# ------------------------------------------------------------------ conversions

_A = np.float32(-0.75)  # Keys' cubic convolution, PyTorch's bicubic A


def _near(x):
    return ((_A + np.float32(2)) * x - (_A + np.float32(3))) * x * x + np.float32(1)


def _far(x):
    return ((_A * x - np.float32(5) * _A) * x + np.float32(8) * _A) * x - np.float32(4) * _A


def _axis(n: int, m: int):
    """Per output sample the 4 clamped source indices and weights along one
    axis of n samples resampled to m (positions.rs:72-96)."""
    ratio = np.float32(n) / np.float32(m)
    out = []
    for o in range(m):
        real = ratio * (np.float32(o) + np.float32(0.5)) - np.float32(0.5)
        i = min(int(math.floor(real)), n - 1)
        t = np.float32(min(max(real - np.float32(i), np.float32(0)), np.float32(1)))
        rest = np.float32(1) - t
        w = (_far(t + np.float32(1)), _near(t), _near(rest), _far(rest + np.float32(1)))
        idx = tuple(min(max(i - 1 + j, 0), n - 1) for j in range(4))
        out.append((idx, w))
    return out


def interpolate_positions(values: np.ndarray, to: tuple) -> np.ndarray:
    """The stored position embedding [rows][C] (class row first, then a
    square grid) with the grid resampled bicubically to ``to`` = (height,
    width), as transformers' Dinov2 interpolate_pos_encoding does through
    torch's bicubic interpolate (align_corners False, A = -0.75, indices
    clamped; width first, then height; f32) (positions.rs:1-144)."""
    values = np.asarray(values, np.float32)
    rows, ch = values.shape
    side = math.isqrt(rows - 1) if rows >= 1 else 0
    if rows < 1 or side * side != rows - 1 or side == 0 or ch == 0 or to[0] <= 0 or to[1] <= 0:
        raise LoadError("Shape", "position embedding of %d rows is not a class row and a "
                        "square grid, or the size %s is empty" % (rows, tuple(to)))
    grid = values[1:].reshape(side, side, ch)
    ys, xs = _axis(side, to[0]), _axis(side, to[1])
    out = np.empty((to[0], to[1], ch), np.float32)
    for oy, (yi, wy) in enumerate(ys):
        for ox, (xi, wx) in enumerate(xs):
            acc = None
            for j in range(4):
                r = grid[yi[j]]
                along = r[xi[0]] * wx[0] + r[xi[1]] * wx[1] + r[xi[2]] * wx[2] + r[xi[3]] * wx[3]
                term = along * wy[j]
                acc = term if acc is None else acc + term
            out[oy, ox] = acc
    return np.concatenate([values[:1], out.reshape(-1, ch)])


def linear(w: np.ndarray) -> np.ndarray:
    """Convert::Linear: a stored [out][in] weight as [in][out]."""
    return np.ascontiguousarray(np.asarray(w, np.float32).T)


def conv(w: np.ndarray) -> np.ndarray:
    """Convert::Conv: a stored [out][in][kh][kw] weight as [kh][kw][in][out]."""
    return np.ascontiguousarray(np.asarray(w, np.float32).transpose(2, 3, 1, 0))


def encoder_weights(source, cfg, stored_side: int = 518) -> dict:
    """The encoder's weight dict (``model.Encoder``'s ``w``) from a
    checkpoint: a path, a safetensors buffer or a parsed dict. Linear weights
    go to [in][out] with Q|K|V side by side, the patch projection to HWIO,
    the position embedding is resampled when ``cfg.side`` differs from the
    side it is stored for."""
    if isinstance(source, str):
        tensors = read_file(source)
    elif isinstance(source, dict):
        tensors = source
    else:
        tensors = parse(source)
    inv = inventory(cfg, mask_token="backbone.embeddings.mask_token" in tensors,
                    stored_side=stored_side)
    check(tensors, inv)
    get = lambda name: tensors[name].to_f32()
    blocks = []
    for layer in range(cfg.layers):
        p = lambda s: get("backbone.encoder.layer.%d.%s" % (layer, s))
        blocks.append({
            "norm1_g": p("norm1.weight"), "norm1_b": p("norm1.bias"),
            "qkv_w": np.concatenate([linear(p("attention.attention.%s.weight" % q))
                                     for q in ("query", "key", "value")], axis=1),
            "qkv_b": np.concatenate([p("attention.attention.%s.bias" % q)
                                     for q in ("query", "key", "value")]),
            "proj_w": linear(p("attention.output.dense.weight")),
            "proj_b": p("attention.output.dense.bias"), "ls1": p("layer_scale1.lambda1"),
            "norm2_g": p("norm2.weight"), "norm2_b": p("norm2.bias"),
            "fc1_w": linear(p("mlp.fc1.weight")), "fc1_b": p("mlp.fc1.bias"),
            "fc2_w": linear(p("mlp.fc2.weight")), "fc2_b": p("mlp.fc2.bias"),
            "ls2": p("layer_scale2.lambda1")})
    pos = get("backbone.embeddings.position_embeddings")[0]
    if pos.shape[0] != cfg.tokens:
        pos = interpolate_positions(pos, (cfg.grid, cfg.grid))
    return {"blocks": blocks,
            "patch_w": conv(get("backbone.embeddings.patch_embeddings.projection.weight")),
            "patch_b": get("backbone.embeddings.patch_embeddings.projection.bias"),
            "cls": get("backbone.embeddings.cls_token").reshape(-1), "pos": pos,
            "norm_g": get("backbone.layernorm.weight"), "norm_b": get("backbone.layernorm.bias")}
