"""Real-weight loading (beatlm_b200.load): the safetensors reader's format
checks (reader.rs), the transformer part of Depth Anything V2's inventory
(load/depth_anything_v2.rs:470-590), the layout conversions
(model/mod.rs:272-353) and the position-embedding resampling
(model/positions.rs, with its own cases and torch's bicubic interpolate).
Host only; no GPU."""
import json
import struct

import numpy as np
import pytest

from beatlm_b200 import load
from beatlm_b200.model import ViTConfig


def _checkpoint(cfg, seed=0, stored_side=518, extra=True):
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape, _ in load.inventory(cfg, stored_side=stored_side):
        out[name] = rng.standard_normal(shape).astype(np.float32)
    if extra:  # the DPT neck's tensors, which the encoder does not read
        out["neck.convs.0.weight"] = rng.standard_normal((64, 48, 3, 3)).astype(np.float32)
    return out


# ------------------------------------------------------------ reader

def test_a_written_buffer_reads_back_with_names_types_and_shapes():
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    b = np.array([1.5, -2.0], np.float32)
    t = load.parse(load.write({"a": a, "b": b}, metadata={"format": "pt"}))
    assert set(t) == {"a", "b"}
    assert t["a"].dtype == "F32" and t["a"].shape == (3, 4)
    assert np.array_equal(t["a"].to_f32(), a) and np.array_equal(t["b"].to_f32(), b)


def _raw(header: dict, data: bytes) -> bytes:
    h = json.dumps(header).encode()
    return struct.pack("<Q", len(h)) + h + data


@pytest.mark.parametrize("header,data,what", [
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 12, "cover"),
    ({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8, "bytes for shape"),
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
      "b": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}, b"\0" * 12, "overlap"),
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 16]}}, b"\0" * 8, "outside"),
    ({"a": {"dtype": "Q9", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 8, "dtype"),
    ({"a": {"shape": [2]}}, b"", "malformed"),
])
def test_malformed_files_are_format_errors(header, data, what):
    with pytest.raises(load.LoadError, match=what) as e:
        load.parse(_raw(header, data))
    assert e.value.kind == "Format"


def test_truncated_headers_are_format_errors():
    for buf in (b"\x01\x02", struct.pack("<Q", 1 << 40) + b"{}", struct.pack("<Q", 3) + b"{x}"):
        with pytest.raises(load.LoadError) as e:
            load.parse(buf)
        assert e.value.kind == "Format"


def test_half_and_brain_float_tensors_read_as_f32():
    x = np.array([1.0, -2.5, 0.15625], np.float32)
    h = x.astype("<f2").tobytes()
    bf = (x.view(np.uint32) >> 16).astype("<u2").tobytes()
    hdr = {"h": {"dtype": "F16", "shape": [3], "data_offsets": [0, 6]},
           "b": {"dtype": "BF16", "shape": [3], "data_offsets": [6, 12]}}
    t = load.parse(_raw(hdr, h + bf))
    assert np.array_equal(t["h"].to_f32(), x) and np.array_equal(t["b"].to_f32(), x)


# ------------------------------------------------------------ inventory

def test_the_small_inventory_names_every_transformer_tensor():  # depth_anything_v2.rs:760-790
    cfg = ViTConfig.small()
    inv = {n: s for n, s, _ in load.inventory(cfg)}
    assert len(inv) == 3 + 2 + 12 * 18 + 2
    assert inv["backbone.encoder.layer.11.attention.attention.query.weight"] == (384, 384)
    assert "backbone.encoder.layer.12.norm1.weight" not in inv
    assert inv["backbone.encoder.layer.0.mlp.fc1.weight"] == (1536, 384)
    assert inv["backbone.embeddings.position_embeddings"] == (1, 1370, 384)
    assert inv["backbone.embeddings.patch_embeddings.projection.weight"] == (384, 3, 14, 14)
    assert "backbone.embeddings.mask_token" not in {n for n, _, _ in
                                                    load.inventory(cfg, mask_token=False)}


def test_a_file_that_disagrees_with_the_inventory_is_refused():  # depth_anything_v2.rs:853-890
    cfg = ViTConfig.small(layers=2)
    ck = _checkpoint(cfg)
    gone = dict(ck)
    del gone["backbone.encoder.layer.1.mlp.fc2.weight"]
    with pytest.raises(load.LoadError, match="layer.1.mlp.fc2.weight") as e:
        load.encoder_weights(load.write(gone), cfg)
    assert e.value.kind == "Missing"
    bad = dict(ck)
    bad["backbone.encoder.layer.0.norm1.weight"] = np.zeros(383, np.float32)
    with pytest.raises(load.LoadError) as e:
        load.encoder_weights(load.write(bad), cfg)
    assert e.value.kind == "Shape"
    # the version-5 module names are not what a file of this model holds
    renamed = {k.replace("attention.attention.query", "attention.q_proj"): v for k, v in ck.items()}
    with pytest.raises(load.LoadError) as e:
        load.encoder_weights(load.write(renamed), cfg)
    assert e.value.kind == "Missing"


# ------------------------------------------------------------ conversions

def test_checkpoint_layouts_become_the_encoder_layouts():  # model/mod.rs:272-353
    cfg = ViTConfig.small(layers=2)
    ck = _checkpoint(cfg)
    w = load.encoder_weights(load.write(ck), cfg)
    b1 = w["blocks"][1]
    L = "backbone.encoder.layer.1."
    q, k, v = (ck[L + "attention.attention.%s.weight" % s] for s in ("query", "key", "value"))
    assert b1["qkv_w"].shape == (384, 1152)
    assert np.array_equal(b1["qkv_w"], np.concatenate([q.T, k.T, v.T], axis=1))
    assert np.array_equal(b1["qkv_b"][384:768], ck[L + "attention.attention.key.bias"])
    assert np.array_equal(b1["fc1_w"], ck[L + "mlp.fc1.weight"].T)
    assert np.array_equal(b1["fc2_w"], ck[L + "mlp.fc2.weight"].T)
    assert np.array_equal(b1["ls2"], ck[L + "layer_scale2.lambda1"])
    pw = ck["backbone.embeddings.patch_embeddings.projection.weight"]  # [o][i][y][x]
    assert w["patch_w"].shape == (14, 14, 3, 384)
    assert w["patch_w"][5, 7, 2, 100] == pw[100, 2, 5, 7]
    assert np.array_equal(w["pos"], ck["backbone.embeddings.position_embeddings"][0])
    assert np.array_equal(w["cls"], ck["backbone.embeddings.cls_token"].reshape(-1))


def test_another_image_side_resamples_the_stored_positions():
    cfg = ViTConfig.small(layers=1, side=266)  # 19 x 19 patches
    ck = _checkpoint(cfg, stored_side=518)
    w = load.encoder_weights(load.write(ck), cfg)
    assert w["pos"].shape == (19 * 19 + 1, 384)
    assert np.array_equal(w["pos"][0], ck["backbone.embeddings.position_embeddings"][0, 0])


# ------------------------------------------------------------ positions

def test_the_weights_are_keys_cubic_with_a_of_minus_three_quarters():  # positions.rs:150
    halved = load._axis(4, 2)
    assert halved[0][0] == (0, 0, 1, 2)
    assert [float(x) for x in halved[0][1]] == [-0.09375, 0.59375, 0.59375, -0.09375]
    assert halved[1][0] == (1, 2, 3, 3)
    doubled = load._axis(2, 4)
    assert doubled[0][0] == (0, 0, 0, 1)
    t = np.float32(0.75)
    assert [float(x) for x in doubled[0][1]] == [float(load._far(t + np.float32(1))),
                                                 float(load._near(t)),
                                                 float(load._near(np.float32(1) - t)),
                                                 float(load._far(np.float32(2) - t))]
    for _, w in halved + doubled:
        assert abs(sum(float(x) for x in w) - 1.0) < 1e-6


def test_the_same_size_is_the_identity_and_a_constant_stays_constant():  # positions.rs:175
    grid = (np.arange(3 * 3 * 2, dtype=np.float32) * 0.25 - 1.0).reshape(9, 2)
    vals = np.concatenate([np.zeros((1, 2), np.float32), grid])
    assert np.array_equal(load.interpolate_positions(vals, (3, 3)), vals)
    flat = np.full((26, 3), 1.5, np.float32)
    for to in [(2, 2), (7, 7), (3, 6)]:
        out = load.interpolate_positions(flat, to)
        assert out.shape == (1 + to[0] * to[1], 3)
        assert np.all(np.abs(out[1:] - 1.5) < 1e-5), to


def test_a_two_by_two_grid_halved_is_the_mean_of_its_four_positions():  # positions.rs:189
    values = np.array([9, -9, 1, 10, 2, 20, 3, 30, 4, 40], np.float32).reshape(5, 2)
    out = load.interpolate_positions(values, (1, 1))
    assert list(out[0]) == [9.0, -9.0]
    assert abs(out[1, 0] - 2.5) < 1e-6 and abs(out[1, 1] - 25.0) < 1e-5


def test_halving_a_row_weights_its_neighbours_by_the_cubic():  # positions.rs:199
    grid = np.array([i % 4 for i in range(16)], np.float32).reshape(16, 1)
    vals = np.concatenate([np.zeros((1, 1), np.float32), grid])
    out = load.interpolate_positions(vals, (2, 2))[1:, 0]
    want0 = 0.59375 - 0.09375 * 2.0
    assert abs(out[0] - want0) < 1e-6 and abs(out[2] - want0) < 1e-6


def test_a_grid_that_is_not_square_is_refused():  # positions.rs:210
    for vals, to in [(np.zeros((4, 1)), (2, 2)), (np.zeros((5, 1)), (0, 2))]:
        with pytest.raises(load.LoadError):
            load.interpolate_positions(vals, to)


@pytest.mark.parametrize("to", [(19, 19), (37, 37), (74, 74), (10, 23)])
def test_resampling_matches_torch_bicubic_interpolate(to):
    import torch
    rng = np.random.default_rng(5)
    g, c = 37, 8
    vals = rng.standard_normal((1 + g * g, c)).astype(np.float32)
    got = load.interpolate_positions(vals, to)
    grid = torch.from_numpy(vals[1:].reshape(g, g, c)).permute(2, 0, 1)[None]
    want = torch.nn.functional.interpolate(grid, size=to, mode="bicubic", align_corners=False)
    want = want[0].permute(1, 2, 0).reshape(-1, c).numpy()
    assert np.allclose(got[1:], want, rtol=1e-5, atol=1e-5)
    assert np.array_equal(got[0], vals[0])
