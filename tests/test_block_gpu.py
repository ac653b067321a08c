"""One pre-norm ViT block (5 fused launches) and the encoder against the
oracle's forward pass (reference.rs:520-544 vit_block; encoder ops
reference.rs:388-430), mirroring the reference's
one_encoder_block_with_random_weights_matches_the_reference_block
(crates/beatlm-bench/src/vit.rs:240-309): ViT-S shapes (T=1370, D=384, H=6,
MLP=1536), weights by role, input U(-2, 2) from seed 20.

The oracle is given the weights as the device holds them (rounded to the
compute type) and the packed Q|K|V rounded as stored (Q/K compute type, V
f16). The kernels additionally round three GEMM inputs to 16 bits (the
normalised rows, the attention output and the GELU output) that the f32
reference keeps in f32; those roundings are the stated difference. Bound:
relative L2 <= 1e-3 (f16) and <= 4e-3 (bf16) on the block output."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

T, D, H, MLP = 1370, 384, 6, 1536
REL = {"f16": 1e-3, "bf16": 4e-3}


def _rel(got, want):
    got, want = np.asarray(got, np.float64).ravel(), np.asarray(want, np.float64).ravel()
    return float(np.linalg.norm(got - want) / np.linalg.norm(want)), float(
        np.max(np.abs(got - want)))


@pytest.mark.parametrize("fused_ln", [False, True, "epilogue"])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_one_block_matches_the_reference_block(dtype, fused_ln):
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import (Buffers, DeviceBlock, ViTConfig, block_weights_by_role,
                                   run_block)
    cfg = ViTConfig.small()
    w = block_weights_by_role(100, D, MLP, uniform=oracle.uniform)
    x = oracle.uniform(20, T * D, -2.0, 2.0)
    blk = DeviceBlock(w, D, MLP, dtype)
    buf = Buffers(cfg, 1, dtype, features=False)
    buf.x.copy_(torch.from_numpy(x.reshape(T, D)))
    run_block(blk, cfg, buf, fused_ln=fused_ln)
    torch.cuda.synchronize()
    st = bl.status(reset=True)
    assert st.code == 0, hex(st.code)
    got = buf.x.cpu().numpy()
    want = oracle.vit_block(x, DeviceBlock.rounded(w, dtype), T, H, 64, MLP, 1e-6,
                            qkv_round="qk_" + dtype)
    rel, mx = _rel(got, want)
    print("block %s: rel-L2 %.3e max-abs %.3e" % (dtype, rel, mx))
    assert rel <= REL[dtype]


def _encoder_weights(cfg, layers, seed=1):
    rng = np.random.default_rng(seed)
    from beatlm_b200.model import block_weights_normal
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    return {
        "blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(layers)],
        "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
        "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
        "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32),
    }


def imagenet_image(rng, side, frames=1):
    """U[0,1] pixels normalised by the ImageNet mean/std
    (load/depth_anything_v2/reference.rs:58-62), NHWC."""
    mean = np.array([0.485, 0.456, 0.406], np.float32)
    std = np.array([0.229, 0.224, 0.225], np.float32)
    u = rng.random((frames, side, side, 3), dtype=np.float32)
    return ((u - mean) / std).astype(np.float32)


def oracle_encoder(cfg, w, image, layers, dtype):
    """The reference's encoder chain (depth_anything_v2.rs:435-545, evaluated
    as reference.rs:552-625 does) through the oracle, with the image, the
    patch weights and the block weights rounded as the device holds them."""
    from beatlm_b200.model import DeviceBlock
    rnd = oracle.round_bf16 if dtype == "bf16" else oracle.round_f16
    wr = dict(w, patch_w=rnd(w["patch_w"]),
              blocks=[DeviceBlock.rounded(w["blocks"][i], dtype) for i in range(layers)])
    return oracle.encoder_frame(rnd(image), wr, cfg.grid, cfg.patch, cfg.cin, cfg.dim, cfg.heads,
                                cfg.mlp, cfg.eps, cfg.out_indices, layers=layers,
                                qkv_round="qk_" + dtype)


@pytest.mark.parametrize("dtype,fused_ln", [("bf16", False), ("f16", False), ("bf16", True),
                                            ("bf16", "epilogue")])
def test_encoder_features_match_the_reference_chain(dtype, fused_ln):
    """Config-3 shapes (518 px, ViT-S) with 3 blocks and a feature taken after
    blocks 1 and 3, batch 2 frames; also with the LayerNorms fed by the
    statistics of the GEMMs before them."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Encoder, ViTConfig
    layers = 3
    cfg = ViTConfig.small(layers=layers, out_indices=(1, 3))
    w = _encoder_weights(cfg, layers)
    rng = np.random.default_rng(7)
    image = imagenet_image(rng, cfg.side, frames=2)
    enc = Encoder(cfg, w, dtype, fused_ln=fused_ln)
    feats = enc.forward(torch.from_numpy(image).cuda(), frames=2)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    for f in range(2):
        want = oracle_encoder(cfg, w, image[f], layers, dtype)
        for i, ft in enumerate(feats):
            got = ft.cpu().numpy().reshape(2, -1)[f]
            rel, mx = _rel(got, want[i])
            print("encoder %s frame %d feature %d: rel-L2 %.3e max-abs %.3e" % (
                dtype, f, i, rel, mx))
            assert rel <= REL[dtype]


def test_encoder_with_layernorms_in_the_gemm_epilogues_matches_the_reference():
    """One frame (132 column tiles of 32 per GEMM, all resident): proj and
    fc2 write the next LayerNorm's rows from their epilogues. Features after
    blocks 1 and 3 against the oracle chain, and the program has 5 kernels per
    block after the first."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Encoder, ViTConfig
    layers = 3
    cfg = ViTConfig.small(layers=layers, out_indices=(1, 3))
    w = _encoder_weights(cfg, layers, seed=3)
    image = imagenet_image(np.random.default_rng(8), cfg.side, frames=1)
    enc = Encoder(cfg, w, "bf16", fused_ln="epilogue")
    feats = enc.forward(torch.from_numpy(image).cuda(), frames=1)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    assert enc.launches_per_frame_batch(frames=1) == 2 + 6 + 5 + 5 + 2
    want = oracle_encoder(cfg, w, image[0], layers, "bf16")
    for i, ft in enumerate(feats):
        rel, mx = _rel(ft.cpu().numpy().ravel(), want[i])
        print("encoder (epilogue LayerNorm) feature %d: rel-L2 %.3e max-abs %.3e" % (i, rel, mx))
        assert rel <= REL["bf16"]
    # the exchange buffer is left zero-filled for the next launch
    buf = enc.buffers(1)
    ctr = buf.norm_sync[:16 * ((8 * ((buf.rows + 127) // 128) + 15) // 16)]
    assert int(ctr.count_nonzero()) == 0


def test_vit_l_block_matches_the_reference_block():
    """Config-4 block shape: D=1024, 16 heads, MLP 4096, T=1370, bf16, weights
    N(0, 0.02) with gamma 1 / beta 0 / LayerScale 1, input N(0, 1)."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Buffers, DeviceBlock, ViTConfig, block_weights_normal, run_block
    cfg = ViTConfig.large()
    rng = np.random.default_rng(24)
    w = block_weights_normal(rng, cfg.dim, cfg.mlp)
    x = rng.standard_normal(cfg.tokens * cfg.dim, dtype=np.float32)
    blk = DeviceBlock(w, cfg.dim, cfg.mlp, "bf16")
    buf = Buffers(cfg, 1, "bf16", features=False)
    buf.x.copy_(torch.from_numpy(x.reshape(cfg.tokens, cfg.dim)))
    run_block(blk, cfg, buf)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    want = oracle.vit_block(x, DeviceBlock.rounded(w, "bf16"), cfg.tokens, cfg.heads, 64,
                            cfg.mlp, cfg.eps, qkv_round="qk_bf16")
    rel, mx = _rel(buf.x.cpu().numpy(), want)
    print("ViT-L block bf16: rel-L2 %.3e max-abs %.3e" % (rel, mx))
    assert rel <= REL["bf16"]


@pytest.mark.parametrize("side", [518, 266])
def test_encoder_from_a_checkpoint_file_matches_the_reference(side, tmp_path):
    """A safetensors file in the checkpoint's names and layouts (random
    values) through beatlm_b200.load into the encoder: linear weights
    transposed, Q|K|V side by side, the patch projection to HWIO and, at 266
    px, the stored 37 x 37 position grid resampled to 19 x 19. Features
    against the oracle chain fed the converted weights."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200 import load
    from beatlm_b200.model import Encoder, ViTConfig
    layers = 2
    cfg = ViTConfig.small(layers=layers, out_indices=(2,), side=side)
    rng = np.random.default_rng(11)
    ck = {}
    for name, shape, role in load.inventory(cfg):
        r = role[1] if isinstance(role, tuple) else role
        if r in ("norm1_g", "norm2_g", "norm_g"):
            ck[name] = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        elif r in ("ls1", "ls2"):
            ck[name] = rng.uniform(0.1, 1.0, shape).astype(np.float32)
        else:
            ck[name] = (0.02 * rng.standard_normal(shape)).astype(np.float32)
    path = tmp_path / "model.safetensors"
    path.write_bytes(load.write(ck, metadata={"format": "pt"}))
    w = load.encoder_weights(str(path), cfg)
    image = imagenet_image(np.random.default_rng(12), cfg.side, frames=1)
    enc = Encoder(cfg, w, "bf16")
    feats = enc.forward(torch.from_numpy(image).cuda(), frames=1)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    flat = {k: (np.asarray(v).ravel() if k != "blocks" else
                [{bk: np.asarray(bv).ravel() for bk, bv in b.items()} for b in v])
            for k, v in w.items()}
    want = oracle_encoder(cfg, flat, image[0], layers, "bf16")
    rel, mx = _rel(feats[0].cpu().numpy().ravel(), want[0])
    print("encoder from a checkpoint at %d px: rel-L2 %.3e max-abs %.3e" % (side, rel, mx))
    assert rel <= REL["bf16"]


def test_vit_l_encoder_matches_the_reference_chain():
    """Config 4 as benched: the whole 24-block ViT-L/14 encoder at 518 px
    (T=1370, D=1024, 16 heads, MLP 4096), bf16, weights N(0, 0.02) with LN
    gamma 1 / beta 0 / LayerScale 1, one frame through the planned program
    (every tensor in one allocation), against the oracle chain on every host
    core. The four feature maps (after blocks 6, 12, 18 and 24) within the
    bf16 block bound."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Encoder, ViTConfig
    cfg = ViTConfig.large()
    w = _encoder_weights(cfg, cfg.layers, seed=44)
    image = imagenet_image(np.random.default_rng(45), cfg.side, frames=1)
    enc = Encoder(cfg, w, "bf16", planned_frames=1)
    feats = enc.forward(torch.from_numpy(image).cuda(), frames=1)
    torch.cuda.synchronize()
    assert bl.status(reset=True).code == 0
    got = [f.cpu().numpy().ravel() for f in feats]
    want = oracle_encoder(cfg, w, image[0], cfg.layers, "bf16")
    assert len(got) == len(want) == 4
    for i, (g, r) in enumerate(zip(got, want)):
        rel, mx = _rel(g, r)
        print("ViT-L encoder feature after block %d: rel-L2 %.3e max-abs %.3e"
              % (cfg.out_indices[i], rel, mx))
        assert rel <= REL["bf16"]


def test_encoder_forward_on_a_side_stream_equals_the_current_stream():
    """Encoder.forward(stream=s) with s not the current stream: the image
    copy and every kernel run on s, so the result equals a pass on the
    current stream bit for bit."""
    import torch
    from beatlm_b200.model import Encoder, ViTConfig
    cfg = ViTConfig.small(layers=2, out_indices=(2,))
    w = _encoder_weights(cfg, 2, seed=9)
    enc = Encoder(cfg, w, "bf16")
    img = torch.from_numpy(imagenet_image(np.random.default_rng(10), cfg.side)).cuda()
    want = enc.forward(img, frames=1)[0].clone()
    side = torch.cuda.Stream()
    enc.buffers(1).x.fill_(float("nan"))
    torch.cuda.synchronize()
    got = enc.forward(img, frames=1, stream=side)[0]
    side.synchronize()
    assert torch.equal(got, want)
