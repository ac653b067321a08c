"""The kernel IR's lowering on CPU (beatlm_b200/graph.py, a restatement of
crates/beatlm-core/src/kernel.rs:1285-1403 Graph::lower / fuse):

* with the reference's rules only, the block graph of the reference's own
  test (kernel.rs:3625-3752: the same tensor ids, shapes and order) lowers as
  that test says (kernel.rs:3796-3844): the 9 fused kernels, their bindings,
  epilogues and lifetimes, and 15 kernels unfused;
* this backend's forms fold the attention chain into one kernel and place
  the LayerNorms as prologues or epilogues, only where the tensor that
  disappears has one consumer and is no graph output;
* malformed graphs are errors;
* the encoder program the model builds from the lowered encoder graph is,
  launch by launch, the program previously listed by hand (argument structs
  compared byte for byte over CPU tensors standing in for device buffers)."""
import ctypes

import numpy as np
import pytest

from beatlm_b200 import graph as G

T, D, HEADS, HD, MLP = 1370, 384, 6, 64, 1536
X, Y = 0, 1


def _block_graph(outputs=(), extra_reader=None):
    """The reference test's encoder block (kernel.rs:3625-3752: weights
    100-108 and 120-124, activations 109-128, input 0, output 1); `outputs`
    makes those activations graph outputs, `extra_reader` gives one tensor a
    second reader (an operation appended at the end)."""
    g = G.Graph()
    g.tensor(X, G.INPUT, T * D)
    w = lambda i, n: g.tensor(i, G.WEIGHT, n)
    g1, b1, wqkv, bqkv = w(100, D), w(101, D), w(102, D * 3 * D), w(103, 3 * D)
    wo, bo, ls1, g2, b2 = w(104, D * D), w(105, D), w(106, D), w(107, D), w(108, D)
    w1, bf1, w2, bf2, ls2 = w(120, D * MLP), w(121, MLP), w(122, MLP * D), w(123, D), w(124, D)

    def act(i, n):
        return g.tensor(i, G.OUTPUT if i in outputs else G.ACTIVATION, n)
    ln = lambda inp, gm, bt: G.LayerNorm(inp, gm, bt, T, D, 1e-6)
    n1 = g.op(ln(X, g1, b1), act(109, T * D))
    qkv = g.op(G.MatMul(n1, wqkv, bqkv, T, D, 3 * D), act(110, T * 3 * D))
    sc = g.op(G.AttentionScores(qkv, T, HEADS, HD), act(111, T * HEADS * T))
    scaled = g.op(G.Scale(sc, 0.125, T * HEADS * T), act(112, T * HEADS * T))
    probs = g.op(G.Softmax(scaled, T * HEADS, T), act(113, T * HEADS * T))
    vals = g.op(G.AttentionValues(probs, qkv, T, HEADS, HD), act(114, T * D))
    proj = g.op(G.MatMul(vals, wo, bo, T, D, D), act(115, T * D))
    l1 = g.op(G.ChannelScale(proj, ls1, T, D), act(116, T * D))
    x1 = g.op(G.Add(l1, X, T * D), act(118, T * D))
    n2 = g.op(ln(x1, g2, b2), act(119, T * D))
    hid = g.op(G.MatMul(n2, w1, bf1, T, D, MLP), act(125, T * MLP))
    a = g.op(G.GeluErf(hid, T * MLP), act(126, T * MLP))
    out = g.op(G.MatMul(a, w2, bf2, T, MLP, D), act(127, T * D))
    l2 = g.op(G.ChannelScale(out, ls2, T, D), act(128, T * D))
    g.tensor(Y, G.OUTPUT, T * D)
    g.op(G.Add(x1, l2, T * D), Y)
    if extra_reader is not None:
        g.tensor(500, G.OUTPUT, g.tensors[extra_reader][1])
        g.op(G.Relu(extra_reader, g.tensors[extra_reader][1]), 500, "extra")
    return g


def test_the_reference_rules_lower_the_block_as_the_reference_test_says():
    g = _block_graph()
    p = g.lower(G.Fusion.ON, forms=(), binding_limit=8)
    assert p.names() == ["layernorm", "matmul", "attention_scores+scale", "softmax",
                         "attention_values", "matmul+channel_scale+add", "layernorm",
                         "matmul+gelu_erf", "matmul+channel_scale+add"]
    # the output projection binds the values, its weights and bias, the
    # LayerScale vector, the residual and its output
    assert p.kernels[5].bindings() == [114, 104, 105, 106, X, 118]
    assert [(e.kind, e.tensor, e.channels) for e in p.kernels[5].epilogue] == [
        ("channel_scale", 106, D), ("add", X, None)]
    assert [(e.kind, e.value) for e in p.kernels[2].epilogue] == [("scale", 0.125)]
    assert [e.kind for e in p.kernels[7].epilogue] == ["gelu_erf"]
    for gone in (111, 115, 116, 125, 127, 128):  # fused intermediates
        assert p.lifetime(gone) is None, gone
    # lifetimes from the kernels (kernel.rs:3846-3858)
    assert p.lifetime(110) == (1, 4) and p.lifetime(112) == (2, 3)
    assert p.lifetime(113) == (3, 4) and p.lifetime(118) == (5, 8) and p.lifetime(X) == (0, 8)
    unfused = g.lower(G.Fusion.OFF)
    assert len(unfused.kernels) == 15
    assert unfused.names()[3] == "map+scale" and unfused.names()[11] == "map+gelu_erf"
    assert unfused.names()[7] == "map+channel_scale"
    assert unfused.kernels[7].bindings() == [115, 106, 116]


def test_the_b200_forms_make_one_attention_kernel_and_place_the_layernorms():
    g = _block_graph()
    p = g.lower(G.Fusion.ON, forms=("attention",))
    assert p.names() == ["layernorm", "matmul", "attention", "matmul+channel_scale+add",
                         "layernorm", "matmul+gelu_erf", "matmul+channel_scale+add"]
    att = p.kernels[2].main
    assert isinstance(att, G.Attention) and att.scale == 0.125 and att.qkv == 110
    assert p.kernels[2].bindings() == [110, 114]
    # no scores, no probabilities; Q|K|V from its projection to the attention
    assert p.lifetime(112) is None and p.lifetime(113) is None and p.lifetime(110) == (1, 2)
    # norm1 reads the block's input, which no kernel writes: it stays a
    # kernel; norm2 reads what the out-projection (a MatMul) writes
    pro = g.lower(G.Fusion.ON, forms=("attention", "ln_prologue"))
    assert pro.names() == ["layernorm", "matmul", "attention", "matmul+channel_scale+add",
                           "layernorm-matmul+gelu_erf", "matmul+channel_scale+add"]
    assert pro.kernels[4].main.a == 118 and pro.lifetime(119) is None
    epi = g.lower(G.Fusion.ON, forms=("attention", "ln_epilogue"))
    assert epi.names() == ["layernorm", "matmul", "attention",
                           "matmul+channel_scale+add+layernorm", "matmul+gelu_erf",
                           "matmul+channel_scale+add"]
    assert epi.kernels[3].writes() == [118, 119] and epi.lifetime(119) == (3, 4)


@pytest.mark.parametrize("tensor,forms,kept", [
    (119, ("attention", "ln_prologue"), "layernorm"),   # norm2's rows are an output
    (119, ("attention", "ln_epilogue"), "layernorm"),
    (112, ("attention",), "softmax"),                   # the scaled scores are an output
    (113, ("attention",), "attention_values"),          # the probabilities are an output
])
def test_no_form_folds_a_graph_output(tensor, forms, kept):
    g = _block_graph(outputs=(tensor,))
    assert kept in g.lower(G.Fusion.ON, forms=forms).names()


@pytest.mark.parametrize("reader,forms,kept", [
    (119, ("attention", "ln_prologue"), "layernorm"),   # norm2's rows read twice
    (119, ("attention", "ln_epilogue"), "layernorm"),
    (113, ("attention",), "softmax"),                   # the probabilities read twice
    (116, (), "map+add"),                               # rule 2: LayerScale output read twice
])
def test_no_form_folds_a_tensor_with_another_reader(reader, forms, kept):
    g = _block_graph(extra_reader=reader)
    names = g.lower(G.Fusion.ON, forms=forms).names()
    assert any(n.startswith(kept) for n in names), names


def test_the_binding_limit_stops_rule_2():
    g = _block_graph()
    # the out-projection with its LayerScale and residual binds 6 tensors
    assert "map+add" in g.lower(G.Fusion.ON, forms=(), binding_limit=5).names()


def test_malformed_graphs_are_errors():
    g = G.Graph()
    g.tensor(0, G.INPUT, 4)
    with pytest.raises(G.GraphError, match="declared twice"):
        g.tensor(0, G.INPUT, 4)
    g.tensor(1, G.ACTIVATION, 4)
    g.tensor(2, G.WEIGHT, 4)
    with pytest.raises(G.GraphError, match="read before"):
        g.op(G.Relu(1, 4), 1)
    with pytest.raises(G.GraphError, match="writes weight"):
        g.op(G.Relu(0, 4), 2)
    g.op(G.Relu(0, 4), 1)
    with pytest.raises(G.GraphError, match="written twice"):
        g.op(G.Relu(0, 4), 1)
    g.tensor(3, G.OUTPUT, 4)
    with pytest.raises(G.GraphError, match="never written"):
        g.lower()
    with pytest.raises(G.GraphError, match="no operations"):
        G.Graph().lower()


def test_the_encoder_graph_lowers_to_the_fused_program():
    from beatlm_b200.model import ViTConfig, encoder_graph, lowering_forms
    cfg = ViTConfig.small()
    g, blocks, maps = encoder_graph(cfg)
    p = g.lower(G.Fusion.ON, lowering_forms(False, cfg.tokens, cfg.dim, 148))
    names = p.names()
    assert names[0] == "patch_embed+prepend_token+add"
    assert names[1:8] == ["layernorm", "matmul", "attention", "matmul+channel_scale+add",
                          "layernorm", "matmul+gelu_erf", "matmul+channel_scale+add"]
    assert names.count("layernorm+tokens_to_map") == 4 and len(names) == 1 + 12 * 7 + 4
    # the embedding's intermediates and every block's scores are gone
    assert p.lifetime(10) is None and p.lifetime(11) is None
    assert all(p.lifetime(b["scores"]) is None for b in blocks)
    # LayerNorm prologues: every block's norm1 but the first (its input comes
    # from the embedding kernel, not a MatMul) and every norm2
    pro = g.lower(G.Fusion.ON, lowering_forms(True, cfg.tokens, cfg.dim, 148))
    assert len(pro.kernels) == 1 + 6 + 11 * 5 + 4
    # LayerNorm epilogues need every column tile resident: not at 8 frames
    assert lowering_forms("epilogue", 8 * cfg.tokens, cfg.dim, 148) == G.B200_FORMS
    epi = g.lower(G.Fusion.ON, lowering_forms("epilogue", cfg.tokens, cfg.dim, 148))
    assert len(epi.kernels) == 1 + 6 + 11 * 5 + 4
    last_fc2 = [k for k in epi.kernels if k.label == "block11.fc2"][0]
    assert last_fc2.name() == "matmul+channel_scale+add"  # nothing after it needs rows


# ----------------------------------------------------- the listed program
# The encoder's kernels as model.py listed them by hand before they were
# generated from the lowered graph, kept as the expected program. In the
# prologue form the listing also had the last block's fc2 write row
# statistics nothing reads; the generated program leaves them out, and so
# does this listing.

def _listed_block(blk, cfg, buf, layer, fused_ln, next_norm, last):
    from beatlm_b200 import ops
    from beatlm_b200.runtime import Spec
    wg = lambda w, **kw: ops.gemm_args(w, weights_static=True, **kw)
    d, name = cfg.dim, "block%d." % layer
    attn = Spec(ops.attention_args(buf.qkv, tokens=buf.tokens, heads=cfg.heads,
                                   head_dim=cfg.head_dim, batch=buf.frames, qk_dtype=blk.dtype,
                                   out=buf.o), name + "attention")
    if fused_ln == "epilogue":
        ep = lambda w: None if w is None else (w[0], w[1], cfg.eps, buf.xn)
        head = ([Spec(ops.layernorm_args(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps, out=buf.xn),
                      name + "norm1")] if layer == 0 else [])
        return head + [
            Spec(wg(blk.qkv_w, a=buf.xn, bias=blk.qkv_b, out=buf.qkv, out_dtype=blk.dtype,
                    out_split=(2 * d, "f16")), name + "qkv"),
            attn,
            Spec(wg(blk.proj_w, a=buf.o, bias=blk.proj_b, chan_scale=blk.ls1, residual=buf.x,
                    out=buf.x, norm=ep(blk.norm2), norm_sync=buf.norm_sync), name + "proj"),
            Spec(wg(blk.fc1_w, a=buf.xn, bias=blk.fc1_b, act="gelu_erf", out=buf.h),
                 name + "fc1"),
            Spec(wg(blk.fc2_w, a=buf.h, bias=blk.fc2_b, chan_scale=blk.ls2, residual=buf.x,
                    out=buf.x, norm=ep(next_norm),
                    norm_sync=buf.norm_sync if next_norm is not None else None), name + "fc2"),
        ]
    stats = (lambda s: s) if fused_ln else (lambda s: None)
    proj = Spec(wg(blk.proj_w, a=buf.o, bias=blk.proj_b, chan_scale=blk.ls1, residual=buf.x,
                   out=buf.x, stats_out=stats(buf.stats2)), name + "proj")
    fc2 = Spec(wg(blk.fc2_w, a=buf.h, bias=blk.fc2_b, chan_scale=blk.ls2, residual=buf.x,
                  out=buf.x, stats_out=None if last else stats(buf.stats1)), name + "fc2")
    if fused_ln:
        if layer == 0:
            head = [Spec(ops.layernorm_args(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps,
                                            out=buf.xn), name + "norm1"),
                    Spec(wg(blk.qkv_w, a=buf.xn, bias=blk.qkv_b, out=buf.qkv, out_dtype=blk.dtype,
                            out_split=(2 * d, "f16")), name + "qkv")]
        else:
            head = [Spec(wg(blk.qkv_w, ln=(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps),
                            ln_stats=buf.stats1, bias=blk.qkv_b, out=buf.qkv,
                            out_dtype=blk.dtype, out_split=(2 * d, "f16")), name + "qkv")]
        return head + [attn, proj,
                       Spec(wg(blk.fc1_w, ln=(buf.x, blk.norm2[0], blk.norm2[1], cfg.eps),
                               ln_stats=buf.stats2, bias=blk.fc1_b, act="gelu_erf",
                               out=buf.h), name + "fc1"), fc2]
    return [
        Spec(ops.layernorm_args(buf.x, blk.norm1[0], blk.norm1[1], cfg.eps, out=buf.xn),
             name + "norm1"),
        Spec(wg(blk.qkv_w, a=buf.xn, bias=blk.qkv_b, out=buf.qkv, out_dtype=blk.dtype,
                out_split=(2 * d, "f16")), name + "qkv"),
        attn, proj,
        Spec(ops.layernorm_args(buf.x, blk.norm2[0], blk.norm2[1], cfg.eps, out=buf.xn),
             name + "norm2"),
        Spec(wg(blk.fc1_w, a=buf.xn, bias=blk.fc1_b, act="gelu_erf", out=buf.h), name + "fc1"),
        fc2,
    ]


def _listed_encoder(enc, frames):
    from beatlm_b200 import ops
    from beatlm_b200.runtime import Spec
    cfg, buf, t = enc.cfg, enc.buffers(frames), enc.cfg.tokens
    out = [Spec(ops.patchify_args(buf.images[0], frames=frames, side=cfg.side, patch=cfg.patch,
                                  cin=cfg.cin, k_pad=cfg.k_pad, a_out=buf.patches,
                                  a_dtype=enc.dtype, cls=enc.cls, pos=enc.pos, x=buf.x),
                "embed.patchify"),
           Spec(ops.gemm_args(enc.patch_w, a=buf.patches, bias=enc.patch_b, residual=enc.pos,
                              res_period=t, out=buf.x, out_row_offset=1, out_group=(t - 1, 1),
                              weights_static=True), "embed.patch")]
    for i in range(cfg.layers):
        nxt = enc.blocks[i + 1].norm1 if i + 1 < cfg.layers else None
        out += _listed_block(enc.blocks[i], cfg, buf, i, enc.fused_ln, nxt, i + 1 == cfg.layers)
        if (i + 1) in cfg.out_indices:
            f = buf.slot_features[0][cfg.out_indices.index(i + 1)]
            out.append(Spec(ops.layernorm_args(buf.x, enc.norm[0], enc.norm[1], cfg.eps, out=f,
                                               in_row_offset=1, in_group=(t - 1, 1)),
                            "features.%d" % (i + 1)))
    return out


def _key(spec):
    return (spec.label, spec.op, spec.parts, ctypes.string_at(ctypes.addressof(spec.args),
                                                              ctypes.sizeof(spec.args)))


def _small_encoder(fused_ln):
    from beatlm_b200.model import Encoder, ViTConfig, block_weights_normal
    cfg = ViTConfig.small(layers=4, out_indices=(2, 4))
    rng = np.random.default_rng(0)
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(cfg.layers)],
         "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
         "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
         "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
    # CPU tensors stand in for device buffers: only their addresses and
    # shapes enter the argument structs
    return Encoder(cfg, w, "bf16", device="cpu", fused_ln=fused_ln, sms=148)


@pytest.mark.parametrize("fused_ln", [False, True, "epilogue"])
def test_the_generated_encoder_program_is_the_listed_one(fused_ln):
    enc = _small_encoder(fused_ln)
    got = [_key(s) for s in enc.specs(1)]
    want = [_key(s) for s in _listed_encoder(enc, 1)]
    assert [g[0] for g in got] == [w_[0] for w_ in want]
    assert got == want
    assert enc.specs_layout(1) == [g[0] for g in got]
    assert enc.launches_per_frame_batch(frames=1) == len(got)


def test_buffer_lifetimes_come_from_the_launches():
    """The memory plan's lifetimes are the launches that bind each buffer:
    the patch matrix lives for the embedding's two launches; each block
    buffer from its first launch to its last; inputs and outputs whole."""
    from beatlm_b200.memory import DeviceProfile
    from beatlm_b200.model import Buffers
    enc = _small_encoder(False)
    _, used = enc._launches(1, None, 1, 0, enc.buffers(1))
    last = len(used) - 1
    assert Buffers.lifetime("patches", used) == (0, 1)
    labels = enc.specs_layout(1)
    assert Buffers.lifetime("qkv", used) == (labels.index("block0.qkv"),
                                             labels.index("block3.attention"))
    assert Buffers.lifetime("h", used) == (labels.index("block0.fc1"), labels.index("block3.fc2"))
    assert Buffers.lifetime("image", used) == (0, last)
    assert Buffers.lifetime("features.2", used) == (0, last)
    plan, _, acts = enc.memory_plan(1, DeviceProfile.webgpu_baseline())
    assert plan.total_bytes() > 0
