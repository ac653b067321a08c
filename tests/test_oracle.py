"""The C oracle against the reference's own known-answer tests
(tests/golden/reference_kats.json) and against float64 restatements, on CPU."""
import json
import math
import os

import numpy as np
import pytest

import oracle

KATS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_kats.json")))


def test_layernorm_gives_zero_mean_unit_variance():
    k = KATS["layernorm"]
    out = oracle.layernorm(k["x"], k["gamma"], k["beta"], k["eps"])
    mean = float(np.float32(out.sum()) / np.float32(4))
    var = float(((out - mean) ** 2).sum() / 4)
    assert abs(mean) < k["mean_abs_below"]
    assert abs(var - 1.0) < k["var_minus_one_abs_below"]


def test_matmul_multiplies_and_adds_the_bias_per_column():
    k = KATS["matmul"]
    assert oracle.matmul(k["a"], k["b"], None, 2, 2, 2).tolist() == k["want"]
    assert oracle.matmul(k["a"], k["b"], k["bias"], 2, 2, 2).tolist() == k["want_bias"]


def test_element_wise_operations_compute_what_they_say():
    k = KATS["elementwise"]
    assert oracle.add(k["add"]["a"], k["add"]["b"]).tolist() == k["add"]["want"]
    assert oracle.scale(k["scale"]["x"], k["scale"]["factor"]).tolist() == k["scale"]["want"]


def test_erf_has_its_tabulated_values():
    k = KATS["erf"]
    for x, want in k["points"]:
        assert abs(oracle.erf(x) - want) < k["tolerance"], (x, oracle.erf(x))
    assert oracle.erf(k["exact_one_at"]) == 1.0
    for x in np.linspace(-6, 6, 97):
        assert abs(oracle.erf(float(x)) - math.erf(float(x))) < 1e-13


def test_gelu_erf_reference_values():
    k = KATS["gelu_erf"]
    assert oracle.gelu_erf([0.0])[0] == 0.0
    assert abs(float(oracle.gelu_erf([1.0])[0]) - k["at_one"]) < k["at_one_tolerance"]


def _gelu_erf_as_kernels_compute(x):
    """A&S 7.1.26 in f32 as the GPU epilogue evaluates it (numpy f32)."""
    c = KATS["gelu_erf_constants"]
    p = np.float32(c["p"])
    a1, a2, a3, a4, a5 = (np.float32(v) for v in c["a"])
    x = np.asarray(x, np.float32)
    z = np.abs(x) * np.float32(1.0 / math.sqrt(2.0))
    t = np.float32(1) / (np.float32(1) + p * z)
    poly = t * (a1 + t * (a2 + t * (a3 + t * (a4 + t * a5))))
    q = np.float32(0.5) * poly * np.exp(-z * z)
    return x * np.where(x >= 0, np.float32(1) - q, q)


def test_the_erf_approximation_is_within_its_stated_error():
    grid = (-10.0 + np.arange(81921, dtype=np.float32) / np.float32(4096)).astype(np.float32)
    exact = np.array([0.5 * float(v) * (1.0 + oracle.erf(float(v) / math.sqrt(2.0))) for v in grid])
    worst = np.max(np.abs(_gelu_erf_as_kernels_compute(grid).astype(np.float64) - exact))
    assert worst <= KATS["gelu_erf"]["approximation_max_error"], worst
    # and the oracle's own GELU is the exact one to f32 rounding
    assert np.max(np.abs(oracle.gelu_erf(grid).astype(np.float64) - exact)) < 1e-6


def test_softmax_rows_sum_to_one_and_survive_large_scores():
    k = KATS["softmax"]
    p = oracle.softmax(k["x"], k["cols"])
    assert abs(float(p[:3].sum()) - 1.0) < k["row0_sum_tolerance"]
    assert p[2] > p[1] > p[0]
    assert p[3:].tolist() == k["row1_exact"]


def test_attention_reads_its_head_of_the_packed_rows():
    k = KATS["attention"]
    s = oracle.attention_scores(k["qkv"], k["t"], k["h"], k["d"])
    assert s.tolist() == k["scores"]
    v = oracle.attention_values(k["probs"], k["qkv"], k["t"], k["h"], k["d"])
    assert v.tolist() == k["values"]


def test_patch_embedding_of_one_hot_weights():
    k = KATS["patch_embed"]
    image = np.arange(16, dtype=np.float32)
    w = np.zeros(8, np.float32)
    for i in k["weights_one_at"]:
        w[i] = 1.0
    out = oracle.patch_embed(image, w, k["bias"], k["gh"], k["gw"], k["p"], k["cin"], k["cout"])
    assert out.tolist() == k["want"]
    assert oracle.tokens_to_map(oracle.prepend_token(k["token"], out), 2).tolist() == out.tolist()
    cs = k["channel_scale"]
    assert oracle.channel_scale(cs["x"], cs["s"]).tolist() == cs["want"]


def test_lcg_matches_the_reference_generator():
    k = KATS["lcg"]
    s = 7
    want = []
    for _ in range(5):
        s = (s * k["multiplier"] + k["increment"]) % (1 << 64)
        want.append(np.float32(s >> k["shift"]) / np.float32(1 << 24))
    got = oracle.uniform(7, 5, 0.0, 1.0)
    assert got.tolist() == [float(w) for w in want]
    u = oracle.uniform(3, 1000, -2.0, 2.0)
    assert u.min() >= -2.0 and u.max() < 2.0


def test_normal_draws_have_unit_moments():
    z = oracle.normal(11, 200000)
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1.0) < 0.01


def test_streamed_attention_equals_the_materialised_chain():
    """orc_attention_rows must be the scores -> scale -> softmax -> values chain
    (reference.rs:437-494) bit for bit."""
    t, h, d = 37, 3, 16
    qkv = oracle.normal(5, t * 3 * h * d)
    s = oracle.scale(oracle.attention_scores(qkv, t, h, d), 0.25)
    p = oracle.softmax(s, t)
    want = oracle.attention_values(p, qkv, t, h, d)
    got = oracle.attention(qkv, t, h, d, scale_=0.25)
    assert np.array_equal(got, want)
    part = oracle.attention(qkv, t, h, d, scale_=0.25, rows=(5, 20), heads=(1, 2))
    full = want.reshape(t, h, d)
    assert np.array_equal(part.reshape(15, h, d)[:, 1], full[5:20, 1])
    assert not part.reshape(15, h, d)[:, 0].any()


def test_attention_against_float64_softmax_attention():
    torch = pytest.importorskip("torch")
    t, h, d = 129, 2, 64
    qkv = oracle.normal(9, t * 3 * h * d).reshape(t, 3, h, d)
    got = oracle.attention(qkv, t, h, d).reshape(t, h, d)
    q, k, v = (torch.from_numpy(qkv[:, i].astype(np.float64)).transpose(0, 1) for i in range(3))
    want = torch.softmax(q @ k.transpose(1, 2) * 0.125, -1) @ v
    assert np.allclose(got, want.transpose(0, 1).numpy(), atol=2e-6, rtol=1e-5)


def test_threads_do_not_change_results():
    t, w = 65, 48
    x = oracle.normal(1, t * w)
    b = oracle.normal(2, w * 3 * w)
    one = oracle.matmul(x, b, None, t, w, 3 * w, threads=1)
    many = oracle.matmul(x, b, None, t, w, 3 * w, threads=4)
    assert np.array_equal(one, many)
    qkv = oracle.normal(3, t * 3 * w)
    assert np.array_equal(oracle.attention(qkv, t, 3, 16, threads=1),
                          oracle.attention(qkv, t, 3, 16, threads=3))


def _block_weights(seed, w, mlp):
    """Weights by role as reference vit.rs:203-238 draws them."""
    u = oracle.uniform
    fan = lambda s, n, f: u(s, n, -1 / math.sqrt(f), 1 / math.sqrt(f))
    return {
        "norm1_g": u(seed, w, 0.8, 1.2), "norm1_b": u(seed + 1, w, -0.1, 0.1),
        "qkv_w": fan(seed + 2, w * 3 * w, w), "qkv_b": u(seed + 3, 3 * w, -0.1, 0.1),
        "proj_w": fan(seed + 4, w * w, w), "proj_b": u(seed + 5, w, -0.1, 0.1),
        "ls1": u(seed + 6, w, 0.1, 1.0),
        "norm2_g": u(seed + 7, w, 0.8, 1.2), "norm2_b": u(seed + 8, w, -0.1, 0.1),
        "fc1_w": fan(seed + 9, w * mlp, w), "fc1_b": u(seed + 10, mlp, -0.1, 0.1),
        "fc2_w": fan(seed + 11, mlp * w, mlp), "fc2_b": u(seed + 12, w, -0.1, 0.1),
        "ls2": u(seed + 13, w, 0.1, 1.0),
    }


def test_vit_block_against_float64_restatement():
    torch = pytest.importorskip("torch")
    t, h, d, mlp = 33, 2, 16, 128
    w = h * d
    x = oracle.uniform(20, t * w, -2, 2)
    W = _block_weights(100, w, mlp)
    got = oracle.vit_block(x, W, t, h, d, mlp, 1e-6)
    T = {k: torch.from_numpy(v.astype(np.float64)) for k, v in W.items()}
    X = torch.from_numpy(x.astype(np.float64)).reshape(t, w)
    ln = lambda z, g, b: torch.nn.functional.layer_norm(z, (w,), g, b, 1e-6)
    qkv = ln(X, T["norm1_g"], T["norm1_b"]) @ T["qkv_w"].reshape(w, 3 * w) + T["qkv_b"]
    qkv = qkv.reshape(t, 3, h, d)
    q, k, v = (qkv[:, i].transpose(0, 1) for i in range(3))
    a = (torch.softmax(q @ k.transpose(1, 2) * 0.25, -1) @ v).transpose(0, 1).reshape(t, w)
    x1 = X + T["ls1"] * (a @ T["proj_w"].reshape(w, w) + T["proj_b"])
    hdn = ln(x1, T["norm2_g"], T["norm2_b"]) @ T["fc1_w"].reshape(w, mlp) + T["fc1_b"]
    hdn = torch.nn.functional.gelu(hdn)
    want = x1 + T["ls2"] * (hdn @ T["fc2_w"].reshape(mlp, w) + T["fc2_b"])
    assert np.allclose(got.reshape(t, w), want.numpy(), atol=1e-5, rtol=1e-5)


def test_rounding_helpers():
    x = np.array([1.0, 1.0 + 2 ** -12, 3.14159, -65504.0, 1e-8], np.float32)
    assert oracle.round_f16(x).tolist() == x.astype(np.float16).astype(np.float32).tolist()
    torch = pytest.importorskip("torch")
    assert oracle.round_bf16(x).tolist() == torch.from_numpy(x).bfloat16().float().tolist()
