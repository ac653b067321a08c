"""The static memory plan through the C ABI (host-only, no GPU), mirroring the
reference's planner tests (crates/beatlm-core/src/memory.rs:600-841) case by
case, and checked placement for placement against the Python restatement in
oracle/memory_plan.py on the reference's own generated graphs."""
import pytest

from beatlm_b200.memory import F16, F32, DeviceProfile, MemoryPlan, PlanError, TensorDesc
from oracle import memory_plan as orc


def f32s(n, elements, first, last):
    return TensorDesc(n, F32, elements, first, last)


def baseline():
    return DeviceProfile.webgpu_baseline()


def with_(p, **kw):
    d = dict(max_binding_bytes=p.max_binding_bytes, max_buffer_bytes=p.max_buffer_bytes,
             offset_alignment=p.offset_alignment)
    d.update(kw)
    return DeviceProfile(**d)


def oracle_plan(tensors, profile):
    return orc.plan([(t.id, 4 if t.dtype == F32 else 2, t.elements, t.first_use, t.last_use)
                     for t in tensors],
                    (profile.max_binding_bytes, profile.max_buffer_bytes,
                     profile.offset_alignment))


def plan_both(tensors, profile):
    """The C-ABI plan, after checking that the oracle makes the same one."""
    plan = MemoryPlan(tensors, profile)
    want = oracle_plan(tensors, profile)
    assert not isinstance(want[0], str), want
    arenas, placements, peak = want
    assert plan.arenas() == arenas
    assert {i: (p.arena, p.offset, p.size) for i, p in plan.placements()} == placements
    assert plan.peak_live_bytes() == peak
    return plan


def error_both(tensors, profile):
    with pytest.raises(PlanError) as e:
        MemoryPlan(tensors, profile)
    want = oracle_plan(tensors, profile)
    assert isinstance(want[0], str)
    got = e.value
    assert (got.kind, got.id, got.a, got.b) == want, (got.kind, want)
    return got


class Lcg:
    """The reference tests' generator (memory.rs:524-538): state * 6364136223846793005
    + 1442695040888963407 mod 2^64, output state >> 33."""

    def __init__(self, s):
        self.s = s

    def next(self):
        self.s = (self.s * 6364136223846793005 + 1442695040888963407) & ((1 << 64) - 1)
        return self.s >> 33

    def below(self, bound):
        return self.next() % bound


def random_graph(rng, max_elements):
    """memory.rs:541-556, in the same draw order."""
    count = 1 + rng.below(40)
    ops = 1 + rng.below(30)
    out = []
    for n in range(count):
        first = rng.below(ops)
        last = first + rng.below(ops - first)
        dtype = F32 if rng.below(2) == 0 else F16
        out.append(TensorDesc(n, dtype, 1 + rng.below(max_elements), first, last))
    return out


def random_profile(rng):
    """memory.rs:558-565."""
    align = [4, 16, 64, 256][rng.below(4)]
    binding = 4096 * (1 + rng.below(8))
    return DeviceProfile(binding, binding * 2, align)


def assert_plan_holds(tensors, profile, plan):
    """Rules 1 to 3 and the accessors' consistency (memory.rs:567-598)."""
    alignment, cap = profile.offset_alignment, profile.max_arena_size()
    arenas = plan.arenas()
    for d in tensors:
        p = plan.placement(d.id)
        nbytes = d.elements * (4 if d.dtype == F32 else 2)
        assert p.offset % alignment == 0
        assert p.size % 4 == 0 and nbytes <= p.size < nbytes + 4
        assert p.end() <= arenas[p.arena]
    assert all(a <= cap for a in arenas)
    for i, a in enumerate(tensors):
        for b in tensors[i + 1:]:
            pa, pb = plan.placement(a.id), plan.placement(b.id)
            if a.first_use <= b.last_use and b.first_use <= a.last_use and pa.arena == pb.arena:
                assert pa.end() <= pb.offset or pb.end() <= pa.offset
    assert plan.peak_live_bytes() <= plan.total_bytes()
    assert plan.valid_on(profile)


def test_the_baseline_profile_is_the_webgpu_defaults():
    b = baseline()
    assert (b.max_binding_bytes, b.max_buffer_bytes, b.offset_alignment) == (
        128 << 20, 256 << 20, 256)


def test_disjoint_lifetimes_share_the_same_bytes():
    plan = plan_both([f32s(0, 1024, 0, 1), f32s(1, 1024, 2, 3)], baseline())
    a, b = plan.placement(0), plan.placement(1)
    assert (a.arena, a.offset) == (b.arena, b.offset)
    assert plan.total_bytes() == 4096 and plan.peak_live_bytes() == 4096


def test_lifetimes_are_inclusive_at_both_ends():
    plan = plan_both([f32s(0, 1024, 0, 2), f32s(1, 1024, 2, 4)], baseline())
    a, b = plan.placement(0), plan.placement(1)
    assert a.end() <= b.offset or b.end() <= a.offset
    assert plan.peak_live_bytes() == 8192


def test_overlapping_lifetimes_do_not_share_bytes():
    t = [f32s(0, 100, 0, 5), f32s(1, 50, 3, 8), f32s(2, 70, 4, 4)]
    assert_plan_holds(t, baseline(), plan_both(t, baseline()))


def test_offsets_are_aligned_and_sizes_rounded_to_four_bytes():
    t = [TensorDesc(0, F16, 3, 0, 1), TensorDesc(1, F16, 1, 0, 1)]
    plan = plan_both(t, baseline())
    a, b = plan.placement(0), plan.placement(1)
    assert (a.size, b.size) == (8, 4)
    assert (a.offset, b.offset) == (0, 256)
    assert plan.arenas() == [260]


def test_a_tensor_larger_than_an_arena_is_an_error():
    p = with_(baseline(), max_binding_bytes=1024)
    e = error_both([f32s(0, 256, 0, 0), f32s(1, 257, 0, 0)], p)
    assert (e.kind, e.id, e.a, e.b) == ("TensorTooLarge", 1, 1028, 1024)
    e = error_both([f32s(0, 257, 0, 0)], with_(baseline(), max_buffer_bytes=1024))
    assert e.kind == "TensorTooLarge"


def test_a_tensor_exactly_the_arena_size_fits():
    plan = plan_both([f32s(0, 256, 0, 0)], with_(baseline(), max_binding_bytes=1024))
    assert plan.arenas() == [1024]


def test_a_full_arena_opens_a_new_one():
    p = with_(baseline(), max_binding_bytes=1024)
    t = [f32s(0, 200, 0, 1), f32s(1, 200, 0, 1)]
    plan = plan_both(t, p)
    assert len(plan.arenas()) == 2
    assert plan.placement(0).arena != plan.placement(1).arena
    assert_plan_holds(t, p, plan)


def test_duplicate_ids_are_an_error():
    e = error_both([f32s(7, 4, 0, 0), f32s(7, 8, 1, 1)], baseline())
    assert (e.kind, e.id) == ("DuplicateTensor", 7)


def test_a_first_use_after_the_last_is_an_error():
    e = error_both([f32s(3, 4, 5, 4)], baseline())
    assert (e.kind, e.id, e.a, e.b) == ("InvalidLifetime", 3, 5, 4)


def test_empty_tensors_overflow_and_bad_profiles_are_errors():
    assert error_both([f32s(0, 0, 0, 0)], baseline()).kind == "EmptyTensor"
    assert error_both([f32s(0, (1 << 64) - 1, 0, 0)], baseline()).kind == "SizeOverflow"
    assert error_both([f32s(0, 1, 0, 0)], with_(baseline(), offset_alignment=0)).kind == \
        "InvalidProfile"
    assert error_both([f32s(0, 1, 0, 0)], with_(baseline(), max_buffer_bytes=0)).kind == \
        "InvalidProfile"


def test_no_tensors_is_an_empty_plan():
    plan = plan_both([], baseline())
    assert plan.arenas() == [] and plan.total_bytes() == 0 and plan.peak_live_bytes() == 0
    assert plan.placement(0) is None


def test_the_plan_does_not_depend_on_the_order_tensors_are_listed_in():
    rng = Lcg(7)
    for _ in range(50):
        profile = random_profile(rng)
        tensors = random_graph(rng, 600)
        forward = MemoryPlan(tensors, profile)
        backward = MemoryPlan(list(reversed(tensors)), profile)
        assert forward == backward
        assert forward == MemoryPlan(list(reversed(tensors)), profile)


def test_peak_live_bytes_is_the_most_live_at_one_operation():
    plan = plan_both([f32s(0, 100, 0, 2), f32s(1, 50, 1, 1), f32s(2, 25, 3, 3)], baseline())
    assert plan.peak_live_bytes() == 600


def test_a_chain_of_operations_reuses_memory_down_to_two_activations():
    act = 1 << 20
    plan = plan_both([f32s(n, act, n, n + 1) for n in range(8)], baseline())
    assert plan.peak_live_bytes() == 2 * act * 4
    assert plan.total_bytes() == 2 * act * 4


def test_rules_one_to_three_hold_on_many_generated_graphs():
    """memory.rs:783-812, and each plan equals the oracle's."""
    rng = Lcg(0x5EED)
    multi_arena = reused = too_large = 0
    for _ in range(500):
        profile = random_profile(rng)
        tensors = random_graph(rng, 3000)
        want = oracle_plan(tensors, profile)
        try:
            plan = MemoryPlan(tensors, profile)
        except PlanError as e:
            assert e.kind == "TensorTooLarge" and want[0] == "TensorTooLarge"
            assert (e.id, e.a, e.b) == want[1:]
            too_large += 1
            assert e.a > e.b
            d = next(t for t in tensors if t.id == e.id)
            assert d.elements * (4 if d.dtype == F32 else 2) + 3 >= e.a
            continue
        assert_plan_holds(tensors, profile, plan)
        arenas, placements, peak = want
        assert plan.arenas() == arenas and plan.peak_live_bytes() == peak
        assert {i: (p.arena, p.offset, p.size) for i, p in plan.placements()} == placements
        multi_arena += len(plan.arenas()) > 1
        reused += plan.total_bytes() < sum(p.size for _, p in plan.placements())
    assert multi_arena > 20 and reused > 20 and too_large > 5, (multi_arena, reused, too_large)


def test_rules_one_to_three_hold_on_wide_graphs_against_the_baseline():
    rng = Lcg(99)
    profile = baseline()
    for _ in range(200):
        tensors = random_graph(rng, 1 << 22)
        assert_plan_holds(tensors, profile, plan_both(tensors, profile))


def test_a_baseline_plan_is_valid_on_a_larger_device_but_not_the_reverse():
    on_baseline = MemoryPlan([f32s(0, 1 << 20, 0, 1)], baseline())
    big = DeviceProfile(1 << 30, 1 << 31, 64)
    assert on_baseline.valid_on(big)
    on_big = MemoryPlan([f32s(0, 40 << 20, 0, 1)], big)
    assert not on_big.valid_on(baseline())
    assert not on_baseline.valid_on(with_(baseline(), offset_alignment=512))


def test_the_oracle_pins_the_reference_known_answers():
    """The exact values the reference's tests state, on the oracle alone."""
    b = (128 << 20, 256 << 20, 256)
    arenas, pl, _ = orc.plan([(0, 2, 3, 0, 1), (1, 2, 1, 0, 1)], b)
    assert arenas == [260] and pl == {0: (0, 0, 8), 1: (0, 256, 4)}
    assert orc.plan([(0, 4, 256, 0, 0), (1, 4, 257, 0, 0)], (1024, 256 << 20, 256)) == (
        "TensorTooLarge", 1, 1028, 1024)
    assert orc.plan([(0, 4, 100, 0, 2), (1, 4, 50, 1, 1), (2, 4, 25, 3, 3)], b)[2] == 600


def test_the_encoder_plan_keeps_the_rules_and_reuses_the_patch_matrix():
    """The ViT-S encoder's weights and activation buffers planned against a
    B200-like profile (one arena up to the device's memory): one arena, and
    the patch matrix, dead after the patch GEMM, shares bytes with the block
    scratch born after it."""
    import numpy as np
    from beatlm_b200.model import Encoder, ViTConfig, block_weights_normal
    cfg = ViTConfig.small(layers=2, out_indices=(1, 2))
    rng = np.random.default_rng(3)
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(cfg.layers)],
         "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
         "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
         "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
    enc = Encoder(cfg, w, "bf16", device="cpu")
    plan, wts, acts = enc.memory_plan(1, DeviceProfile(180 << 30, 180 << 30, 256))
    assert len(plan.arenas()) == 1
    # patch_w/b, cls, pos, final norm gamma/beta; 14 per block (two norms, four
    # linear weights and biases, two LayerScales)
    assert len(wts) == 6 + 14 * cfg.layers
    names = [a[0] for a in acts]
    assert "image" in names and "features.1" in names
    ids = {name: k for k, name in enumerate(names, start=len(wts))}
    patches = plan.placement(ids["patches"])
    scratch = [plan.placement(ids[k]) for k in ("qkv", "o", "xn", "h")]
    assert any(not (p.end() <= patches.offset or patches.end() <= p.offset) for p in scratch)
    assert plan.total_bytes() < sum(p.size for _, p in plan.placements())
    assert plan.peak_live_bytes() <= plan.total_bytes()
