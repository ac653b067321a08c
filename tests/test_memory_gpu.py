"""The plan realised on the device: ONE allocation for every arena, bindings
inside it, host writes and reads, the reference's binding errors
(arenas.rs:131-160 and its test one_buffer_per_arena_is_created_and_
placements_bind_inside_it, arenas.rs:183-199), and the encoder run from its
planned arena giving the same features as the separately allocated one."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _plan():
    from beatlm_b200.memory import F32, DeviceProfile, MemoryPlan, TensorDesc
    t = [TensorDesc(0, F32, 1000, 0, 1), TensorDesc(1, F32, 1000, 1, 2),
         TensorDesc(2, F32, 1000, 3, 4)]
    return MemoryPlan(t, DeviceProfile.webgpu_baseline())


def test_one_allocation_holds_every_arena_and_placements_bind_inside_it():
    from beatlm_b200.memory import F32, Arenas, DeviceProfile, MemoryPlan, TensorDesc
    p = DeviceProfile(4096, 8192, 256)  # small arenas: force several
    plan = MemoryPlan([TensorDesc(i, F32, 700, 0, 1) for i in range(4)], p)
    assert len(plan.arenas()) > 1
    a = Arenas(plan)
    bases = [a.buffer(i) for i in range(len(plan.arenas()))]
    assert all(b % 256 == 0 for b in bases)
    assert a.bytes() >= plan.total_bytes()
    assert bases[-1] + plan.arenas()[-1] <= bases[0] + a.bytes()  # one contiguous allocation
    for _, pl in plan.placements():
        assert a.binding(pl) == bases[pl.arena] + pl.offset


def test_host_writes_and_reads_round_trip_through_placements():
    import torch
    from beatlm_b200.memory import Arenas
    plan = _plan()
    a = Arenas(plan)
    for i, pl in plan.placements():
        src = np.arange(1000, dtype=np.float32) * (i + 1)
        a.write(pl, src)
        dst = np.zeros(1000, np.float32)
        a.read(pl, dst)
        torch.cuda.synchronize()
        assert np.array_equal(src, dst)
        assert torch.equal(a.tensor(pl, (1000,), "f32").cpu(), torch.from_numpy(src))


def test_bindings_from_another_plan_are_errors():
    import beatlm_b200 as bl
    from beatlm_b200.memory import Arenas, Placement
    plan = _plan()
    a = Arenas(plan)
    size = plan.arenas()[0]
    with pytest.raises(bl.BackendError, match="does not exist"):
        a.binding(Placement(5, 0, 4))
    with pytest.raises(bl.BackendError, match="inside its arena"):
        a.binding(Placement(0, size - 4, 8))
    with pytest.raises(bl.BackendError, match="inside its arena"):
        a.binding(Placement(0, 0, 0))
    with pytest.raises(bl.BackendError, match="aligned"):
        a.binding(Placement(0, 4, 4))
    with pytest.raises(bl.BackendError, match="pass the end"):
        a.write(Placement(0, 0, 16), np.zeros(8, np.float32))


def test_the_planned_encoder_matches_the_separately_allocated_one():
    """Same kernels on the same inputs: bit-identical features; and the
    forward pass allocates nothing (torch's allocator does not grow)."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Encoder, ViTConfig
    from test_block_gpu import _encoder_weights, imagenet_image
    cfg = ViTConfig.small(layers=3, out_indices=(1, 3))
    w = _encoder_weights(cfg, 3)
    image = torch.from_numpy(imagenet_image(np.random.default_rng(4), cfg.side)).cuda()
    ref = [f.clone() for f in Encoder(cfg, w, "bf16").forward(image)]
    enc = Encoder(cfg, w, "bf16", planned_frames=1)
    assert enc.arena.bytes() <= enc.plan.total_bytes() + 256 * len(enc.plan.arenas())
    enc.forward(image)  # builds the program once
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    feats = enc.forward(image)
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == before
    assert bl.status(reset=True).code == 0
    for got, want in zip(feats, ref):
        assert torch.equal(got, want)
    with pytest.raises(ValueError, match="planned"):
        enc.buffers(2)


def test_the_plan_lands_on_the_current_device():
    """One process per GPU sets its device first; "cuda" then means that
    device for the single allocation too (checked without launching work)."""
    import torch
    from beatlm_b200.memory import Arenas
    from beatlm_b200.model import Encoder, ViTConfig
    from test_block_gpu import _encoder_weights
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with torch.cuda.device(1):
        assert Arenas(_plan()).device == 1
        cfg = ViTConfig.small(layers=1, out_indices=(1,))
        enc = Encoder(cfg, _encoder_weights(cfg, 1), "bf16", planned_frames=1)
        assert enc.arena.device == 1
        assert enc.buffers(1).x.device == torch.device("cuda", 1)
        assert enc.blocks[0].qkv_w.device == torch.device("cuda", 1)
