"""Programs of prebuilt launches on the GPU: split parts equal the whole
kernel (Program::split, kernel.rs:2384-2408, rule 6), a captured CUDA graph
equals direct encoding, and the cudaEvent slice timer keeps the reference
SliceTimer's rules (crates/beatlm/src/gpu/timer.rs:185-470)."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

T, D, MLP = 1370, 384, 1536


def _block(dtype="bf16", frames=1):
    import torch
    from beatlm_b200.model import Buffers, DeviceBlock, ViTConfig, block_weights_by_role
    cfg = ViTConfig.small()
    w = block_weights_by_role(100, D, MLP, uniform=oracle.uniform)
    blk = DeviceBlock(w, D, MLP, dtype)
    buf = Buffers(cfg, frames, dtype, features=False)
    x0 = torch.from_numpy(oracle.uniform(20, frames * T * D, -2, 2).reshape(frames * T, D)).cuda()
    return cfg, blk, buf, x0


@pytest.mark.parametrize("parts", [3, 11, 200])
def test_split_block_equals_the_whole_block(parts):
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import block_specs
    from beatlm_b200.runtime import Kernels
    cfg, blk, buf, x0 = _block(frames=2)
    whole = Kernels(block_specs(blk, cfg, buf))
    split = Kernels(block_specs(blk, cfg, buf, parts=parts))
    assert len(whole) == 7
    assert len(split) > 7
    assert split.label(0).startswith("block0.norm1 [1/")
    buf.x.copy_(x0)
    whole.encode_all()
    torch.cuda.synchronize()
    want = buf.x.clone()
    buf.x.copy_(x0)
    split.encode_all()
    torch.cuda.synchronize()
    assert torch.equal(buf.x, want)
    assert bl.status(reset=True).code == 0


def test_graph_replay_equals_direct_encoding():
    import torch
    from beatlm_b200.model import block_specs
    from beatlm_b200.runtime import Kernels
    cfg, blk, buf, x0 = _block()
    k = Kernels(block_specs(blk, cfg, buf))
    buf.x.copy_(x0)
    k.encode_all()
    torch.cuda.synchronize()
    want = buf.x.clone()
    s = torch.cuda.Stream()
    g = k.capture(s)
    buf.x.copy_(x0)
    torch.cuda.synchronize()
    g.launch(s)
    s.synchronize()
    assert torch.equal(buf.x, want)


def test_slice_timer_rules():
    import torch
    from beatlm_b200.model import block_specs
    from beatlm_b200.runtime import Kernels, SliceTimer
    cfg, blk, buf, x0 = _block()
    k = Kernels(block_specs(blk, cfg, buf))
    t = SliceTimer(max_slices=8)
    s = torch.cuda.current_stream()
    handles = []
    for frame in range(3):
        h = t.begin_frame(frame)
        assert h >= 0
        k.encode_all(s, timer=t, frame=h)
        t.submitted(h)
        handles.append(h)
    # every slot is in flight: the fourth frame goes untimed, counted
    assert t.begin_frame(3) == -1
    k.encode_all(s, timer=None)
    t.submitted(-1)
    assert t.stats()["frames_skipped"] == 1
    torch.cuda.synchronize()
    got = t.collect_ready()
    assert [f.frame for f in got] == [0, 1, 2]           # submission order
    for f in got:
        assert [kernel for kernel, _ in f.compute] == [0, 1, 2, 3, 4, 5, 6]
        assert all(us > 0 for _, us in f.compute)
        assert f.begin_us[0] == 0.0 and f.begin_us == sorted(f.begin_us)
    assert t.stats()["frames_collected"] == 3
    assert t.in_flight() == 0

    # a dropped frame is never read; an invalidated one is counted failed
    h = t.begin_frame(10)
    k.encode(0, s, timer=t, frame=h)
    t.drop(h)
    h = t.begin_frame(11)
    k.encode(1, s, timer=t, frame=h)
    t.submitted(h)
    assert t.invalidate_submitted() == 1
    torch.cuda.synchronize()
    assert t.collect_ready() == []
    assert t.stats()["frames_failed"] == 1

    # a held frame holds back later frames until it is settled
    h1 = t.begin_frame(20)
    k.encode(2, s, timer=t, frame=h1)
    t.submitted_held(h1)
    h2 = t.begin_frame(21)
    k.encode(3, s, timer=t, frame=h2)
    t.submitted(h2)
    torch.cuda.synchronize()
    assert t.collect_ready() == []
    t.settle(h1, accept=False)
    got = t.collect_ready()
    assert [f.frame for f in got] == [21]
    assert t.stats()["frames_failed"] == 2

    # more timed passes than the timer holds is an error, not a guess
    small = SliceTimer(max_slices=2)
    h = small.begin_frame(0)
    import beatlm_b200 as bl
    with pytest.raises(bl.BackendError, match="timed passes"):
        k.encode_all(s, timer=small, frame=h)


def test_encoder_program_graph_equals_direct():
    import torch
    from beatlm_b200.model import Encoder, ViTConfig
    from test_block_gpu import _encoder_weights, imagenet_image
    cfg = ViTConfig.small(layers=2, out_indices=(2,))
    enc = Encoder(cfg, _encoder_weights(cfg, 2), "bf16")
    image = torch.from_numpy(imagenet_image(np.random.default_rng(3), cfg.side)).cuda()
    feats = enc.forward(image, frames=1)
    torch.cuda.synchronize()
    want = feats[0].clone()
    prog = enc.program(1)
    assert len(prog) == enc.launches_per_frame_batch()  # one launch record per launch
    s = torch.cuda.Stream()
    g = prog.capture(s)
    enc.buffers(1).features[0].zero_()
    torch.cuda.synchronize()
    g.launch(s)
    s.synchronize()
    assert torch.equal(enc.buffers(1).features[0], want)


def test_host_to_host_graph_equals_the_device_features():
    """Encoder.capture_host: the image copied in, the program, each feature
    copied out on a second stream right after its LayerNorm, in one graph;
    two replays with different images each give that image's features."""
    import torch
    from beatlm_b200.model import Encoder, ViTConfig
    from test_block_gpu import _encoder_weights, imagenet_image
    cfg = ViTConfig.small(layers=3, out_indices=(1, 3))
    enc = Encoder(cfg, _encoder_weights(cfg, 3), "bf16")
    images = [imagenet_image(np.random.default_rng(40 + i), cfg.side) for i in range(2)]
    wants = []
    for im in images:
        feats = enc.forward(torch.from_numpy(im).cuda(), frames=1)
        torch.cuda.synchronize()
        wants.append([f.cpu().clone() for f in feats])
    host_image = torch.empty((1, cfg.side, cfg.side, cfg.cin), dtype=torch.float32).pin_memory()
    host_feats = [torch.empty(f.shape, dtype=f.dtype).pin_memory() for f in enc.features(1)]
    s = torch.cuda.Stream()
    g = enc.capture_host(1, host_image, host_feats, s)
    for im, want in zip(images, wants):
        host_image.copy_(torch.from_numpy(im).reshape(host_image.shape))
        with torch.cuda.stream(s):
            g.replay()
        s.synchronize()
        for h, w in zip(host_feats, want):
            assert torch.equal(h, w)


def test_the_loop_feeds_timer_measurements_into_the_cost_model():
    """North star (c): the scheduler's slice costs come from cudaEvent timings.
    Each collected frame folds every pass under its kernel index; a frame
    planned once its slices were warm records its measured-over-planned
    ratio (cost.rs:863-870)."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.cost import CostModel, FrameScaled, Measured, WARM_SAMPLES
    from beatlm_b200.model import block_specs
    from beatlm_b200.runtime import Kernels, SliceTimer
    cfg, blk, buf, x0 = _block()
    k = Kernels(block_specs(blk, cfg, buf))
    t = SliceTimer(max_slices=len(k))
    m = CostModel(1000, FrameScaled(8, 2, 0.9))
    buf.x.copy_(x0)
    planned, done = {}, 0
    for f in range(12):
        planned[f] = m.plan_frame(range(len(k)))
        h = t.begin_frame(f)
        k.encode_all(timer=t, frame=h)
        t.submitted(h)
        torch.cuda.synchronize()
        for timing in t.collect_ready():
            assert [kern for kern, _ in timing.compute] == list(range(len(k)))
            m.record_timing(timing, planned=planned.pop(timing.frame))
            done += 1
    assert done == 12
    for s in range(len(k)):
        assert m.samples(s) == 12 and 1 <= m.estimate(s) < 1000
    # frames WARM_SAMPLES.. had a plan: their ratios fill the 2-frame window
    assert isinstance(m.frame_scale(), Measured)
    assert m.frames_recorded() == 12 - WARM_SAMPLES
    assert bl.status(reset=True).code == 0


def test_calibration_splits_by_measured_durations_and_seeds_the_cost_model():
    """calibrate.rs:105-186 on the ViT-S block: pass 1 times whole kernels,
    Program::parts_within splits each for its median, pass 2 times every
    part into the cost model as calibration's measurements."""
    import beatlm_b200 as bl
    from beatlm_b200.calibration import calibrate
    from beatlm_b200.cost import WindowedQuantile
    from beatlm_b200.model import block_specs
    from beatlm_b200.runtime import Kernels, program_parts_within
    cfg, blk, buf, x0 = _block()
    specs = block_specs(blk, cfg, buf)
    buf.x.copy_(x0)
    frames, bound = 8, 4
    cal = calibrate(specs, bound, frames=frames, period_us=2000,
                    estimator=WindowedQuantile(32, 0.9))
    assert len(cal.durations) == len(specs) and all(d >= 1 for d in cal.durations)
    assert cal.parts == program_parts_within(specs, cal.durations, bound)
    assert max(cal.parts) > 1  # the attention alone takes well over 4 us
    split = Kernels(cal.specs)
    assert len(split) == sum(cal.parts)
    for part in range(len(split)):
        assert cal.cost.samples(part) == frames // 2 and cal.cost.estimate(part) >= 1
    assert bl.status(reset=True).code == 0


@pytest.mark.parametrize("kernels", ["trivial", "block"])
def test_pass_cost_frames_time_every_variant(kernels):
    """pass_cost.rs's workload with CUDA launches as passes: every cell is
    timed, spans grow with the pass count, and only A and D carry pairs per
    launch."""
    import beatlm_b200 as bl
    from beatlm_b200.model import block_specs
    from beatlm_b200.pass_cost import DEFAULT_VARIANTS, derive, run
    from beatlm_b200.runtime import Kernels
    program = None
    if kernels == "block":
        cfg, blk, buf, x0 = _block()
        buf.x.copy_(x0)
        program = Kernels(block_specs(blk, cfg, buf))
    passes = (1, 7) if program is not None else (1, 8)
    res = run(passes, DEFAULT_VARIANTS, frames_per_cell=4, period_us=0, kernels=program)
    for (name, p), frames in res.items():
        assert len(frames) == 4
        for f in frames:
            assert f.span_us > 0 and f.encode_us > 0
            want = {"per-pass": p, "ends": 1, "one-pass": 1, "one-pass-pdl": 1,
                    "every:8": len([i for i in range(p) if i % 8 == 0 or i == p - 1])}[name]
            assert f.pairs == want, (name, p)
            if name == "per-pass":
                assert f.passes_us <= f.span_us + 1.0
    d = derive(res, trivial=program is None)
    big = passes[-1]
    assert d["span_us"]["[per-pass,%d]" % big] > d["span_us"]["[per-pass,1]"]
    assert "over_one_pass_us" in d["derived"]["[per-pass,%d]" % big]
    assert bl.status(reset=True).code == 0


def test_the_frame_loop_schedules_timed_slices_and_learns_their_costs():
    """North star (c) end to end: the scheduler plans each frame of the split
    ViT-S block with the cost model, the planned slices run under the
    cudaEvent slice timer, and their measured durations come back into the
    model. With a budget every job fits, every job is delivered on its frame
    (latency 2), and the residual stream equals the block run once per job."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.cost import CostModel
    from beatlm_b200.model import block_specs
    from beatlm_b200.runtime import Kernels, SliceTimer
    from beatlm_b200.schedule import FixedLatency, FrameInfo, FrameLoop, Scheduler
    cfg, blk, buf, x0 = _block()
    k = Kernels(block_specs(blk, cfg, buf, parts=3))
    n = len(k)
    loop = FrameLoop(k, Scheduler(FixedLatency(2), "hold_previous", 5000), CostModel(50),
                     SliceTimer(max_slices=n))
    buf.x.copy_(x0)
    jobs, delivered = 0, []
    for i in range(12):
        submit = i % 2 == 0 and i < 10
        jobs += submit
        p = loop.tick(FrameInfo(i, i * 16667, 16667), 5000, submit)
        torch.cuda.synchronize()
        assert p.spent_estimate <= p.budget and not p.missed, i
        delivered += [(i, d.job) for d in p.delivered]
    loop.collect()
    assert delivered == [(2 * j + 2, j) for j in range(jobs)]
    for s in range(n):
        assert loop.cost.samples(s) >= jobs - 1 and loop.cost.estimate(s) != 50
    got = buf.x.clone()
    buf.x.copy_(x0)
    for _ in range(jobs):
        k.encode_all()
    torch.cuda.synchronize()
    assert torch.equal(got, buf.x)
    assert bl.status(reset=True).code == 0


def test_jobs_in_flight_keep_their_own_input_and_output_slots():
    """The reference's Net slots (crates/beatlm-host/src/slots.rs:1-60) on
    the encoder, bound as binding sets of one program: three slots for
    latency 2, each job a different image, a
    budget of three quarters of a job per frame, so a job spreads over two
    frames and the next one's input is written while it still runs. Every delivered job's features equal a direct
    forward pass of its own image."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.cost import CostModel
    from beatlm_b200.model import Encoder, ViTConfig, block_weights_normal
    from beatlm_b200.runtime import SliceTimer
    from beatlm_b200.schedule import FixedLatency, FrameInfo, FrameLoop, Scheduler, max_in_flight
    cfg = ViTConfig.small(layers=2, out_indices=(2,))
    rng = np.random.default_rng(21)
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(2)],
         "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
         "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
         "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
    policy = FixedLatency(2)
    slots = max_in_flight(policy)
    enc = Encoder(cfg, w, "bf16", planned_frames=1, slots=slots)
    images = [torch.from_numpy(rng.random((1, cfg.side, cfg.side, cfg.cin), dtype=np.float32))
              .cuda() for _ in range(6)]
    want = []
    for img in images:  # direct passes, slot 0
        want.append(enc.forward(img, frames=1)[0].clone())
    torch.cuda.synchronize()
    buf = enc.buffers(1)
    program = enc.program(1)
    assert program.sets == slots
    # only the kernels that read the image or write a feature map get a
    # launch per slot: patchify and the feature LayerNorm here
    assert program.launches == len(program) + (slots - 1) * 2
    programs = [program]
    # measured costs first, so the budget below splits a job over two frames
    cost = CostModel(1)
    loop = FrameLoop(program, Scheduler(policy, "hold_previous", 0), cost,
                     SliceTimer(max_slices=2 * len(programs[0])))
    per_job = None
    got, submitted = {}, [0]

    def write(slot):
        buf.images[slot].copy_(images[submitted[0]])

    for i in range(20):
        submit = i % 2 == 0 and submitted[0] < len(images) and i >= 2
        if i < 2:  # two warm-up jobs to measure every slice
            loop.scheduler.set_expected_budget(10 ** 6)
            loop.tick(FrameInfo(i, i * 16667, 16667), 10 ** 6, True, write_input=write)
            torch.cuda.synchronize()
            loop.collect()
            continue
        if per_job is None:
            per_job = sum(cost.planning_estimate(s) for s in range(len(programs[0])))
            loop.scheduler.set_expected_budget(per_job * 3 // 4 + 1)
        p = loop.tick(FrameInfo(i, i * 16667, 16667), per_job * 3 // 4 + 1, submit,
                      write_input=write if submit else None)
        if submit:
            submitted[0] += 1
        torch.cuda.synchronize()
        assert not p.missed, (i, p.missed)
        for d in p.delivered:
            if d.job >= 2:
                slot = loop.slot_of(d.job)
                got[d.job - 2] = buf.slot_features[slot][0].clone()
    assert sorted(got) == list(range(len(images)))
    for j, f in got.items():
        assert torch.equal(f, want[j]), j
    assert bl.status(reset=True).code == 0


def test_host_pipeline_frames_equal_direct_passes():
    """Encoder.host_pipeline: frames from pinned host memory to pinned host
    memory over two slots, each frame's image copied in beside the previous
    frame's pass and its feature maps copied out inside its own. Six frames,
    each a different image written by the fill callback: every frame's host
    features equal a direct pass over its image, bit for bit, and nothing
    records a device error."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Encoder, ViTConfig, block_weights_normal
    cfg = ViTConfig.small(layers=2, out_indices=(1, 2))
    rng = np.random.default_rng(23)
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(2)],
         "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
         "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
         "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
    enc = Encoder(cfg, w, "bf16", planned_frames=1, slots=2)
    images = [rng.random((1, cfg.side, cfg.side, cfg.cin), dtype=np.float32) for _ in range(6)]
    want = [[f.cpu().clone() for f in enc.forward(torch.from_numpy(img).cuda(), frames=1)]
            for img in images]
    torch.cuda.synchronize()
    hosts = [torch.empty((1, cfg.side, cfg.side, cfg.cin)).pin_memory() for _ in range(2)]
    feats = [[torch.empty(f.shape, dtype=f.dtype).pin_memory() for f in enc.features(1)]
             for _ in range(2)]
    pipe = enc.host_pipeline(1, hosts, feats)
    fed = [0]

    def fill(slot):  # the next frame's pixels into that slot's host buffer
        if fed[0] < len(images):
            hosts[slot].copy_(torch.from_numpy(images[fed[0]]))
        fed[0] += 1

    stream = torch.cuda.Stream()
    got = []
    for k in range(len(images)):
        slot = pipe.step(stream, fill)
        stream.synchronize()
        got.append([f.clone() for f in feats[slot]])
    assert bl.status(reset=True).code == 0
    for k in range(len(images)):
        for g, w_ in zip(got[k], want[k]):
            assert torch.equal(g, w_), k


def test_forked_capture_equals_direct_passes():
    """Encoder.capture: the frame's graph with the feature LayerNorms forked
    onto a second stream and joined before the next write of the residual
    stream gives the same bits as encoding the program directly, for both
    slots and over repeated replays."""
    import torch
    import beatlm_b200 as bl
    from beatlm_b200.model import Encoder, ViTConfig, block_weights_normal
    cfg = ViTConfig.small(layers=4, out_indices=(1, 2, 4))
    rng = np.random.default_rng(29)
    n = lambda *s: rng.standard_normal(int(np.prod(s)), dtype=np.float32) * 0.02
    w = {"blocks": [block_weights_normal(rng, cfg.dim, cfg.mlp) for _ in range(cfg.layers)],
         "patch_w": n(cfg.patch, cfg.patch, cfg.cin, cfg.dim), "patch_b": n(cfg.dim),
         "cls": n(cfg.dim), "pos": n(cfg.tokens, cfg.dim),
         "norm_g": np.ones(cfg.dim, np.float32), "norm_b": np.zeros(cfg.dim, np.float32)}
    enc = Encoder(cfg, w, "bf16", planned_frames=1, slots=2)
    buf = enc.buffers(1)
    prog = enc.program(1)
    stream = torch.cuda.Stream()
    for slot in (0, 1):
        img = torch.from_numpy(rng.random((1, cfg.side, cfg.side, cfg.cin), dtype=np.float32))
        buf.images[slot].copy_(img.cuda())
        torch.cuda.synchronize()
        prog.encode_all(stream, set=slot)
        stream.synchronize()
        want = [f.clone() for f in enc.features(1, slot=slot)]
        for f in enc.features(1, slot=slot):
            f.zero_()
        torch.cuda.synchronize()
        g = enc.capture(1, stream, slot=slot)
        for _ in range(3):
            with torch.cuda.stream(stream):
                g.replay()
        stream.synchronize()
        for got, w_ in zip(enc.features(1, slot=slot), want):
            assert torch.equal(got, w_), slot
    assert bl.status(reset=True).code == 0
