"""Host logic of the program API on CPU: the row split of Program::split and
the part count of parts_within, against the reference's own rules and test
values (crates/beatlm-core/src/kernel.rs:2006-2056, tests 3298-3445)."""
import pytest

from beatlm_b200 import build
from beatlm_b200.runtime import parts_within, split_edges


@pytest.fixture(scope="module", autouse=True)
def _lib():
    build.build()


def counts(max_parts):
    """The reference test's part counts (kernel.rs:3277-3296)."""
    if max_parts <= 40:
        return list(range(0, max_parts + 4))
    return [0, 1, 2, 3, 7, 22, max_parts - 1, max_parts, max_parts + 1, 200]


def reference_edges(extent, grain, count):
    """kernel.rs:2006-2029, restated: blocks B = ceil(extent / grain), count
    clamped to 1..=B, part i covers blocks [B*i/count, B*(i+1)/count)."""
    blocks = -(-extent // grain)
    count = min(max(count, 1), max(blocks, 1))
    return [min(blocks * i // count * grain, extent) for i in range(count + 1)]


@pytest.mark.parametrize("extent,grain", [(1370, 128), (1370, 1), (1369, 128), (128, 128),
                                          (1, 128), (5477, 128), (10960, 128), (1000, 1)])
def test_parts_cover_the_output_exactly_once(extent, grain):
    max_parts = -(-extent // grain)
    for count in counts(max_parts):
        edges = split_edges(extent, grain, count)
        assert edges == reference_edges(extent, grain, count)
        assert len(edges) - 1 == min(max(count, 1), max_parts)
        assert edges[0] == 0 and edges[-1] == extent
        sizes = [b - a for a, b in zip(edges, edges[1:])]
        assert all(s > 0 for s in sizes), "an empty part"
        assert all(e % grain == 0 for e in edges[:-1]), "a boundary inside a tile"
        assert max(sizes) - min(sizes) <= 2 * grain


def test_the_part_count_is_the_duration_over_the_bound_rounded_up_and_clamped():
    # kernel.rs:3404-3445
    assert parts_within(10_000, 1_000, 1) == 1
    for duration, bound, parts in [(0, 1000, 1), (1, 1000, 1), (999, 1000, 1), (1000, 1000, 1),
                                   (1001, 1000, 2), (2700, 1000, 3), (3000, 1000, 3),
                                   (3001, 1000, 4), (5_000_000, 1, 1000),
                                   (2 ** 64 - 1, 1, 1000), (2 ** 64 - 1, 1000, 1000)]:
        assert parts_within(duration, bound, 1000) == parts, (duration, bound)
    assert parts_within(1, 0, 1000) == 0  # ZeroBound


def test_binding_sets_rebind_only_the_kernels_that_touch_their_tensors():
    """Kernels::new's binding sets (crates/beatlm/src/codegen/kernels.rs:63-184)
    on all-gather specs, which need no device to build: a set that
    substitutes a tensor a kernel reads or writes gives that kernel a launch
    of its own; a kernel that touches none shares set 0's launch. Nothing is
    encoded (the communicator handle is never used at build time)."""
    import ctypes
    from beatlm_b200 import _native as N
    from beatlm_b200.runtime import Kernels, Spec
    bufs = [(ctypes.c_uint8 * 64)() for _ in range(6)]
    a = [ctypes.addressof(b) for b in bufs]
    comm = 0x1000  # a handle: only stored at build time
    specs = [Spec(N.AllGatherArgs(comm=comm, send=a[0], recv=a[1], bytes=16), "first"),
             Spec(N.AllGatherArgs(comm=comm, send=a[2] + 8, recv=a[3], bytes=16), "second")]
    k = Kernels(specs)
    assert (len(k), k.sets, k.launches) == (2, 1, 2)
    # set 1 replaces buffer 1 (only the first kernel's), set 2 buffer 2
    # (the second kernel reads 8 bytes into it)
    k = Kernels(specs, sets=[[], [(a[1], a[4], 64)], [(a[2], a[5], 64)]])
    assert (len(k), k.sets, k.launches) == (2, 3, 4)
    with pytest.raises(N.BackendError, match="binding set 3 of 3"):
        k.encode(0, stream=0, set=3)
    with pytest.raises(N.BackendError, match="overlapping"):
        Kernels(specs, sets=[[(a[1], a[4], 64), (a[1] + 32, a[5], 16)]])
    with pytest.raises(N.BackendError, match="empty"):
        Kernels(specs, sets=[[(a[1], a[4], 0)]])
    with pytest.raises(ValueError, match="stand-in"):
        import torch
        Kernels(specs, sets=[[(torch.zeros(4), torch.zeros(8))]])
