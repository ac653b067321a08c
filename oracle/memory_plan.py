"""CPU oracle for the static memory plan: TEST INFRASTRUCTURE ONLY.

A pure-Python restatement of ``MemoryPlan::new`` in
``crates/beatlm-core/src/memory.rs`` of ynishi/beatlm, used by ``tests/`` to
check the C-ABI planner placement for placement. The product never imports
it.

Pinning: the reference is Rust and cannot run here; this restatement is
pinned by the reference's own planner tests (``memory.rs:600-841``: exact
offsets, arena sizes, peak bytes and errors), which ``tests/test_memory_plan.py``
runs against it and against the C-ABI planner alike.

Tensors are tuples ``(id, elem_bytes, elements, first_use, last_use)``; a
profile is ``(max_binding_bytes, max_buffer_bytes, offset_alignment)``. The
result is ``(arenas, {id: (arena, offset, size)}, peak_live_bytes)`` or an
error tuple ``("Kind", id, a, b)``.
"""
from __future__ import annotations

U64 = (1 << 64) - 1
GRANULARITY = 4  # STORAGE_GRANULARITY, memory.rs:85


def _round_up(v, m):
    """round_up (memory.rs:477-485): None on u64 overflow."""
    r = v % m
    out = v if r == 0 else v + (m - r)
    return out if out <= U64 else None


def _overlaps(a, b):
    """TensorDesc::overlaps (memory.rs:193-195), inclusive at both ends."""
    return a[3] <= b[4] and b[3] <= a[4]


def _lowest_fit(placed, item, size, alignment, cap):
    """Arena::lowest_fit (memory.rs:448-466)."""
    busy = sorted((off, min(off + sz, U64)) for (d, off, sz) in placed if _overlaps(d, item))
    candidate = 0
    for start, end in busy:
        aligned = _round_up(candidate, alignment)
        if aligned is None or aligned + size > U64:
            return None
        if aligned + size <= start:
            break
        candidate = max(candidate, end)
    offset = _round_up(candidate, alignment)
    if offset is None or offset + size > U64 or offset + size > cap:
        return None
    return offset


def _peak_live(sized):
    """peak_live (memory.rs:487-506)."""
    deltas = {}
    for d, size in sized:
        b = deltas.setdefault(d[3], [0, 0])
        b[0] += size
        e = deltas.setdefault(d[4] + 1, [0, 0])
        e[1] += size
    live = peak = 0
    for op in sorted(deltas):
        live = max(0, live + deltas[op][0] - deltas[op][1])
        peak = max(peak, live)
    return peak


def plan(tensors, profile):
    """MemoryPlan::new (memory.rs:285-338) with validate (341-372)."""
    max_binding, max_buffer, alignment = profile
    cap = min(max_binding, max_buffer)
    if alignment == 0 or cap == 0:
        return ("InvalidProfile", 0, 0, 0)
    seen, sized = set(), []
    for d in tensors:
        tid, width, elements, first, last = d
        if tid in seen:
            return ("DuplicateTensor", tid, 0, 0)
        seen.add(tid)
        if first > last:
            return ("InvalidLifetime", tid, first, last)
        if elements == 0:
            return ("EmptyTensor", tid, 0, 0)
        nbytes = elements * width
        size = _round_up(nbytes, GRANULARITY) if nbytes <= U64 else None
        if size is None:
            return ("SizeOverflow", tid, 0, 0)
        if size > cap:
            return ("TensorTooLarge", tid, size, cap)
        sized.append((d, size))
    peak = _peak_live(sized)
    order = sorted(sized, key=lambda s: (-s[1], s[0][0]))
    arenas = []  # [placed list, size]
    placements = {}
    for d, size in order:
        slot = None
        for i, (placed, _) in enumerate(arenas):
            off = _lowest_fit(placed, d, size, alignment, cap)
            if off is not None:
                slot = (i, off)
                break
        if slot is None:
            arenas.append([[], 0])
            slot = (len(arenas) - 1, 0)
        i, off = slot
        arenas[i][0].append((d, off, size))
        arenas[i][1] = max(arenas[i][1], off + size)
        placements[d[0]] = (i, off, size)
    return [a[1] for a in arenas], placements, peak
