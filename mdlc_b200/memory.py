"""Arena memory plan for the backend's step list.

Restates the reference planner's algorithm (``mdlc/runtime/memory_planner.py:66-146``:
liveness over the topological order, outputs acquired before inputs are
released, best-fit reuse of free buffers, growing the largest free buffer when
none fits) and adds what a device executor needs (the "memory-planner
upgrade" the reference lists as future work):

* it plans over backend *steps*, so a fused conv+residual group keeps its
  input alive until the fused step has run;
* sizes are the real NHWC footprint (bf16 / fp32 / int8, padded channels);
* buffers become offsets in ONE arena allocation, each aligned to 256 bytes;
* zero-copy aliases (Flatten, Reshape ...) share their source's storage.
Graph outputs are never released.
"""

from __future__ import annotations

from dataclasses import dataclass, field

ALIGN = 256


def _align(v: int) -> int:
    return (v + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class ArenaBuffer:
    id: int
    size: int
    offset: int = 0
    tenants: list = field(default_factory=list)


@dataclass
class ArenaPlan:
    offsets: dict          # storage tensor name -> byte offset in the arena
    buffers: list
    total_bytes: int
    naive_bytes: int
    notes: list = field(default_factory=list)   # how a caller-given plan was applied

    def report(self) -> str:
        mb = 1024 * 1024
        pct = 100.0 * (1 - self.total_bytes / self.naive_bytes) if self.naive_bytes else 0.0
        lines = [f"Arena plan: {len(self.buffers)} buffers, {self.total_bytes / mb:.3f} MB "
                 f"(naive {self.naive_bytes / mb:.3f} MB, {pct:.1f}% saved, {ALIGN} B aligned)"]
        lines += [f"  {n}" for n in self.notes]
        return "\n".join(lines)


def storage_of(tensors: dict, name: str) -> str:
    t = tensors[name]
    return t.alias_of or name


def plan_arena(steps, tensors, inputs, outputs, reuse: bool = True) -> ArenaPlan:
    """Best-fit liveness plan; ``reuse=False`` gives every tensor its own buffer
    (calibration executables read every activation after the run)."""
    out_store = {storage_of(tensors, o) for o in outputs}
    last_use = {}
    for k, st in enumerate(steps):
        for i in st.inputs:
            last_use[storage_of(tensors, i)] = k
    inf = len(steps) + 1
    for o in out_store:
        last_use[o] = inf

    buffers, free, assign = [], [], {}
    naive = 0

    def acquire(name):
        need = _align(tensors[name].nbytes)
        best, best_size = -1, None
        for bid in free:
            sz = buffers[bid].size
            if sz >= need and (best_size is None or sz < best_size):
                best, best_size = bid, sz
        if best == -1:
            if free:
                best = max(free, key=lambda b: buffers[b].size)
                buffers[best].size = max(buffers[best].size, need)
            else:
                best = len(buffers)
                buffers.append(ArenaBuffer(best, need))
        if best in free:
            free.remove(best)
        buffers[best].tenants.append(name)
        return best

    def release(names, k):
        if not reuse:
            return
        for e in names:
            if e in out_store or e not in assign:
                continue
            if last_use.get(e, -1) <= k:
                bid = assign[e]
                if bid not in free:
                    free.append(bid)

    # graph inputs are written (layout conversion) before step 0
    for i in inputs:
        s = storage_of(tensors, i)
        if s not in assign:
            naive += _align(tensors[s].nbytes)
            assign[s] = acquire(s)
    for k, st in enumerate(steps):
        for o in st.outputs:
            s = storage_of(tensors, o)
            if s not in assign:
                naive += _align(tensors[s].nbytes)
                assign[s] = acquire(s)
        release([storage_of(tensors, i) for i in st.inputs], k)
    # inputs never read by any step
    off = 0
    for b in buffers:
        b.offset = off
        off += _align(b.size)
    offsets = {name: buffers[bid].offset for name, bid in assign.items()}
    return ArenaPlan(offsets, buffers, off, naive)


def liveness(steps, tensors, inputs, outputs) -> dict:
    """Storage tensor -> (first, last) step index over the backend steps: a
    graph input is live from -1 (written by the layout conversion before step
    0), a step's output from that step, and a tensor stays live through the
    last step reading it (graph outputs: to the end)."""
    inf = len(steps) + 1
    live = {}
    for i in inputs:
        live[storage_of(tensors, i)] = [-1, -1]
    for k, st in enumerate(steps):
        for o in st.outputs:
            s = storage_of(tensors, o)
            if s not in live:
                live[s] = [k, k]
        for i in st.inputs:
            s = storage_of(tensors, i)
            if s in live:
                live[s][1] = max(live[s][1], k)
    for o in outputs:
        live[storage_of(tensors, o)][1] = inf
    return {s: tuple(v) for s, v in live.items()}


def conflicts(plan: ArenaPlan, steps, tensors, inputs, outputs) -> list:
    """Pairs of storage tensors whose arena ranges overlap while both are live.
    Lifetimes are closed intervals: a step's outputs never share memory with
    its own inputs (no kernel here works in place)."""
    live = liveness(steps, tensors, inputs, outputs)
    spans = sorted((off, off + _align(tensors[s].nbytes), s) for s, off in plan.offsets.items())
    bad = []
    for i, (a0, a1, a) in enumerate(spans):
        for b0, b1, b in spans[i + 1:]:
            if b0 >= a1:
                break
            (fa, la), (fb, lb) = live[a], live[b]
            if fa <= lb and fb <= la:
                bad.append((a, b))
    return bad


def plan_from_reference(steps, tensors, inputs, outputs, assignment: dict) -> ArenaPlan:
    """Arena plan that follows a reference ``MemoryPlan``'s tensor -> buffer
    assignment (``mdlc/runtime/memory_planner.py:30-41``; ``plan_memory``
    computes it over IR nodes, ``:66-146``).

    Each reference buffer becomes one arena region sized for its largest
    tenant's NHWC footprint here. The reference plans over IR nodes; the
    backend runs fused steps (a conv with its residual add reads the conv's
    input and the skip tensor and writes the add's output in one kernel), which
    can keep a tensor live longer than the IR order does. A tenant that would
    share its region with a tensor live at the same time is given a region of
    another (shared only among moved tenants, never live at the same time, best
    fit by size), and each such move is recorded in the plan's notes. Tensors the
    reference plan does not pool (graph inputs, which it leaves to external
    storage) get regions of their own; zero-copy aliases share their source's."""
    assignment = getattr(assignment, "assignment", assignment)   # a MemoryPlan or its dict
    live = liveness(steps, tensors, inputs, outputs)
    order = sorted(live, key=lambda s: (live[s][0], s))
    regions, region_of, notes = {}, {}, []
    for s in order:
        bid = assignment.get(s)
        key = ("ref", bid) if bid is not None and s not in inputs else ("own", s)
        f, l_ = live[s]

        def clash(k):
            return [t for t in regions.get(k, []) if live[t][0] <= l_ and f <= live[t][1]]

        if key[0] == "ref" and clash(key):
            other = clash(key)[0]
            # best fit among the regions it can share: no tenant live at the same
            # time, the smallest that holds it (else the largest)
            need = _align(tensors[s].nbytes)
            free = [k for k in regions if k[0] == "moved" and not clash(k)]
            fits = [k for k in free if max(_align(tensors[t].nbytes) for t in regions[k]) >= need]
            size = lambda k: max(_align(tensors[t].nbytes) for t in regions[k])   # noqa: E731
            key = min(fits, key=size) if fits else (max(free, key=size) if free else ("moved", s))
            notes.append(f"mem_plan: {s!r} moved out of reference buffer {bid} "
                         f"(live with {other!r} across the backend's fused steps)")
        regions.setdefault(key, []).append(s)
        region_of[s] = key
    used_ref = {k[1] for k in regions if k[0] == "ref"}
    missing = sorted(n for n in assignment if n not in live)
    notes.insert(0, f"mem_plan: {len(used_ref)} reference buffers honoured; "
                    f"{len(missing)} planned tensors absent here (fused away or aliased)")
    buffers, off, naive = [], 0, 0
    offsets = {}
    for key, tenants in regions.items():
        size = max(_align(tensors[t].nbytes) for t in tenants)
        buffers.append(ArenaBuffer(len(buffers), size, off, list(tenants)))
        for t in tenants:
            offsets[t] = off
            naive += _align(tensors[t].nbytes)
        off += size
    return ArenaPlan(offsets, buffers, off, naive, notes)
