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

    def report(self) -> str:
        mb = 1024 * 1024
        pct = 100.0 * (1 - self.total_bytes / self.naive_bytes) if self.naive_bytes else 0.0
        return (f"Arena plan: {len(self.buffers)} buffers, {self.total_bytes / mb:.3f} MB "
                f"(naive {self.naive_bytes / mb:.3f} MB, {pct:.1f}% saved, {ALIGN} B aligned)")


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
