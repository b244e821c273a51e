"""``compile(graph) -> Executable``: the drop-in for mdlc's codegen + GPU runtime.

Reference surface replaced (``mdlc/compiler.py:64-95`` builds ``Compiled``
with a ``CudaModule`` from ``emit_cuda_module`` (``codegen/cuda/emit.py:292``)
that ``GpuExecutor(module).run(feeds, timing)`` executes
(``codegen/cuda/gpu_executor.py:38-98``)). Here:

    exe = compile(graph, dtype="bf16", batch=256, devices=8)
    out = exe.run({"input": x})          # dict name -> np.ndarray (fp32, reference layout)
    exe.report(); exe.fallbacks() == []  # no host fallbacks, ever
    exe.time_ms(iters=50, warmup=10)     # CUDA-event timing (nvrtc_runtime.py:211-225)

``graph`` is the passes-optimised IR — the reference's own ``Graph`` from
``default_pipeline()`` works by duck typing, as does
:class:`mdlc_b200.ir.Graph` from :func:`mdlc_b200.passes.default_pipeline`.
Two schedule hooks: ``schedule_fn(node, (M, N, K)) -> GemmSchedule`` is the
reference codegen's own hook (``emit.py:27,100``; a reference ``Tuner`` works
as one), called with the same (M, N, K) per node, its output-channel tile
mapped to this kernel's tile width (:func:`mdlc_b200.tuner.from_reference_schedule`);
``tuner(kind, geom) -> (bn, stages) | None`` (:class:`mdlc_b200.tuner.Tuner`)
searches this kernel's own tile configurations.

``mem_plan`` (a reference ``MemoryPlan``, ``mdlc/runtime/memory_planner.py:30-41``,
or its ``assignment`` dict) lays the arena out by the plan's tensor -> buffer
sharing where that is safe for the backend's fused steps
(:func:`mdlc_b200.memory.plan_from_reference`; ``report()`` lists what moved).

Multi-GPU: ``devices=G`` shards the batch into G contiguous slices, one per
GPU, with weights replicated and no collective; each device runs its slice
on its own stream from its own host thread and the outputs are gathered on
the host.
"""

from __future__ import annotations

import ctypes as C
import threading
from dataclasses import dataclass

import numpy as np

from mdlc_b200 import _lib as L
from mdlc_b200 import lowering, memory
from mdlc_b200 import tuner as tuner_mod
from mdlc_b200 import shapes as S

DTYPES = {"bf16": L.BF16, "fp32": L.F32, "f32": L.F32, "int8": L.U8}


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN stays a quiet NaN)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = (u + (((u >> 16) & 1) + 0x7FFF)) >> 16
    r = np.where(np.isnan(a), 0x7FC0, r)
    return r.astype(np.uint16)


def _has_static_shapes(graph) -> bool:
    vi = graph.value_info
    for n in graph.nodes:
        for o in n.outputs:
            if o and (o not in vi or not all(isinstance(d, (int, np.integer)) and d >= 0
                                             for d in vi[o].shape)):
                return False
    return True


@dataclass
class _ConvCall:
    desc: L.ConvDesc
    x: str
    y: str
    res: str
    weight: str
    epi: L.Epilogue
    cfg: L.TileCfg


class _Device:
    """Per-GPU state: context, weights, arena, staging buffers, prepared calls."""

    def __init__(self, exe: "Executable", device: int, batch: int):
        self.exe = exe
        self.ctx = L.Context(device)
        self.batch = batch
        lo = exe._lowered_for(batch)
        self.lo = lo
        ref_plan = exe.ref_mem_plan
        if ref_plan is not None and not exe.keep_all:
            # the reference MemoryPlan's tensor -> buffer assignment (or that dict itself)
            assignment = getattr(ref_plan, "assignment", ref_plan)
            self.plan = memory.plan_from_reference(lo.steps, lo.tensors, lo.inputs, lo.outputs, assignment)
            bad = memory.conflicts(self.plan, lo.steps, lo.tensors, lo.inputs, lo.outputs)
            if bad:
                raise RuntimeError(f"internal: arena plan from mem_plan overlaps live tensors {bad[:3]}")
        else:
            self.plan = memory.plan_arena(lo.steps, lo.tensors, lo.inputs, lo.outputs, reuse=not exe.keep_all)
        self.q = exe.qplan
        self.arena = self.ctx.alloc(max(self.plan.total_bytes, 256))
        self.addr = {name: self.arena + off for name, off in self.plan.offsets.items()}
        # weights (packed on the host by the library's packer, uploaded once)
        self.wbuf, self.bbuf = {}, {}
        self.qbuf = {}
        for wname, (geom, wt, bias) in lo.weights.items():
            desc = self._desc(geom, lo)
            if self.q is not None:
                cq = self.q.convs[wname]
                ks = desc.k_stride
                # a paired stem computes two output columns per row: its per-channel
                # parameters repeat for the second column
                rep = 2 if geom.get("paired") else 1

                def pad(a, dt):
                    a = np.tile(np.asarray(a, dt), rep)
                    return np.concatenate([a, np.zeros(ks - len(a), dt)])
                self.wbuf[wname] = self.ctx.to_device(L.pack_weights(desc, cq.w_q))
                self.bbuf[wname] = self.ctx.to_device(pad(cq.bias32, np.int32))
                self.qbuf[wname] = {
                    "mult": self.ctx.to_device(pad(cq.rq_mult, np.int32)) if cq.rq_mult is not None else 0,
                    "res_mult": self.ctx.to_device(pad(cq.rq_res_mult, np.int32)) if cq.rq_mult is not None else 0,
                    "shift": self.ctx.to_device(pad(cq.rq_shift, np.int32)) if cq.rq_mult is not None else 0,
                    "scale": self.ctx.to_device(pad(cq.rq_scale, np.float32)),
                    "deq_scale": self.ctx.to_device(pad(cq.deq_scale, np.float32)) if cq.deq_scale is not None else 0,
                    "deq_bias": self.ctx.to_device(pad(cq.deq_bias, np.float32)) if cq.deq_bias is not None else 0}
            else:
                packed = L.pack_weights(desc, wt)
                self.wbuf[wname] = self.ctx.to_device(packed)
                self.bbuf[wname] = self.ctx.to_device(bias)
        # squeeze-excite gates: fp32 FC weights and biases as they are
        self.sebuf = {}
        for st in lo.steps:
            if st.kind == "se":
                p = st.params
                self.sebuf[id(st)] = tuple(self.ctx.to_device(p[k]) for k in ("w1", "b1", "w2t", "b2"))
        # elementwise constant operands are read in the tensors' own dtype
        self.cbuf = {name: self.ctx.to_device(_bf16_bits(arr) if lo.dtype == L.BF16 else arr)
                     for name, arr in lo.consts.items()}
        # staging: fp32 NCHW feeds / outputs on device and pinned on the host, in
        # two slots (slot 1 allocated on first use) so that one slot's upload can
        # overlap the other slot's forward
        self.in_dev, self.in_host, self.out_dev, self.out_host = {}, {}, {}, {}
        for name in lo.inputs:
            nbytes = int(np.prod(lo.shapes[name])) * 4
            self.in_dev[name] = [self.ctx.alloc(nbytes), None]
            self.in_host[name] = [self.ctx.host_alloc(nbytes), None]
        for name in lo.outputs:
            nbytes = int(np.prod(lo.shapes[name])) * 4
            t = lo.tensors[name]
            direct = t.dtype == L.F32 and t.cs == t.c and t.h * t.w == 1
            self.out_dev[name] = None if direct else self.ctx.alloc(nbytes)
            self.out_host[name] = [self.ctx.host_alloc(nbytes), None]
        self.calls = self._prepare()
        self.graph_ready = False

    def ptr(self, name):
        return self.addr[memory.storage_of(self.lo.tensors, name)]

    def _desc(self, geom, lo):
        k = geom["k"]
        a8 = 16 if lo.dtype in (L.U8, L.S8) else 8
        return L.ConvDesc(n=geom["n"], h=geom["h"], w=geom["w"], c=geom["c"],
                          c_stride=geom.get("cs", lowering.round_up(geom["c"], a8)), k=k,
                          k_stride=lowering.round_up(k, a8),
                          r=geom["r"], s=geom["s"], stride_h=geom["sh"], stride_w=geom["sw"],
                          pad_t=geom["pt"], pad_l=geom["pl"], dil_h=geom["dh"], dil_w=geom["dw"],
                          oh=geom["oh"], ow=geom["ow"], groups=geom["groups"], in_type=lo.dtype,
                          out_type=lo.dtype, res_stride=0, in_zp=0)

    def _prepare(self):
        lo, calls = self.lo, []
        for st in lo.steps:
            if st.kind == "conv":
                geom, _, _ = lo.weights[st.params["weight"]]
                d = self._desc(geom, lo)
                yt = lo.tensors[st.outputs[0]]
                d.in_type = lo.tensors[st.inputs[0]].dtype   # int8 graphs: signed network input
                d.out_type = yt.dtype
                a = st.params["attrs"]
                act = st.params["act"]
                epi = L.Epilogue(act=lowering.ACT_CODES[act], alpha=float(a.get("alpha", 0.01)),
                                 beta=float(a.get("beta", 0.5)),
                                 clip_lo=-np.inf if a.get("clip_min") is None else float(a["clip_min"]),
                                 clip_hi=np.inf if a.get("clip_max") is None else float(a["clip_max"]))
                if act == "HardSigmoid":
                    epi.alpha = float(a.get("alpha", 0.2))
                if self.q is not None:
                    cq = self.q.convs[st.params["weight"]]
                    qb = self.qbuf[st.params["weight"]]
                    s_x, zp_x = self.q.tensors[self._store(st.inputs[0])]
                    d.in_zp = zp_x
                    if yt.dtype != L.F32:
                        epi.act = L.ACT_NONE     # the activation is the integer clamp
                    epi.rq_scale = qb["scale"]
                    if yt.dtype != L.F32 and qb["mult"]:
                        epi.rq_mult, epi.rq_res_mult, epi.rq_shift = qb["mult"], qb["res_mult"], qb["shift"]
                    epi.deq_scale, epi.deq_bias = qb["deq_scale"] or None, qb["deq_bias"] or None
                    if cq.residual:
                        epi.res_zp = self.q.tensors[self._store(cq.residual)][1]
                        epi.res_scale = cq.res_scale
                        epi.res_signed = int(lo.tensors[cq.residual].dtype == L.S8)
                    if yt.dtype != L.F32:
                        epi.out_zp = self.q.tensors[st.outputs[0]][1]
                        epi.qmin, epi.qmax = cq.qmin, cq.qmax
                cfg = None
                choice = None
                if self.exe.tuner is not None:
                    choice = self.exe.tuner("conv", dict(geom, dtype=lo.dtype))
                elif self.exe.schedule_fn is not None:
                    choice = tuner_mod.from_reference_schedule(self.exe.schedule_fn,
                                                               self.exe.node_by_name.get(st.nodes[0]), geom)
                if choice:
                    cfg = L.TileCfg(bn=choice[0], stages=choice[1], flags=0)
                    self.exe.schedules[st.params["weight"]] = tuple(choice)
                calls.append(("conv", d, self.ptr(st.inputs[0]), self.wbuf[st.params["weight"]],
                              self.bbuf[st.params["weight"]],
                              self.ptr(st.params["residual"]) if st.params["residual"] else 0,
                              self.ptr(st.outputs[0]), epi, cfg))
            elif st.kind == "copy":
                yt = lo.tensors[st.outputs[0]]
                for part in st.params["parts"]:
                    xt = lo.tensors[part["src"]]
                    d = L.CopyDesc(dtype=yt.dtype, in_cs=xt.cs, out_cs=yt.cs, mode=part["mode"],
                                   pad_mode=part["pad_mode"], value=part["value"])
                    for i, v in enumerate((xt.n, xt.c, xt.h, xt.w)):
                        d.in_dims[i] = v
                    for i, v in enumerate((yt.n, yt.c, yt.h, yt.w)):
                        d.out_dims[i] = v
                    for i in range(4):
                        d.src_dim[i] = part["src_dim"][i]
                        d.offset[i] = part["offset"][i]
                    calls.append(("copy", d, self.ptr(part["src"]), self.ptr(st.outputs[0])))
            elif st.kind == "softmax":
                t = lo.tensors[st.inputs[0]]
                d = L.SoftmaxDesc(dtype=t.dtype, cs=t.cs, axis=st.params["axis"])
                for i, v in enumerate((t.n, t.c, t.h, t.w)):
                    d.dims[i] = v
                calls.append(("softmax", d, self.ptr(st.inputs[0]), self.ptr(st.outputs[0])))
            elif st.kind == "se":
                xt, yt = lo.tensors[st.inputs[0]], lo.tensors[st.outputs[0]]
                p = st.params
                rd, c = p["w1"].shape
                # hw > 1: the step absorbed the global average pool and reads its input
                d = L.SeDesc(n=xt.n, c=c, c_stride=xt.cs, rd=rd, dtype=xt.dtype, hw=xt.h * xt.w)
                if yt.cs != xt.cs:
                    raise RuntimeError(f"internal: se step {st.label()} with different channel strides")
                for i, (act, a) in enumerate(((p["act1"], p["attrs1"]), (p["act2"], p["attrs2"])), 1):
                    setattr(d, f"act{i}", lowering.ACT_CODES[act])
                    setattr(d, f"alpha{i}", float(a.get("alpha", 0.2 if act == "HardSigmoid" else 0.01)))
                    setattr(d, f"beta{i}", float(a.get("beta", 0.5)))
                    setattr(d, f"lo{i}", -np.inf if a.get("clip_min") is None else float(a["clip_min"]))
                    setattr(d, f"hi{i}", np.inf if a.get("clip_max") is None else float(a["clip_max"]))
                w1, b1, w2t, b2 = self.sebuf[id(st)]
                calls.append(("se", d, self.ptr(st.inputs[0]), w1, b1, w2t, b2, self.ptr(st.outputs[0])))
            elif st.kind == "pool":
                xt, yt = lo.tensors[st.inputs[0]], lo.tensors[st.outputs[0]]
                p = st.params
                d = L.PoolDesc(kind=p["kind"], n=xt.n, h=xt.h, w=xt.w, c=xt.c, c_stride=xt.cs,
                               kh=p.get("kh", 1), kw=p.get("kw", 1), stride_h=p.get("sh", 1),
                               stride_w=p.get("sw", 1), pad_t=p.get("pt", 0), pad_l=p.get("pl", 0),
                               oh=p.get("oh", 1), ow=p.get("ow", 1), count_include_pad=p.get("cip", 0),
                               dtype=xt.dtype)
                if self.q is not None and p["kind"] == 2:
                    d.rq_mult, d.rq_shift, d.in_zp, d.out_zp = self.q.gap[st.outputs[0]]
                calls.append(("pool", d, self.ptr(st.inputs[0]), self.ptr(st.outputs[0])))
            else:
                yt = lo.tensors[st.outputs[0]]
                p = st.params
                prog = L.EwProg(n=yt.n, hw=yt.h * yt.w, c=yt.c, c_stride=yt.cs, dtype=yt.dtype,
                                n_inputs=len(p["operands"]), n_outputs=len(st.outputs),
                                n_instr=len(p["code"]))
                for i, m in enumerate(p["bcast"]):
                    prog.bcast[i] = m
                for i, r in enumerate(p["out_regs"]):
                    prog.out_reg[i] = r
                for i, (op, dst, s0, s1, f0, f1) in enumerate(p["code"]):
                    prog.code[i] = L.EwInstr(op=op, dst=dst, src0=s0, src1=s1, imm0=f0, imm1=f1)
                ins = [self.cbuf[o] if o in self.cbuf else self.ptr(o) for o in p["operands"]]
                calls.append(("eltwise", prog, ins, [self.ptr(o) for o in st.outputs]))
        return calls

    # -------------------------------------------------------------- execution
    def issue_steps(self):
        ctx = self.ctx
        for c in self.calls:
            if c[0] == "conv":
                _, d, x, w, b, r, y, epi, cfg = c
                ctx.conv2d(d, x, w, b, r, y, epi, cfg)
            elif c[0] == "pool":
                ctx.pool2d(c[1], c[2], c[3])
            elif c[0] == "copy":
                ctx.copy4d(c[1], c[2], c[3])
            elif c[0] == "softmax":
                ctx.softmax(c[1], c[2], c[3])
            elif c[0] == "se":
                ctx.se_fc(*c[1:])
            else:
                ctx.eltwise(c[1], c[2], c[3])

    def _store(self, name):
        return memory.storage_of(self.lo.tensors, name)

    def _slot(self, slot):
        if slot not in (0, 1):
            raise ValueError("slot must be 0 or 1")
        if slot == 1 and self.lo.inputs and self.in_dev[self.lo.inputs[0]][1] is None:
            for name in self.lo.inputs:
                nbytes = int(np.prod(self.lo.shapes[name])) * 4
                self.in_dev[name][1] = self.ctx.alloc(nbytes)
                self.in_host[name][1] = self.ctx.host_alloc(nbytes)
            for name in self.lo.outputs:
                self.out_host[name][1] = self.ctx.host_alloc(int(np.prod(self.lo.shapes[name])) * 4)
        return slot

    def issue_inputs(self, slot=0):
        for name in self.lo.inputs:
            t = self.lo.tensors[name]
            inv, zp = 1.0, 0
            if self.q is not None:
                s_x, zp = self.q.tensors[name]
                inv = float(np.float32(1.0) / np.float32(s_x))
            if t.layout == "s2d2":
                n, c, h, w = self.lo.shapes[name]
                self.ctx.to_s2d(self.in_dev[name][slot], n, c, h, w, self.ptr(name), t.cs, t.dtype, inv, zp)
            else:
                self.ctx.to_nhwc(self.in_dev[name][slot], t.n, t.c, t.h, t.w, self.ptr(name), t.cs, t.dtype,
                                 inv, zp)

    def issue_outputs(self):
        for name in self.lo.outputs:
            t = self.lo.tensors[name]
            if self.out_dev[name] is not None:
                scale, zp = (1.0, 0) if self.q is None or t.dtype == L.F32 else self.q.tensors[self._store(name)]
                self.ctx.to_nchw(self.ptr(name), t.n, t.c, t.h, t.w, t.cs, t.dtype, self.out_dev[name],
                                 float(scale), zp)

    def read_tensors(self):
        """Every stored activation as an NCHW array (a keep_all executable keeps
        each one in its own buffer): float32 values of fp32 executables, the
        8-bit codes (or fp32 logits) of int8 ones."""
        if self.lo.dtype not in (L.F32, L.U8):
            raise ValueError("read_tensors: fp32 and int8 executables only")
        self.ctx.sync()
        out = {}
        for name, t in self.lo.tensors.items():
            if t.alias_of or name not in self.addr or t.layout != "nhwc":
                continue
            npdt = {L.F32: np.float32, L.S8: np.int8}.get(t.dtype, np.uint8)
            a = self.ctx.download(self.addr[name], (t.n, t.h, t.w, t.cs), npdt)[..., :t.c]
            out[name] = a.transpose(0, 3, 1, 2).reshape(self.lo.shapes[name])
        return out

    def out_src(self, name):
        return self.out_dev[name] if self.out_dev[name] is not None else self.ptr(name)

    def issue_forward(self):
        """Device-resident forward: layout-in, every step, layout-out."""
        self.issue_inputs()
        self.issue_steps()
        self.issue_outputs()

    def capture(self):
        self.ctx.graph_begin()
        try:
            self.issue_forward()
        finally:
            self.ctx.graph_end()
        self.graph_ready = True

    def forward(self, use_graph):
        if use_graph:
            if not self.graph_ready:
                self.capture()
            self.ctx.graph_launch()
        else:
            self.issue_forward()

    def run_host(self, feeds_slice, use_graph=False):
        """Pinned H2D of the feeds, forward, D2H of the outputs (all on the stream)."""
        lo = self.lo
        for name in lo.inputs:
            arr = np.ascontiguousarray(feeds_slice[name], dtype=np.float32)
            host = np.ctypeslib.as_array((C.c_float * arr.size).from_address(self.in_host[name][0]))
            host[:] = arr.reshape(-1)
            self.ctx.upload_async(self.in_dev[name][0], self.in_host[name][0], arr.nbytes)
        self.forward(use_graph)
        outs = {}
        for name in lo.outputs:
            n = int(np.prod(lo.shapes[name]))
            self.ctx.download_async(self.out_host[name][0], self.out_src(name), n * 4)
        self.ctx.sync()
        for name in lo.outputs:
            n = int(np.prod(lo.shapes[name]))
            host = np.ctypeslib.as_array((C.c_float * n).from_address(self.out_host[name][0]))
            outs[name] = host.copy().reshape(lo.shapes[name])
        return outs

    def pinned_views(self, slot=0):
        lo = self.lo
        slot = self._slot(slot)
        ins = {n: np.ctypeslib.as_array((C.c_float * int(np.prod(lo.shapes[n]))).from_address(
            self.in_host[n][slot])).reshape(lo.shapes[n]) for n in lo.inputs}
        outs = {n: np.ctypeslib.as_array((C.c_float * int(np.prod(lo.shapes[n]))).from_address(
            self.out_host[n][slot])).reshape(lo.shapes[n]) for n in lo.outputs}
        return ins, outs

    def issue_pinned(self, use_graph=False):
        """H2D from the pinned feed buffers, forward, D2H into the pinned output buffers."""
        lo = self.lo
        for name in lo.inputs:
            self.ctx.upload_async(self.in_dev[name][0], self.in_host[name][0], int(np.prod(lo.shapes[name])) * 4)
        self.forward(use_graph)
        for name in lo.outputs:
            self.ctx.download_async(self.out_host[name][0], self.out_src(name), int(np.prod(lo.shapes[name])) * 4)

    # fences: 0 + slot upload landed, 2 + slot upload consumed, 4 + slot outputs read back
    def submit(self, slot):
        """Pipelined forward of one slot: the upload of the slot's pinned feeds
        runs on the copy stream (after the slot's previous feeds were consumed),
        the forward and the read-back of its outputs on the compute stream after
        the upload, so an upload overlaps the other slot's forward."""
        ctx, lo = self.ctx, self.lo
        slot = self._slot(slot)
        ctx.fence_wait(2 + slot, L.STREAM_COPY)
        for name in lo.inputs:
            ctx.upload_on(L.STREAM_COPY, self.in_dev[name][slot], self.in_host[name][slot],
                          int(np.prod(lo.shapes[name])) * 4)
        ctx.fence_record(0 + slot, L.STREAM_COPY)
        ctx.fence_wait(0 + slot, L.STREAM_COMPUTE)
        self.issue_inputs(slot)
        ctx.fence_record(2 + slot, L.STREAM_COMPUTE)
        self.issue_steps()
        self.issue_outputs()
        for name in lo.outputs:
            ctx.download_on(L.STREAM_COMPUTE, self.out_host[name][slot], self.out_src(name),
                            int(np.prod(lo.shapes[name])) * 4)
        ctx.fence_record(4 + slot, L.STREAM_COMPUTE)

    def wait(self, slot, timeout_ms=60000):
        self.ctx.fence_sync(4 + slot, timeout_ms)

    def close(self):
        self.ctx.close()


class Executable:
    """A compiled graph bound to one or more B200s."""

    def __init__(self, graph, *, dtype="bf16", batch=None, devices=1, tuner=None, mem_plan=None,
                 keep_all=False, calib=None, schedule_fn=None, requant="fixed"):
        if dtype not in DTYPES:
            raise ValueError(f"dtype must be one of {sorted(DTYPES)}")
        if tuner not in (None, False) and schedule_fn is not None:
            raise ValueError("give either tuner= or schedule_fn=, not both")
        if tuner is None and schedule_fn is None:
            # the shipped per-shape cache of measured tile configurations
            # (mdlc_b200/tune_cache.json); shapes it lacks keep the library heuristic
            tuner = tuner_mod.Tuner(model=False)
        elif tuner is False:
            tuner = None
        self.schedule_fn = schedule_fn
        self.schedules = {}   # weight name -> (bn, stages) chosen through a hook
        self.node_by_name = {n.name: n for n in graph.nodes}
        self.graph = graph
        self.keep_all = keep_all
        self.qplan = None
        self.calib = calib
        self.dtype_name = dtype
        self.dtype = DTYPES[dtype]
        self.tuner = tuner
        self.ref_mem_plan = mem_plan
        base = S.infer(graph, batch)
        self.batch = int(batch if batch is not None else base[graph.runtime_inputs[0]][0])
        if _has_static_shapes(graph) and batch is None:
            for n in graph.nodes:
                for o in n.outputs:
                    if o and tuple(graph.value_info[o].shape) != tuple(base[o]):
                        raise ValueError(f"recorded shape of {o!r} disagrees with the shape rules")
        if isinstance(devices, int):
            ndev = devices
            devs = list(range(devices))
        else:
            devs = list(devices)
            ndev = len(devs)
        if ndev < 1 or self.batch % ndev:
            raise ValueError(f"batch {self.batch} must split evenly over {ndev} devices")
        self.shard = self.batch // ndev
        self._lowered = {}
        self.lowered = self._lowered_for(self.shard)   # validates the graph (raises on gaps)
        mixing = [st.label() for st in self.lowered.steps if st.params.get("batch_mixing")]
        if ndev > 1 and mixing:
            raise lowering.LoweringError(f"{mixing[0]} mixes images across the batch axis, which "
                                         f"devices={ndev} shards; compile it for one device")
        if self.dtype == L.U8:
            from mdlc_b200 import quant
            ranges = calib
            if ranges is None or isinstance(ranges, list):
                batches = ranges if ranges is not None else quant.calibration_batches(graph)
                ranges = quant.calibrate(graph, batches, device=devs[0])
            self.ranges = ranges
            lo_orig = lowering.lower(graph, S.infer(graph, self.shard), L.U8, s2d=False)
            self.qplan = quant.build_plan(lo_orig, self.lowered, ranges, graph, requant=requant)
        self.devices = [_Device(self, d, self.shard) for d in devs]

    def _lowered_for(self, batch):
        if batch not in self._lowered:
            shp = S.infer(self.graph, batch)
            # a keep_all executable (int8 calibration, debugging) keeps every
            # activation, so it does not fuse squeeze-excite gates away
            lo = lowering.lower(self.graph, shp, self.dtype, fuse_se=not self.keep_all)
            for o in lo.outputs:      # dense-conv graph outputs are written as fp32 directly
                prod = [st for st in lo.steps if o in st.outputs]
                if prod and prod[0].kind == "conv" and lo.weights[prod[0].params["weight"]][0]["groups"] == 1:
                    lo.tensors[o].dtype = L.F32
            self._lowered[batch] = lo
        return self._lowered[batch]

    # ------------------------------------------------------------------ API
    def run(self, feeds: dict, *, use_graph: bool = False) -> dict:
        """Run on host numpy feeds; returns fp32 outputs in the reference layout."""
        names = self.lowered.inputs
        missing = [n for n in names if n not in feeds]
        if missing:
            raise KeyError(f"missing feeds: {missing}")
        slices = []
        for i, _ in enumerate(self.devices):
            lo, hi = i * self.shard, (i + 1) * self.shard
            slices.append({n: np.asarray(feeds[n])[lo:hi] for n in names})
        if len(self.devices) == 1:
            results = [self.devices[0].run_host(slices[0], use_graph)]
        else:
            results = [None] * len(self.devices)
            errors = []

            def work(i):
                try:
                    results[i] = self.devices[i].run_host(slices[i], use_graph)
                except BaseException as e:   # noqa: BLE001 - re-raised below
                    errors.append(e)

            threads = [threading.Thread(target=work, args=(i,)) for i in range(len(self.devices))]
            for t in threads:
                t.start()
            for t in threads:
                t.join()
            if errors:
                raise errors[0]
        return {o: np.concatenate([r[o] for r in results], axis=0) if len(results) > 1 else results[0][o]
                for o in self.lowered.outputs}

    def pinned_inputs(self, device: int = 0, slot: int = 0) -> dict:
        """Numpy views of a device's pinned feed buffers (fill them, then
        ``run_pinned`` for slot 0, or ``submit(slot)``)."""
        return self.devices[device].pinned_views(slot)[0]

    def pinned_outputs(self, device: int = 0, slot: int = 0) -> dict:
        """Numpy views of a device's pinned output buffers (valid after
        ``run_pinned`` + ``sync``, or ``wait(slot)``)."""
        return self.devices[device].pinned_views(slot)[1]

    def submit(self, slot: int = 0) -> None:
        """Asynchronous, double-buffered serving call: upload the pinned feeds of
        ``slot`` (0 or 1) on each device's copy stream, run the forward and read
        the outputs back into the slot's pinned outputs. Alternating slots lets
        the upload of one batch overlap the forward of the other. Fill a slot's
        inputs / read its outputs only after ``wait(slot)``."""
        for d in self.devices:
            d.submit(slot)

    def wait(self, slot: int = 0) -> dict:
        """Block until the last ``submit(slot)`` has finished; returns device
        0's pinned output views for the slot. Device errors surface at ``sync``."""
        for d in self.devices:
            d.wait(slot)
        return self.pinned_outputs(0, slot)

    def run_pinned(self, use_graph: bool = False, sync: bool = True) -> None:
        """Zero-copy host API: pinned H2D of the feeds, forward, D2H of the outputs."""
        for d in self.devices:
            d.issue_pinned(use_graph)
        if sync:
            self.sync()

    def forward_device(self, use_graph: bool = False) -> None:
        """Issue one forward on every device with inputs already resident."""
        for d in self.devices:
            d.forward(use_graph)

    def sync(self) -> None:
        for d in self.devices:
            d.ctx.sync()

    def read_tensors(self, device: int = 0) -> dict:
        """Every stored activation of one device's last forward (``keep_all`` executables)."""
        if not self.keep_all:
            raise ValueError("read_tensors needs an executable compiled with keep_all=True")
        return self.devices[device].read_tensors()

    def time_ms(self, iters: int = 50, warmup: int = 10, use_graph: bool = False) -> float:
        """Device time per forward (CUDA events on each device's stream; max over devices)."""
        for _ in range(warmup):
            self.forward_device(use_graph)
        self.sync()
        for d in self.devices:
            d.ctx.event_record(0)
        for _ in range(iters):
            self.forward_device(use_graph)
        for d in self.devices:
            d.ctx.event_record(1)
        self.sync()
        return max(d.ctx.event_elapsed(0, 1) for d in self.devices) / iters

    def fallbacks(self) -> list:
        """Host-executed operations: always none (``emit.py:57-72`` lists them in the reference)."""
        return []

    def launches_per_forward(self) -> int:
        return len(self.lowered.steps) + len(self.lowered.inputs) + sum(
            1 for o in self.lowered.outputs if self.devices[0].out_dev[o] is not None)

    def report(self) -> str:
        lo = self.lowered
        kinds = {}
        for st in lo.steps:
            kinds[st.kind] = kinds.get(st.kind, 0) + 1
        lines = ["== mdlc_b200 executable ==",
                 f"dtype {self.dtype_name}, batch {self.batch} over {len(self.devices)} device(s) "
                 f"({self.shard} per device)",
                 f"steps: {len(lo.steps)} (" + ", ".join(f"{k}x{v}" for k, v in sorted(kinds.items())) + ")",
                 f"kernel launches per forward: {self.launches_per_forward()}",
                 "host fallbacks: none",
                 self.devices[0].plan.report()]
        w = sum(L.weight_bytes(self.devices[0]._desc(g, lo)) for g, _, _ in lo.weights.values())
        lines.append(f"packed weights: {w / 2**20:.3f} MB per device")
        for st in lo.steps:
            lines.append(f"  {st.label()}: {', '.join(st.inputs)} -> {', '.join(st.outputs)}")
        return "\n".join(lines)

    def close(self) -> None:
        for d in self.devices:
            d.close()
        self.devices = []


def compile(graph, *, mem_plan=None, dtype: str = "bf16", batch=None, devices=1, tuner=None,
            schedule_fn=None, calib=None, requant: str = "fixed") -> Executable:
    """Compile a post-pass Graph IR for B200 execution (see module docstring).

    ``mem_plan``: a reference ``MemoryPlan`` (or its tensor -> buffer id dict)
    to lay the activation arena out by. ``schedule_fn``: the reference's
    ``schedule_fn(node, (M, N, K))`` hook; ``tuner``: this backend's
    ``tuner(kind, geom)`` hook (at most one of the two).

    ``dtype="int8"`` quantises the graph (:mod:`mdlc_b200.quant`): ``calib`` is
    either a dict of per-tensor (min, max) ranges, a list of feed dicts to
    calibrate on, or None for 32 seeded N(0, 1) batches of 4 images; ``requant``
    selects the 8-bit conv requantisation: ``"fixed"`` (default; integer
    multiplier and shift, one rounding) or ``"fp32"`` (an fp32 scale, rint).
    """
    return Executable(graph, dtype=dtype, batch=batch, devices=devices, tuner=tuner, schedule_fn=schedule_fn,
                      mem_plan=mem_plan, calib=calib, requant=requant)
