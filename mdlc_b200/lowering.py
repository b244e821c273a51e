"""Lower a post-pass Graph IR to a list of backend steps.

This replaces the reference's ``CudaCodegen.lower`` (``mdlc/codegen/cuda/emit.py:137-293``):
instead of emitting CUDA C per node and bouncing unsupported ops to the host
(``emit.py:32-35,148-157,175-180``), each IR node (or fused group of nodes)
becomes one call of a prebuilt kernel in ``libmdlc_b200.so``:

* ``Conv`` / ``FusedConvAct`` / ``FusedConvBNAct`` / ``Gemm`` / ``FusedGemmAct``
  / ``MatMul`` -> ``conv`` step (implicit GEMM; depthwise when
  ``group == C == K``), with bias and activation in the epilogue.
* Backend-level epilogue fusion on top of the reference passes: a plain conv
  whose single consumer is ``Add(conv, skip)`` (bare, or a ``FusedElementwise``
  ``[Add, act]``) absorbs the add and activation as a residual epilogue; the
  opset-17 GELU decomposition ``x * 0.5 * (1 + erf(x / sqrt 2))`` hanging off a
  conv becomes a GELU epilogue.
* ``MaxPool`` / ``AveragePool`` / ``GlobalAveragePool`` / ``ReduceMean`` over
  H,W -> ``pool`` step.
* Remaining elementwise nodes and ``FusedElementwise`` groups -> ``eltwise``
  step (an interpreted register program, broadcasting per (n, c), per c, or
  scalar operands).
* ``Flatten`` / ``Reshape`` / ``Squeeze`` / ``Unsqueeze`` / ``Identity`` ->
  zero-copy aliases when the NHWC storage order is unchanged.
Nothing is executed on the host; an op the backend cannot lower raises at
compile time (the executable's ``fallbacks()`` is always empty).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np

from mdlc_b200 import _lib as L
from mdlc_b200 import shapes as S


class LoweringError(NotImplementedError):
    pass


ACT_CODES = {None: L.ACT_NONE, "Identity": L.ACT_NONE, "Relu": L.ACT_RELU, "Clip": L.ACT_CLIP,
             "Relu6": L.ACT_CLIP, "Sigmoid": L.ACT_SIGMOID, "Tanh": L.ACT_TANH,
             "LeakyRelu": L.ACT_LEAKY_RELU, "HardSigmoid": L.ACT_HARD_SIGMOID,
             "HardSwish": L.ACT_HARD_SWISH, "Gelu": L.ACT_GELU}
UNARY_EW = {"Relu": L.EW_RELU, "Clip": L.EW_CLIP, "Sigmoid": L.EW_SIGMOID, "Tanh": L.EW_TANH,
            "LeakyRelu": L.EW_LEAKY_RELU, "HardSigmoid": L.EW_HARD_SIGMOID,
            "HardSwish": L.EW_HARD_SWISH, "Erf": L.EW_ERF, "Gelu": L.EW_GELU}
BINARY_EW = {"Add": L.EW_ADD, "Sub": L.EW_SUB, "Mul": L.EW_MUL, "Div": L.EW_DIV}
ELEMENTWISE_OPS = set(UNARY_EW) | set(BINARY_EW)
ALIAS_OPS = {"Flatten", "Reshape", "Squeeze", "Unsqueeze", "Identity"}


def round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


@dataclass
class TensorSpec:
    """An activation tensor stored NHWC with channel stride ``cs``."""

    name: str
    shape: tuple          # logical (reference) shape, NCHW or (N, C)
    n: int
    c: int
    h: int
    w: int
    cs: int
    dtype: int
    alias_of: Optional[str] = None
    layout: str = "nhwc"   # "s2d2": 2x2 space-to-depth of a graph input (see space_to_depth_stem)

    @property
    def nbytes(self) -> int:
        return self.n * self.h * self.w * self.cs * L.ELEM_BYTES[self.dtype]


@dataclass
class Step:
    kind: str                      # "conv" | "pool" | "eltwise" | "copy" | "softmax" | "se"
    inputs: list                   # activation tensors read
    outputs: list                  # activation tensors written
    nodes: list                    # IR node names covered
    params: dict = field(default_factory=dict)

    def label(self) -> str:
        return f"{self.kind}[{'+'.join(self.nodes)}]"


@dataclass
class Lowered:
    steps: list
    tensors: dict                  # name -> TensorSpec
    weights: dict                  # name -> (desc, oihw fp32 array, bias fp32 array)
    consts: dict                   # name -> np.ndarray (eltwise operands uploaded once)
    inputs: list
    outputs: list
    shapes: dict
    dtype: int


def _is_scalar(arr) -> bool:
    return arr is not None and np.asarray(arr).size == 1


class _Lowerer:
    def __init__(self, graph, shapes: dict, dtype: int):
        self.g = graph
        self.shapes = shapes
        self.dtype = dtype
        self.consts = {}
        self.weights = {}
        self.tensors = {}
        self.steps = []
        self.order = graph.topo_sort()
        self.pos = {id(n): k for k, n in enumerate(self.order)}
        self.consumers = {}
        for n in self.order:
            for i in n.inputs:
                if i:
                    self.consumers.setdefault(i, []).append(n)
        self.graph_outputs = set(graph.outputs)
        self.absorbed = set()   # ids of nodes folded into another step
        self.deferred = {}      # id(node) -> Step to emit at that node's position

    # ---------------------------------------------------------- helpers
    def const(self, name):
        if not name:
            return None
        return self.g.initializers.get(name)

    def uses(self, name) -> int:
        return len(self.consumers.get(name, [])) + (1 if name in self.graph_outputs else 0)

    def tensor(self, name) -> TensorSpec:
        if name in self.tensors:
            return self.tensors[name]
        shp = tuple(self.shapes[name])
        if len(shp) == 4:
            n, c, h, w = shp
        elif len(shp) == 2:
            n, c, h, w = shp[0], shp[1], 1, 1
        elif len(shp) == 3:
            n, c, h, w = shp[0], shp[1], shp[2], 1
        else:
            raise LoweringError(f"tensor {name!r} of rank {len(shp)} is not supported")
        t = TensorSpec(name, shp, n, c, h, w, round_up(c, 16 if self.dtype in (L.U8, L.S8) else 8), self.dtype)
        self.tensors[name] = t
        return t

    # ---------------------------------------------------------- convs
    def conv_step(self, node):
        op, a = node.op_type, node.attrs
        x = node.inputs[0]
        xt = self.tensor(x)
        if op in ("Conv", "FusedConvAct", "FusedConvBNAct"):
            w = self.const(node.inputs[1])
            if w is None:
                raise LoweringError(f"{node.name}: conv weight must be constant")
            b = self.const(node.inputs[2]) if len(node.inputs) > 2 and node.inputs[2] else None
            if len(node.inputs) > 2 and node.inputs[2] and b is None:
                raise LoweringError(f"{node.name}: conv bias must be constant")
            oh, ow, (pt, pb), (pl, pr) = S.conv_geometry(a, (xt.n, xt.c, xt.h, xt.w), w.shape)
            k, icg, r, s = w.shape
            group = a.get("group", 1)
            sh, sw = a.get("strides", [1, 1])
            dh, dw = a.get("dilations", [1, 1])
            if group != 1 and (xt.c % group or k % group or icg * group != xt.c):
                raise LoweringError(f"{node.name}: grouped conv with group={group} does not divide "
                                    f"C={xt.c} / K={k}")
            wt = np.asarray(w, dtype=np.float32)
            geom = dict(n=xt.n, h=xt.h, w=xt.w, c=xt.c, k=k, r=r, s=s, sh=sh, sw=sw, pt=pt, pl=pl,
                        dh=dh, dw=dw, oh=oh, ow=ow, groups=group)
        else:  # Gemm / FusedGemmAct / MatMul: y[M,N] = x[M,K] . W[N,K]^T
            if op == "MatMul":
                B = self.const(node.inputs[1])
                if B is None or B.ndim != 2:
                    raise LoweringError(f"{node.name}: MatMul needs a constant 2-D right operand")
                wt, b = np.asarray(B, np.float32).T, None
                alpha, beta = 1.0, 1.0
            else:
                if a.get("transA", 0):
                    # the activation is [K, M]: a transpose step makes it [M, K]
                    k_, m_ = (int(v) for v in self.shapes[x])
                    xT = f"{node.name}.A_T"
                    self.shapes[xT] = (m_, k_)
                    self.steps.append(self.transpose_step(f"{node.name}.transA", x, xT, [1, 0]))
                    self.tensor(xT)
                    x = xT
                    xt = self.tensor(xT)
                B = self.const(node.inputs[1])
                if B is None:
                    raise LoweringError(f"{node.name}: Gemm weight must be constant")
                wt = np.asarray(B, np.float32)
                wt = wt if a.get("transB", 0) else wt.T
                alpha, beta = float(a.get("alpha", 1.0)), float(a.get("beta", 1.0))
                b = self.const(node.inputs[2]) if len(node.inputs) > 2 and node.inputs[2] else None
                if len(node.inputs) > 2 and node.inputs[2] and b is None:
                    raise LoweringError(f"{node.name}: Gemm C must be constant")
                if b is not None:
                    b = np.asarray(b, np.float32)
                    if b.size not in (1, wt.shape[0]) or (b.ndim == 2 and b.shape[0] != 1):
                        raise LoweringError(f"{node.name}: Gemm C of shape {b.shape} (full matrix) "
                                            "is not supported")
                    b = np.broadcast_to(b.reshape(-1), (wt.shape[0],)) * np.float32(beta)
            if xt.h * xt.w != 1:
                raise LoweringError(f"{node.name}: GEMM input must be 2-D")
            if alpha != 1.0:
                wt = wt * np.float32(alpha)
            k, kin = wt.shape
            if kin != xt.c:
                raise LoweringError(f"{node.name}: GEMM inner dim {kin} != {xt.c}")
            wt = wt.reshape(k, kin, 1, 1)
            geom = dict(n=xt.n, h=1, w=1, c=xt.c, k=k, r=1, s=1, sh=1, sw=1, pt=0, pl=0, dh=1, dw=1,
                        oh=1, ow=1, groups=1)
        geom["flops"] = 2.0 * geom["n"] * geom["oh"] * geom["ow"] * geom["k"] * (geom["c"] // geom["groups"]) \
            * geom["r"] * geom["s"]   # algorithmic work of the node as written in the graph
        # the (M, N, K) the reference codegen passes to its schedule hook for this
        # node (mdlc/codegen/cuda/emit.py:202 conv: (OC, OH*OW, C/g*KH*KW) per
        # image; :225 Gemm / :240 MatMul: (rows, out features, in features)),
        # and which of M / N is the output-channel axis
        if op in ("Conv", "FusedConvAct", "FusedConvBNAct"):
            geom["ref_mnk"] = (geom["k"], geom["oh"] * geom["ow"], (geom["c"] // geom["groups"]) * geom["r"] * geom["s"])
            geom["ref_channel_axis"] = "M"
        else:
            geom["ref_mnk"] = (geom["n"], geom["k"], geom["c"])
            geom["ref_channel_axis"] = "N"
        bias = np.zeros(round_up(geom["k"], 16), np.float32)
        if b is not None:
            bias[:geom["k"]] = np.asarray(b, np.float32).reshape(-1)
        wname = f"{node.name or node.outputs[0]}.w"
        self.weights[wname] = (geom, wt, bias)
        act = a.get("activation") if op.startswith("Fused") else None
        return Step("conv", [x], [node.outputs[0]], [node.name],
                    dict(weight=wname, act=act, attrs=dict(a), residual=None))

    def try_absorb_residual(self, node, step):
        """Plain conv whose only consumer is Add(conv, skip) [+ activation]."""
        t = node.outputs[0]
        if self.uses(t) != 1 or t in self.graph_outputs:
            return None
        cons = self.consumers[t][0]
        if id(cons) in self.absorbed:      # already fused into another conv's epilogue
            return None
        skip = act = None
        act_attrs = {}
        out = None
        if cons.op_type == "Add" and len(cons.real_inputs()) == 2:
            other = [i for i in cons.inputs if i != t]
            if len(other) != 1 or self.const(other[0]) is not None:
                return None
            skip, out = other[0], cons.outputs[0]
        elif cons.op_type == "FusedElementwise":
            sub = cons.attrs["subgraph"]
            if not (1 <= len(sub) <= 2 and sub[0].op_type == "Add") or len(cons.outputs) != 1:
                return None
            add = sub[0]
            other = [i for i in add.inputs if i != t]
            if t not in add.inputs or len(other) != 1 or self.const(other[0]) is not None:
                return None
            skip = other[0]
            if len(sub) == 2:
                a2 = sub[1]
                if a2.op_type not in ACT_CODES or a2.inputs[0] != add.outputs[0]:
                    return None
                act = a2.op_type
                if act == "Clip":
                    lo = self._scalar_input(a2, 1, a2.attrs.get("min"))
                    hi = self._scalar_input(a2, 2, a2.attrs.get("max"))
                    if lo is False or hi is False:
                        return None
                    act_attrs = {"clip_min": lo, "clip_max": hi}
                elif act in ("LeakyRelu", "HardSigmoid"):
                    act_attrs = {k: v for k, v in a2.attrs.items() if k in ("alpha", "beta")}
                out = a2.outputs[0]
            else:
                out = add.outputs[0]
            if cons.outputs[0] != out:
                return None
        else:
            return None
        if tuple(self.shapes[skip]) != tuple(self.shapes[t]):
            return None
        step.inputs.append(skip)
        step.outputs = [out]
        step.nodes.append(cons.name)
        step.params["residual"] = skip
        step.params["act"] = act
        step.params["attrs"].update(act_attrs)
        return cons

    def try_absorb_gelu(self, node, step):
        """conv -> Div(t, sqrt2) -> Erf -> (Add 1, Mul t, Mul 0.5) as a GELU epilogue."""
        t = node.outputs[0]
        if t in self.graph_outputs:
            return None
        cons = self.consumers.get(t, [])
        if len(cons) != 2:
            return None
        div = next((c for c in cons if c.op_type == "Div" and c.inputs[0] == t), None)
        if div is None or not _is_scalar(self.const(div.inputs[1])):
            return None
        if not math.isclose(float(np.asarray(self.const(div.inputs[1])).item()), math.sqrt(2.0),
                            rel_tol=1e-6):
            return None
        erf_nodes = self.consumers.get(div.outputs[0], [])
        if len(erf_nodes) != 1 or erf_nodes[0].op_type != "Erf" or self.uses(div.outputs[0]) != 1:
            return None
        erf = erf_nodes[0]
        tail = self.consumers.get(erf.outputs[0], [])
        other = next(c for c in cons if c is not div)
        if id(other) in self.absorbed:
            return None
        if len(tail) != 1 or tail[0] is not other or other.op_type != "FusedElementwise":
            return None
        sub = other.attrs["subgraph"]
        if [s.op_type for s in sub] != ["Add", "Mul", "Mul"] or len(other.outputs) != 1:
            return None
        add, m1, m2 = sub
        e = erf.outputs[0]

        def const_is(name, val):
            c = self.const(name)
            return _is_scalar(c) and math.isclose(float(np.asarray(c).item()), val, rel_tol=1e-6)

        ok = (e in add.inputs and any(const_is(i, 1.0) for i in add.inputs if i != e)
              and set(m1.inputs) == {t, add.outputs[0]}
              and m1.outputs[0] in m2.inputs and any(const_is(i, 0.5) for i in m2.inputs if i != m1.outputs[0])
              and other.outputs[0] == m2.outputs[0])
        if not ok:
            return None
        step.outputs = [other.outputs[0]]
        step.nodes += [div.name, erf.name, other.name]
        step.params["act"] = "Gelu"
        self.absorbed.update({id(div), id(erf)})
        return other

    def _scalar_input(self, node, idx, fallback):
        if len(node.inputs) > idx and node.inputs[idx]:
            c = self.const(node.inputs[idx])
            if not _is_scalar(c):
                return False
            return float(np.asarray(c).item())
        return None if fallback is None else float(fallback)

    # ---------------------------------------------------------- elementwise
    def eltwise_step(self, node, sub, ext_inputs, outputs):
        """Compile an elementwise (sub)graph into an interpreter program."""
        out_shape = tuple(self.shapes[outputs[0]])
        for o in outputs:
            if tuple(self.shapes[o]) != out_shape:
                raise LoweringError(f"{node.name}: elementwise outputs of different shapes")
        o4 = self.tensor(outputs[0])
        reg_of, tensor_inputs, bcast = {}, [], []
        imm = {}
        for e in ext_inputs:
            c = self.const(e)
            if _is_scalar(c):
                imm[e] = float(np.asarray(c).item())
                continue
            if c is not None:
                cshape = tuple(np.asarray(c).shape)
                full = (1, o4.c, 1, 1)
                cc = np.asarray(c, np.float32)
                if cc.size == o4.c and cc.reshape(-1).shape[0] == o4.c and len(cshape) in (1, 3, 4):
                    cname = f"{node.name}.{e}"
                    padded = np.zeros(o4.cs, np.float32)
                    padded[:o4.c] = cc.reshape(-1)
                    self.consts[cname] = padded
                    mode, src = L.BC_C, cname
                else:
                    raise LoweringError(f"{node.name}: constant operand {e!r} of shape {cshape} vs {full}")
            else:
                shp = tuple(self.shapes[e])
                t = self.tensor(e)
                if shp == out_shape:
                    mode = L.BC_FULL
                elif t.n == o4.n and t.c == o4.c and t.h * t.w == 1:
                    mode = L.BC_NC
                elif t.n == 1 and t.c == o4.c and t.h * t.w == 1:
                    mode = L.BC_C
                elif int(np.prod(shp)) == 1:
                    mode = L.BC_SCALAR
                else:
                    raise LoweringError(f"{node.name}: operand {e!r} {shp} does not broadcast to {out_shape}")
                src = e
            if len(tensor_inputs) >= L.EW_MAX_INPUTS:
                raise LoweringError(f"{node.name}: more than {L.EW_MAX_INPUTS} tensor operands")
            reg_of[e] = len(tensor_inputs)
            tensor_inputs.append(src)
            bcast.append(mode)
        code = []
        free_regs = [r for r in range(8) if r >= len(tensor_inputs)]
        remaining = {}
        for sn in sub:
            for i in sn.real_inputs():
                remaining[i] = remaining.get(i, 0) + 1

        def alloc():
            if not free_regs:
                raise LoweringError(f"{node.name}: elementwise program needs more than 8 registers")
            return free_regs.pop(0)

        for sn in sub:
            op, ins = sn.op_type, [i for i in sn.inputs if i]
            if op in BINARY_EW:
                a_, b_ = ins[0], ins[1]
                if a_ in imm and b_ in imm:
                    raise LoweringError(f"{sn.name}: constant-only elementwise node")
                if b_ in imm:
                    opc = {"Add": L.EW_ADDI, "Sub": L.EW_SUBI, "Mul": L.EW_MULI, "Div": L.EW_DIVI}[op]
                    ins_code = (opc, reg_of[a_], 0, imm[b_], 0.0)
                elif a_ in imm:
                    opc = {"Add": L.EW_ADDI, "Sub": L.EW_RSUBI, "Mul": L.EW_MULI, "Div": L.EW_RDIVI}[op]
                    ins_code = (opc, reg_of[b_], 0, imm[a_], 0.0)
                else:
                    ins_code = (BINARY_EW[op], reg_of[a_], reg_of[b_], 0.0, 0.0)
            elif op in UNARY_EW:
                i0 = i1 = 0.0
                if op == "Clip":
                    lo = self._scalar_input(sn, 1, sn.attrs.get("min"))
                    hi = self._scalar_input(sn, 2, sn.attrs.get("max"))
                    if lo is False or hi is False:
                        raise LoweringError(f"{sn.name}: Clip bounds must be constant scalars")
                    i0 = -np.inf if lo is None else lo
                    i1 = np.inf if hi is None else hi
                elif op == "LeakyRelu":
                    i0 = float(sn.attrs.get("alpha", 0.01))
                elif op == "HardSigmoid":
                    i0, i1 = float(sn.attrs.get("alpha", 0.2)), float(sn.attrs.get("beta", 0.5))
                ins_code = (UNARY_EW[op], reg_of[ins[0]], 0, i0, i1)
            else:
                raise LoweringError(f"{sn.name}: {op} inside an elementwise group")
            for i in sn.real_inputs():
                remaining[i] -= 1
                if remaining[i] == 0 and i in reg_of and i not in outputs and reg_of[i] >= len(tensor_inputs):
                    free_regs.append(reg_of[i])
                    free_regs.sort()
            dst = alloc()
            reg_of[sn.outputs[0]] = dst
            opc, s0, s1, f0, f1 = ins_code
            code.append((opc, dst, s0, s1, f0, f1))
        if len(code) > L.EW_MAX_INSTR:
            raise LoweringError(f"{node.name}: elementwise program longer than {L.EW_MAX_INSTR}")
        if len(outputs) > L.EW_MAX_OUTPUTS:
            raise LoweringError(f"{node.name}: more than {L.EW_MAX_OUTPUTS} outputs")
        return Step("eltwise", [s for s in tensor_inputs if s not in self.consts], list(outputs), [node.name],
                    dict(code=code, operands=tensor_inputs, bcast=bcast,
                         out_regs=[reg_of[o] for o in outputs]))

    # ---------------------------------------------------------- main walk
    def run(self) -> Lowered:
        for name in self.g.runtime_inputs:
            self.tensor(name)
        for node in self.order:
            if id(node) in self.absorbed:
                if id(node) in self.deferred:
                    self.steps.append(self.deferred.pop(id(node)))
                continue
            op = node.op_type
            if op in ("Conv", "FusedConvAct", "FusedConvBNAct", "Gemm", "FusedGemmAct", "MatMul"):
                step = self.conv_step(node)
                self.tensor(node.outputs[0])
                absorbed = None
                if not step.params["act"]:
                    absorbed = self.try_absorb_residual(node, step) or self.try_absorb_gelu(node, step)
                if absorbed is not None:
                    self.absorbed.add(id(absorbed))
                    self.deferred[id(absorbed)] = step
                    for o in step.outputs:
                        self.tensor(o)
                else:
                    self.steps.append(step)
            elif op in ("MaxPool", "AveragePool"):
                xt = self.tensor(node.inputs[0])
                oh, ow, (pt, pb), (pl, pr) = S.pool_geometry(node.attrs, (xt.n, xt.c, xt.h, xt.w),
                                                             op == "MaxPool")
                if op == "MaxPool" and node.attrs.get("dilations", [1, 1]) != [1, 1]:
                    raise LoweringError(f"{node.name}: dilated MaxPool")
                kh, kw = node.attrs["kernel_shape"]
                sh, sw = node.attrs.get("strides", [1, 1])
                if op == "AveragePool" and node.attrs.get("count_include_pad", 0) and (pb > pt or pr > pl):
                    raise LoweringError(f"{node.name}: asymmetric count_include_pad AveragePool")
                self.tensor(node.outputs[0])
                self.steps.append(Step("pool", [node.inputs[0]], [node.outputs[0]], [node.name],
                                       dict(kind=0 if op == "MaxPool" else 1, kh=kh, kw=kw, sh=sh, sw=sw,
                                            pt=pt, pl=pl, oh=oh, ow=ow,
                                            cip=int(node.attrs.get("count_include_pad", 0)))))
            elif op == "GlobalAveragePool" or (
                    op == "ReduceMean" and self._reduce_axes(node) == [2, 3]
                    and node.attrs.get("keepdims", 1)):
                self.tensor(node.inputs[0])
                self.tensor(node.outputs[0])
                self.steps.append(Step("pool", [node.inputs[0]], [node.outputs[0]], [node.name], dict(kind=2)))
            elif op == "BatchNormalization":
                self.steps.append(self.batchnorm_step(node))
            elif op == "Softmax":
                rank = len(self.shapes[node.inputs[0]])
                self.tensor(node.inputs[0])
                self.tensor(node.outputs[0])
                axis = int(node.attrs.get("axis", -1)) % rank
                self.steps.append(Step("softmax", [node.inputs[0]], [node.outputs[0]], [node.name],
                                       dict(axis=axis, batch_mixing=axis == 0)))
            elif op == "Transpose":
                x = node.inputs[0]
                rank = len(self.shapes[x])
                perm = [int(v) for v in node.attrs.get("perm", list(range(rank))[::-1])]
                self.tensor(x)
                self.tensor(node.outputs[0])
                self.steps.append(self.transpose_step(node.name, x, node.outputs[0], perm))
            elif op == "Pad":
                self.steps.append(self.pad_step(node))
            elif op == "Concat":
                self.steps.append(self.concat_step(node))
            elif op in ALIAS_OPS:
                src = self.tensor(node.inputs[0])
                out_shape = tuple(self.shapes[node.outputs[0]])
                dst = self.tensor(node.outputs[0])
                same_order = (src.h * src.w == 1 and dst.h * dst.w == 1 and src.c == dst.c) or \
                    (tuple(src.shape) == out_shape)
                if not same_order or src.n != dst.n:
                    raise LoweringError(f"{node.name}: {op} {src.shape}->{out_shape} changes NHWC order")
                dst.alias_of = src.alias_of or src.name
            elif op == "FusedElementwise":
                sub = node.attrs["subgraph"]
                for o in node.outputs:
                    self.tensor(o)
                self.steps.append(self.eltwise_step(node, sub, list(node.inputs), list(node.outputs)))
            elif op in ELEMENTWISE_OPS:
                self.tensor(node.outputs[0])
                self.steps.append(self.eltwise_step(node, [node], node.real_inputs(), [node.outputs[0]]))
            else:
                raise LoweringError(f"no B200 lowering for op {op!r} (node {node.name!r})")
        if self.deferred:
            raise LoweringError("internal: unplaced fused step")
        return Lowered(self.steps, self.tensors, self.weights, self.consts, list(self.g.runtime_inputs),
                       list(self.g.outputs), self.shapes, self.dtype)

    # ---------------------------------------------------------- data movement
    def transpose_step(self, name, x, y, perm):
        """out axis i reads source axis perm[i] (ONNX Transpose, ops.py:229-230);
        the axes past the tensor's rank (h, w of a 2-D one) stay in place."""
        rank = len(perm)
        if rank > 4 or sorted(perm) != list(range(rank)):
            raise LoweringError(f"{name}: Transpose perm {perm} is not a permutation of rank <= 4")
        src_dim = list(perm) + list(range(rank, 4))
        part = dict(src=x, mode=0, src_dim=src_dim, offset=[0, 0, 0, 0], pad_mode=0, value=0.0)
        return Step("copy", [x], [y], [name], dict(parts=[part], batch_mixing=perm[0] != 0))

    def pad_step(self, node):
        """ONNX Pad (ops.py:249-255): constant / edge / reflect over up to 4 axes."""
        x, y = node.inputs[0], node.outputs[0]
        rank = len(self.shapes[x])
        pads = self.const(node.inputs[1]) if len(node.inputs) > 1 and node.inputs[1] else node.attrs.get("pads")
        if pads is None:
            raise LoweringError(f"{node.name}: Pad needs constant pads")
        pads = [int(v) for v in np.asarray(pads).ravel()]
        val = self.const(node.inputs[2]) if len(node.inputs) > 2 and node.inputs[2] else node.attrs.get("value", 0.0)
        if len(node.inputs) > 2 and node.inputs[2] and val is None:
            raise LoweringError(f"{node.name}: Pad value must be constant")
        mode = node.attrs.get("mode", "constant")
        if isinstance(mode, bytes):
            mode = mode.decode()
        if mode not in ("constant", "edge", "reflect") or len(pads) != 2 * rank or rank > 4:
            raise LoweringError(f"{node.name}: Pad mode {mode!r} / pads {pads} not supported")
        self.tensor(x)
        self.tensor(y)
        begin = pads[:rank] + [0] * (4 - rank)
        part = dict(src=x, mode=0, src_dim=[0, 1, 2, 3], offset=begin,
                    pad_mode={"constant": 0, "edge": 1, "reflect": 2}[mode],
                    value=float(np.asarray(0.0 if val is None else val).item()))
        return Step("copy", [x], [y], [node.name], dict(parts=[part], batch_mixing=pads[0] != 0 or pads[rank] != 0))

    def concat_step(self, node):
        """ONNX Concat (ops.py:233-234): the first input gathered into the output
        (zero elsewhere), every other one scattered at its offset along the axis."""
        ins, y = [i for i in node.inputs if i], node.outputs[0]
        rank = len(self.shapes[y])
        axis = int(node.attrs.get("axis", 0)) % rank
        if rank > 4:
            raise LoweringError(f"{node.name}: Concat of rank {rank}")
        for i in ins:
            if self.const(i) is not None:
                raise LoweringError(f"{node.name}: Concat of a constant operand")
            self.tensor(i)
        self.tensor(y)
        parts, off = [], 0
        for k, i in enumerate(ins):
            offset = [0, 0, 0, 0]
            offset[axis] = off
            parts.append(dict(src=i, mode=0 if k == 0 else 1, src_dim=[0, 1, 2, 3], offset=offset,
                              pad_mode=0, value=0.0))
            off += int(self.shapes[i][axis])
        return Step("copy", list(ins), [y], [node.name], dict(parts=parts, batch_mixing=axis == 0))

    def batchnorm_step(self, node):
        """Inference BatchNormalization (ops.py:95-106) not folded into a conv:
        y = x * s + t per channel, s = scale / sqrt(var + eps), t = bias - mean * s."""
        x, y = node.inputs[0], node.outputs[0]
        prm = [self.const(i) for i in node.inputs[1:5]]
        if any(p is None for p in prm):
            raise LoweringError(f"{node.name}: BatchNormalization parameters must be constant")
        scale, bias, mean, var = (np.asarray(p, np.float64).reshape(-1) for p in prm)
        eps = float(node.attrs.get("epsilon", 1e-5))
        sc = scale / np.sqrt(var + eps)
        sh = bias - mean * sc
        xt = self.tensor(x)
        self.tensor(y)
        names = []
        for tag, arr in (("scale", sc), ("shift", sh)):
            padded = np.zeros(xt.cs, np.float32)
            padded[:xt.c] = arr.astype(np.float32)
            cname = f"{node.name}.{tag}"
            self.consts[cname] = padded
            names.append(cname)
        code = [(L.EW_MUL, 3, 0, 1, 0.0, 0.0), (L.EW_ADD, 3, 3, 2, 0.0, 0.0)]
        return Step("eltwise", [x], [y], [node.name],
                    dict(code=code, operands=[x] + names, bcast=[L.BC_FULL, L.BC_C, L.BC_C], out_regs=[3]))

    def _reduce_axes(self, node):
        axes = node.attrs.get("axes")
        if axes is None and len(node.inputs) > 1 and node.inputs[1]:
            axes = [int(v) for v in np.asarray(self.const(node.inputs[1])).ravel()]
        rank = len(self.shapes[node.inputs[0]])
        return sorted(int(a) % rank for a in axes) if axes is not None else None


def s2d_weights(wt: np.ndarray, pad_t: int, pad_l: int):
    """Re-index a stride-2 conv's OIHW weights for a 2x2 space-to-depth input.

    With X'[(dy, dx, c), Y, X] = x[c, 2Y + dy, 2X + dx], the tap r of the
    original kernel reads row 2*oy + r - pad_t = 2*(oy + ty) + dy with
    ty = floor((r - pad_t) / 2), dy = (r - pad_t) mod 2. The same conv is
    therefore a stride-1 conv over X' with taps Ty = ty + ceil(pad_t / 2),
    weight W'[o, (dy*2 + dx)*C + c, Ty, Tx] = w[o, c, r, s] (zero where r or s
    falls outside the original kernel) and top/left padding ceil(pad / 2).
    Returns (W', new_pad_t, new_pad_l).
    """
    k, c, R, S = wt.shape
    pt2, pl2 = -(-pad_t // 2), -(-pad_l // 2)
    R2 = (R - 1 - pad_t) // 2 + pt2 + 1
    S2 = (S - 1 - pad_l) // 2 + pl2 + 1
    out = np.zeros((k, 4 * c, R2, S2), np.float32)
    for r in range(R):
        ty, dy = divmod(r - pad_t, 2)
        for s_ in range(S):
            tx, dx = divmod(s_ - pad_l, 2)
            out[:, (dy * 2 + dx) * c:(dy * 2 + dx + 1) * c, ty + pt2, tx + pl2] = wt[:, :, r, s_]
    return out, pt2, pl2


def space_to_depth_stem(lo: Lowered) -> None:
    """Rewrite a stride-2 conv that reads a graph input with <= 4 channels
    (the stem) as a stride-1 conv over the input's 2x2 space-to-depth form.

    The graph-input conversion kernel writes the space-to-depth layout
    directly, so the rewrite costs nothing at run time; it shrinks the
    reduction from R*S*8 to about R*S*16/4 elements and makes every filter tap
    a contiguous 32-byte run (16 bf16 channels, or 32 8-bit channels) that the
    im2col tensor-memory-accelerator path loads whole.
    """
    for name in lo.inputs:
        t = lo.tensors.get(name)
        if t is None or t.c > 4 or t.h % 2 or t.w % 2 or t.h * t.w == 1:
            continue
        readers = [st for st in lo.steps if name in st.inputs]
        if len(readers) != 1 or readers[0].kind != "conv" or name in lo.outputs:
            continue
        st = readers[0]
        if st.params.get("residual") or st.inputs[0] != name:
            continue
        geom, wt, bias = lo.weights[st.params["weight"]]
        if geom["groups"] != 1 or geom["sh"] != 2 or geom["sw"] != 2 or geom["dh"] != 1 or geom["dw"] != 1:
            continue
        w2, pt2, pl2 = s2d_weights(wt, geom["pt"], geom["pl"])
        cs = 32 if t.dtype in (L.U8, L.S8) else 16      # 32-byte pixels either way
        g2 = dict(geom, h=geom["h"] // 2, w=geom["w"] // 2, c=4 * geom["c"], cs=cs, r=w2.shape[2],
                  s=w2.shape[3], sh=1, sw=1, pt=pt2, pl=pl2, pt_orig=geom["pt"], pl_orig=geom["pl"])
        lo.weights[st.params["weight"]] = (g2, w2, bias)
        t.layout, t.c, t.h, t.w, t.cs = "s2d2", 4 * t.c, t.h // 2, t.w // 2, cs
        st.params["s2d"] = True


def pair_weights(wt: np.ndarray, cs: int, pad_l: int):
    """Re-index a stride-1 conv's OIHW weights for column pairing.

    The input [N, H, W, cs] is read as [N, H, W/2, 2cs] (super-pixels of two
    horizontally adjacent pixels: the same bytes) and the output [N, OH, OW, K]
    as [N, OH, OW/2, 2K]: output super-pixel p holds output columns 2p + q,
    q in {0, 1}. Output column 2p + q, tap s reads input column 2p + q + s - pad_l,
    i.e. super-pixel p + s' - pad_l' half `sub` with 2 s' - 2 pad_l' + sub =
    q + s - pad_l, so the paired conv has S' = floor((S - pad_l) / 2) +
    ceil(pad_l / 2) + 1 taps, left padding pad_l' = ceil(pad_l / 2) and
    W'[q K + o, sub cs + c, r, s'] = w[o, c, r, 2 s' - 2 pad_l' + sub - q + pad_l]
    where that tap exists (zero elsewhere, and for the padding channels
    c >= C). Returns (W', S', pad_l')."""
    k, c, R, S = wt.shape
    pl2 = -(-pad_l // 2)
    S2 = (S - pad_l) // 2 + pl2 + 1
    out = np.zeros((2 * k, 2 * cs, R, S2), np.float32)
    for q in range(2):
        for s2 in range(S2):
            for sub in range(2):
                s_ = 2 * s2 - 2 * pl2 + sub - q + pad_l
                if 0 <= s_ < S:
                    out[q * k:(q + 1) * k, sub * cs:sub * cs + c, :, s2] = wt[:, :, :, s_]
    return out, S2, pl2


def pair_stem_columns(lo: Lowered) -> None:
    """Compute the space-to-depth stem two output columns per GEMM row.

    After the space-to-depth rewrite the stem is a 4x4 stride-1 conv over
    16-channel (32-byte) pixels with 64 outputs: its A operand arrives as 16
    small per-tap TMA loads per 128-pixel tile and its MMAs are only 64 wide.
    Paired (see pair_weights), the same bytes are a 4x3 conv over 32-channel
    super-pixels with 128 outputs: 64-byte taps, 128-wide MMAs, 12 loads per
    256 output pixels instead of 32. The output keeps its tensor (identical
    bytes); per-channel epilogue parameters are duplicated for the two output
    columns (int8: by the executable, the quantisation plan keeps the graph's K)."""
    for st in lo.steps:
        if st.kind != "conv" or not st.params.get("s2d") or st.params.get("residual"):
            continue
        geom, wt, bias = lo.weights[st.params["weight"]]
        k = geom["k"]
        if (geom["sh"], geom["sw"], geom["dh"], geom["dw"]) != (1, 1, 1, 1) or geom["w"] % 2 or geom["ow"] % 2 \
                or k % 8 or geom["groups"] != 1:
            continue
        cs = geom["cs"]
        w2, s2, pl2 = pair_weights(wt, cs, geom["pl"])
        b2 = np.zeros(round_up(2 * k, 16), np.float32)
        b2[:k] = bias[:k]
        b2[k:2 * k] = bias[:k]
        g2 = dict(geom, w=geom["w"] // 2, c=2 * cs, cs=2 * cs, k=2 * k, s=s2, pl=pl2, ow=geom["ow"] // 2,
                  paired=True, cs_unpaired=cs, pl_unpaired=geom["pl"], k_unpaired=k)
        lo.weights[st.params["weight"]] = (g2, w2, b2)
        st.params["paired"] = True


def _is_fc_step(lo: Lowered, st: Step) -> bool:
    if st.kind != "conv" or st.params.get("residual") or st.params.get("s2d"):
        return False
    g = lo.weights[st.params["weight"]][0]
    return (g["r"], g["s"], g["h"], g["w"], g["oh"], g["ow"], g["groups"]) == (1, 1, 1, 1, 1, 1, 1) \
        and not g.get("paired")


def fuse_squeeze_excite(lo: Lowered) -> None:
    """Two 1x1 convs on a 1x1 map in a row, the first's output read only by
    the second and the second's channel count equal to the first's input
    channels (FC, act, FC, act of a squeeze-excite gate): one "se" step, run by
    mdlc_se_fc. The weights leave ``lo.weights`` (they are not conv-packed):
    w1 [rd][c] and w2 transposed, [rd][c], with the biases, go into the step.
    A global average pool whose output only the gate reads is absorbed too:
    the step then reads the pool's input and averages it in the same kernel."""
    readers = {}
    for st in lo.steps:
        for t in st.inputs:
            readers[t] = readers.get(t, 0) + 1
        if st.params.get("residual"):
            readers[st.params["residual"]] = readers.get(st.params["residual"], 0) + 1
    out, i = [], 0
    while i < len(lo.steps):
        a = lo.steps[i]
        b = lo.steps[i + 1] if i + 1 < len(lo.steps) else None
        if (b is not None and _is_fc_step(lo, a) and _is_fc_step(lo, b) and b.inputs[0] == a.outputs[0]
                and readers.get(a.outputs[0], 0) == 1 and a.outputs[0] not in lo.outputs
                and b.outputs[0] not in lo.outputs):
            ga, wa, ba = lo.weights[a.params["weight"]]
            gb, wb, bb = lo.weights[b.params["weight"]]
            c, rd = ga["c"], ga["k"]
            if gb["c"] == rd and gb["k"] == c and c <= 4096 and rd <= 1024:
                del lo.weights[a.params["weight"]], lo.weights[b.params["weight"]]
                src, nodes = a.inputs[0], a.nodes + b.nodes
                g = out[-1] if out else None
                if (g is not None and g.kind == "pool" and g.params["kind"] == 2 and g.outputs[0] == src
                        and readers.get(src, 0) == 1 and src not in lo.outputs):
                    out.pop()
                    src, nodes = g.inputs[0], g.nodes + nodes
                out.append(Step("se", [src], [b.outputs[0]], nodes, dict(
                    w1=np.ascontiguousarray(np.asarray(wa, np.float32).reshape(rd, c)),
                    b1=np.ascontiguousarray(ba[:rd], np.float32),
                    w2t=np.ascontiguousarray(np.asarray(wb, np.float32).reshape(c, rd).T),
                    b2=np.ascontiguousarray(bb[:c], np.float32),
                    act1=a.params["act"], attrs1=a.params["attrs"], act2=b.params["act"], attrs2=b.params["attrs"],
                    flops=ga["flops"] + gb["flops"])))
                i += 2
                continue
        out.append(a)
        i += 1
    lo.steps = out


def lower(graph, shapes: dict, dtype: int, s2d: bool = True, fuse_se: bool = True) -> Lowered:
    """Lower a post-pass graph to backend steps. For 8-bit lowering the graph
    inputs are signed (symmetric int8, zero point 0: padded taps read real
    zeros) and every other activation is unsigned."""
    lo = _Lowerer(graph, shapes, dtype).run()
    if dtype == L.U8:
        for name in lo.inputs:
            lo.tensors[name].dtype = L.S8
    if s2d:
        space_to_depth_stem(lo)
        # Pairing buys 128-wide MMAs and fewer, larger loads at the price of
        # 1.5x the reduction length (4x3 super-pixel taps hold 4x4 useful
        # ones); measured faster for every dtype, fp32 (3xTF32) included
        # (ResNet-18 b=256 fp32 stem: 1466 us paired, 1680 us unpaired)
        pair_stem_columns(lo)
    if fuse_se and dtype in (L.BF16, L.F32):
        fuse_squeeze_excite(lo)
    return lo
