"""Graph IR types accepted by :func:`mdlc_b200.compiler.compile`.

The backend consumes the reference compiler's post-pass Graph IR
(``mdlc/ir/graph.py``, ``mdlc/ir/node.py``, ``mdlc/ir/tensor.py``) by duck
typing: any object with ``nodes``, ``inputs``, ``outputs``, ``initializers``,
``value_info`` and ``topo_sort()`` works, so a graph produced by the reference's
own ``default_pipeline()`` can be passed straight in.

This module holds a small standalone implementation of the same interface so
that model builders, the pass pipeline and the benchmark can produce graphs on
machines where the reference package is not installed. Field names, the empty
string convention for omitted inputs (``mdlc/ir/node.py:10-12``) and the
Kahn topological order (``mdlc/ir/graph.py:99-138``: FIFO over nodes whose
producers are done, seeded in node-list order) are kept identical because the
memory planner's buffer assignment depends on that order.
"""

from __future__ import annotations

from collections import defaultdict, deque
from dataclasses import dataclass, field
from typing import Any, Iterable, Optional

import numpy as np

FLOAT32 = "float32"
FLOAT16 = "float16"
INT64 = "int64"
INT32 = "int32"
INT8 = "int8"
BOOL = "bool"

_NP = {FLOAT32: np.float32, FLOAT16: np.float16, INT64: np.int64,
       INT32: np.int32, INT8: np.int8, BOOL: np.bool_}


def dtype_from_numpy(dt) -> str:
    dt = np.dtype(dt)
    for name, t in _NP.items():
        if np.dtype(t) == dt:
            return name
    return FLOAT32


@dataclass
class TensorInfo:
    """Static type/shape of one named edge (``mdlc/ir/tensor.py:56-98``)."""

    name: str
    dtype: str = FLOAT32
    shape: tuple = ()

    @property
    def is_static(self) -> bool:
        return all(isinstance(d, (int, np.integer)) and d >= 0 for d in self.shape)

    def numel(self) -> Optional[int]:
        if not self.is_static:
            return None
        return int(np.prod([int(d) for d in self.shape], dtype=np.int64)) if self.shape else 1


@dataclass
class Node:
    """One operator (``mdlc/ir/node.py:8-49``)."""

    op_type: str
    inputs: list = field(default_factory=list)
    outputs: list = field(default_factory=list)
    attrs: dict = field(default_factory=dict)
    name: str = ""
    fused_from: Optional[list] = None

    def attr(self, key: str, default: Any = None) -> Any:
        return self.attrs.get(key, default)

    @property
    def is_fused(self) -> bool:
        return self.fused_from is not None

    def real_inputs(self) -> list:
        return [i for i in self.inputs if i]

    def replace_input(self, old: str, new: str) -> None:
        self.inputs = [new if i == old else i for i in self.inputs]


class Graph:
    """Dataflow graph over named edges (``mdlc/ir/graph.py:13-190``)."""

    def __init__(self, name: str = "graph") -> None:
        self.name = name
        self.nodes: list = []
        self.inputs: list = []
        self.outputs: list = []
        self.initializers: dict = {}
        self.value_info: dict = {}

    def add_node(self, node: Node) -> Node:
        self.nodes.append(node)
        return node

    def set_info(self, info: TensorInfo) -> None:
        self.value_info[info.name] = info

    def info(self, name: str) -> Optional[TensorInfo]:
        return self.value_info.get(name)

    def set_initializer(self, name: str, array) -> None:
        array = np.asarray(array)
        self.initializers[name] = array
        self.set_info(TensorInfo(name, dtype_from_numpy(array.dtype),
                                 tuple(int(d) for d in array.shape)))

    def is_constant(self, name: str) -> bool:
        return name in self.initializers

    @property
    def runtime_inputs(self) -> list:
        return [i for i in self.inputs if i not in self.initializers]

    def producers(self) -> dict:
        out = {}
        for node in self.nodes:
            for o in node.outputs:
                if o:
                    out[o] = node
        return out

    def consumers(self) -> dict:
        out = defaultdict(list)
        for node in self.nodes:
            for i in node.real_inputs():
                out[i].append(node)
        return out

    def use_count(self) -> dict:
        counts = defaultdict(int)
        for node in self.nodes:
            for i in node.real_inputs():
                counts[i] += 1
        for o in self.outputs:
            counts[o] += 1
        return counts

    def topo_sort(self) -> list:
        return topo_sort(self)

    def reorder_topologically(self) -> None:
        self.nodes = self.topo_sort()

    def remove_nodes(self, to_remove: Iterable[Node]) -> None:
        drop = {id(n) for n in to_remove}
        self.nodes = [n for n in self.nodes if id(n) not in drop]

    def clone(self) -> "Graph":
        g = Graph(self.name)
        g.inputs = list(self.inputs)
        g.outputs = list(self.outputs)
        g.initializers = dict(self.initializers)
        g.value_info = {k: TensorInfo(v.name, v.dtype, tuple(v.shape))
                        for k, v in self.value_info.items()}
        for n in self.nodes:
            g.nodes.append(Node(n.op_type, list(n.inputs), list(n.outputs), dict(n.attrs),
                                n.name, None if n.fused_from is None else list(n.fused_from)))
        return g

    def summary(self) -> str:
        hist = defaultdict(int)
        for n in self.nodes:
            hist[n.op_type] += 1
        ops = ", ".join(f"{k}x{v}" for k, v in sorted(hist.items()))
        return (f"Graph {self.name!r}: {len(self.nodes)} nodes\n"
                f"  inputs : {', '.join(self.runtime_inputs) or '(none)'}\n"
                f"  outputs: {', '.join(self.outputs) or '(none)'}\n"
                f"  ops    : {ops}")

    def __iter__(self):
        return iter(self.nodes)

    def __len__(self) -> int:
        return len(self.nodes)


def topo_sort(graph) -> list:
    """Kahn order of ``graph.nodes`` for any duck-typed graph.

    Ready nodes are released FIFO in node-list order, as in
    ``mdlc/ir/graph.py:99-138``; the order fixes buffer lifetimes, so keeping it
    identical lets a reference ``MemoryPlan`` be compared one-to-one.
    """
    nodes = list(graph.nodes)
    available = set(graph.inputs) | set(graph.initializers.keys())
    producer = {}
    for n in nodes:
        for o in n.outputs:
            if o:
                producer[o] = n
    idx = {id(n): k for k, n in enumerate(nodes)}
    indeg = [0] * len(nodes)
    dependents = defaultdict(list)
    for k, n in enumerate(nodes):
        need = set()
        for i in (x for x in n.inputs if x):
            if i in available:
                continue
            p = producer.get(i)
            if p is not None:
                need.add(idx[id(p)])
        indeg[k] = len(need)
        for d in need:
            dependents[d].append(k)
    ready = deque(k for k in range(len(nodes)) if indeg[k] == 0)
    order = []
    while ready:
        k = ready.popleft()
        order.append(nodes[k])
        for m in dependents[k]:
            indeg[m] -= 1
            if indeg[m] == 0:
                ready.append(m)
    if len(order) != len(nodes):
        raise ValueError("graph has a cycle or dangling dependency")
    return order
