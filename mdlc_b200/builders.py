"""Seeded IR-native model builders for the benchmark configurations.

The reference builds its models as ONNX protobufs and imports them
(``mdlc/tools/build_models.py``, ``build_resnet18.py``,
``build_mobilenetv2.py``, ``build_repvit.py``); ``onnx`` is not a dependency
here, so these builders emit the same operator graphs (Conv without bias +
BatchNormalization + activation, Clip with constant bounds for ReLU6, the
Div/Erf/Add/Mul/Mul decomposition torch uses to export GELU at opset 17)
directly in the IR. Every node gets a unique name, because the Conv+BN fold
names its bias ``<conv name>_bias_bnfold``.

Initialisation: conv weights Kaiming-normal
``std = sqrt(2 / fan_out)`` (torchvision's ``mode="fan_out"``), depthwise
convs use the same rule with ``fan_out = 9``; the final FC is Kaiming-normal
in ``fan_in`` mode, ``std = sqrt(2 / fan_in)``; BN ``gamma ~ U(0.5, 1.5)``,
``beta ~ N(0, 0.1)``, ``running_mean ~ N(0, 0.1)``, ``running_var ~ U(0.5, 1.5)``,
``eps = 1e-5``. Inputs are ``N(0, 1)`` from :func:`make_input`.

Untrained depthwise stacks shrink activations geometrically, which makes any
parity check vacuous (``mdlc/testing/harness.py:72-80``). Instead of the
reference exporters' data-dependent LSUV rescale (``export_utils.py:16-50``),
MobileNetV2 and the RepViT-style net use ``fan_in``-mode gains chosen per layer
kind so activations stay O(1) without a forward pass.
"""

from __future__ import annotations

import numpy as np

from mdlc_b200.ir import FLOAT32, Graph, Node, TensorInfo


class _Builder:
    def __init__(self, name: str, seed: int) -> None:
        self.g = Graph(name)
        self.rng = np.random.default_rng(seed)
        self.k = 0

    def uid(self, base: str) -> str:
        self.k += 1
        return f"{base}_{self.k}"

    def input(self, name: str, shape) -> str:
        self.g.inputs.append(name)
        self.g.set_info(TensorInfo(name, FLOAT32, tuple(shape)))
        return name

    def const(self, name: str, arr) -> str:
        self.g.set_initializer(name, np.asarray(arr, dtype=np.float32))
        return name

    def node(self, op, inputs, attrs=None, name=None, n_out=1):
        name = name or self.uid(op.lower())
        outs = [f"{name}_out"] if n_out == 1 else [f"{name}_out{i}" for i in range(n_out)]
        self.g.add_node(Node(op, list(inputs), outs, dict(attrs or {}), name))
        return outs[0] if n_out == 1 else outs

    def conv(self, x, cin, cout, k, stride=1, pad=None, groups=1, bias=False, name=None,
             gain=2.0, std=None):
        name = name or self.uid("conv")
        pad = k // 2 if pad is None else pad
        fan_out = (cout // groups) * k * k
        std = np.sqrt(gain / fan_out) if std is None else std
        w = self.rng.standard_normal((cout, cin // groups, k, k)).astype(np.float32) * np.float32(std)
        ins = [x, self.const(name + ".weight", w)]
        if bias:
            ins.append(self.const(name + ".bias",
                                  self.rng.standard_normal(cout).astype(np.float32) * np.float32(0.1)))
        return self.node("Conv", ins, {"kernel_shape": [k, k], "strides": [stride, stride],
                                       "pads": [pad, pad, pad, pad], "dilations": [1, 1],
                                       "group": groups}, name)

    def bn(self, x, c, name=None):
        name = name or self.uid("bn")
        r = self.rng
        ins = [x,
               self.const(name + ".weight", r.uniform(0.5, 1.5, c).astype(np.float32)),
               self.const(name + ".bias", (r.standard_normal(c) * 0.1).astype(np.float32)),
               self.const(name + ".running_mean", (r.standard_normal(c) * 0.1).astype(np.float32)),
               self.const(name + ".running_var", r.uniform(0.5, 1.5, c).astype(np.float32))]
        return self.node("BatchNormalization", ins, {"epsilon": 1e-5}, name)

    def relu(self, x):
        return self.node("Relu", [x])

    def relu6(self, x):
        name = self.uid("clip")
        lo = self.const(name + ".min", np.float32(0.0))
        hi = self.const(name + ".max", np.float32(6.0))
        return self.node("Clip", [x, lo, hi], None, name)

    def gelu(self, x):
        """torch.onnx opset-17 GELU decomposition: x * 0.5 * (1 + erf(x / sqrt 2))."""
        name = self.uid("gelu")
        d = self.node("Div", [x, self.const(name + ".sqrt2", np.float32(np.sqrt(2.0)))], None, name + ".div")
        e = self.node("Erf", [d], None, name + ".erf")
        a = self.node("Add", [e, self.const(name + ".one", np.float32(1.0))], None, name + ".add")
        m = self.node("Mul", [x, a], None, name + ".mul")
        return self.node("Mul", [m, self.const(name + ".half", np.float32(0.5))], None, name + ".mul2")

    def fc(self, x, cin, cout, name="fc"):
        w = self.rng.standard_normal((cout, cin)).astype(np.float32) * np.float32(np.sqrt(2.0 / cin))
        b = (self.rng.standard_normal(cout) * 0.1).astype(np.float32)
        return self.node("Gemm", [x, self.const(name + ".weight", w), self.const(name + ".bias", b)],
                         {"transB": 1, "alpha": 1.0, "beta": 1.0}, name)

    def finish(self, out: str, out_name: str = "logits") -> Graph:
        # rename the final value to a stable graph output name
        for n in self.g.nodes:
            n.outputs = [out_name if o == out else o for o in n.outputs]
        self.g.outputs = [out_name]
        return self.g


# ---------------------------------------------------------------- ResNet-18

def resnet18(batch: int = 1, seed: int = 0, image: int = 224, num_classes: int = 1000,
             widths=(64, 128, 256, 512)) -> Graph:
    """torchvision ResNet-18 topology, raw (pre-pass) form."""
    b = _Builder("resnet18", seed)
    x = b.input("input", (batch, 3, image, image))
    c0 = widths[0]
    x = b.relu(b.bn(b.conv(x, 3, c0, 7, 2, 3, name="conv1"), c0, "bn1"))
    x = b.node("MaxPool", [x], {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]},
               "maxpool")
    cin = c0
    for li, cout in enumerate(widths):
        for bi in range(2):
            stride = 2 if (li > 0 and bi == 0) else 1
            p = f"layer{li + 1}.{bi}"
            y = b.relu(b.bn(b.conv(x, cin, cout, 3, stride, 1, name=p + ".conv1"), cout, p + ".bn1"))
            y = b.bn(b.conv(y, cout, cout, 3, 1, 1, name=p + ".conv2"), cout, p + ".bn2")
            if stride != 1 or cin != cout:
                sc = b.bn(b.conv(x, cin, cout, 1, stride, 0, name=p + ".downsample.0"), cout,
                          p + ".downsample.1")
            else:
                sc = x
            x = b.relu(b.node("Add", [y, sc], None, p + ".add"))
            cin = cout
    x = b.node("GlobalAveragePool", [x], None, "avgpool")
    x = b.node("Flatten", [x], {"axis": 1}, "flatten")
    return b.finish(b.fc(x, cin, num_classes, "fc"))


# ------------------------------------------------------- small test models

def conv_bn_relu(n=1, cin=3, cout=8, h=16, w=16, k=3, stride=1, seed=0, act="Relu") -> Graph:
    """Conv -> BatchNorm -> act (the canonical fusion target)."""
    b = _Builder("conv_bn_relu", seed)
    x = b.input("x", (n, cin, h, w))
    y = b.bn(b.conv(x, cin, cout, k, stride, k // 2, name="conv"), cout, "bn")
    if act == "Relu":
        y = b.relu(y)
    elif act == "Relu6":
        y = b.relu6(y)
    return b.finish(y, "y")


def residual_block(n=1, c=8, h=16, w=16, seed=1) -> Graph:
    """conv-bn-relu -> conv-bn, + skip, relu (``build_models.py:36-74``)."""
    b = _Builder("residual_block", seed)
    x = b.input("x", (n, c, h, w))
    y = b.relu(b.bn(b.conv(x, c, c, 3, name="conv_a"), c, "bn_a"))
    y = b.bn(b.conv(y, c, c, 3, name="conv_b"), c, "bn_b")
    return b.finish(b.relu(b.node("Add", [y, x], None, "add")), "y")


def mlp(n=4, din=16, dh=32, dout=8, seed=2) -> Graph:
    """Gemm -> Relu -> Gemm with transB=1 (``build_models.py:77-97``)."""
    b = _Builder("mlp", seed)
    x = b.input("x", (n, din))
    h = b.relu(b.fc(x, din, dh, "fc1"))
    return b.finish(b.fc(h, dh, dout, "fc2"), "y")


def grouped_block(n=2, c=64, h=14, w=14, groups=8, width=2, seed=3) -> Graph:
    """ResNeXt-style bottleneck with a grouped 3x3 conv (1 < groups < channels):
    1x1 conv-bn-relu (c -> width*c), 3x3 grouped conv-bn-relu, 1x1 conv-bn, + skip, relu."""
    b = _Builder("grouped_block", seed)
    x = b.input("x", (n, c, h, w))
    m = width * c
    y = b.relu(b.bn(b.conv(x, c, m, 1, name="conv_in"), m, "bn_in"))
    y = b.relu(b.bn(b.conv(y, m, m, 3, groups=groups, name="conv_g"), m, "bn_g"))
    y = b.bn(b.conv(y, m, c, 1, name="conv_out"), c, "bn_out")
    return b.finish(b.relu(b.node("Add", [y, x], None, "add")), "y")


# --------------------------------------------------------------- MobileNetV2

MBV2_SETTINGS = ((1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2),
                 (6, 96, 3, 1), (6, 160, 3, 2), (6, 320, 1, 1))


def mobilenetv2(batch: int = 1, seed: int = 0, image: int = 224, num_classes: int = 1000) -> Graph:
    """MobileNetV2 width 1.0: stem 3x3/2 conv 32, 17 inverted
    residual blocks (1x1 expand t=6, 3x3 depthwise, ReLU6, 1x1 linear project),
    head 1x1 conv 1280, global pool, FC.

    Convs use Kaiming-normal in ``fan_in`` mode with gain 2 (1 for the linear
    projections) so activations stay O(1) through the untrained depthwise stack.
    """
    b = _Builder("mobilenetv2", seed)
    x = b.input("input", (batch, 3, image, image))

    def cbr(x, cin, cout, k, s, groups=1, act=True, name=None):
        fan_in = (cin // groups) * k * k
        y = b.bn(b.conv(x, cin, cout, k, s, k // 2, groups, name=name,
                        std=np.sqrt((2.0 if act else 1.0) / fan_in)), cout)
        return b.relu6(y) if act else y

    x = cbr(x, 3, 32, 3, 2, name="features.0")
    cin = 32
    blk = 1
    for t, c, n, s in MBV2_SETTINGS:
        for i in range(n):
            stride = s if i == 0 else 1
            hid = cin * t
            y = x
            p = f"features.{blk}"
            if t != 1:
                y = cbr(y, cin, hid, 1, 1, name=p + ".expand")
            y = cbr(y, hid, hid, 3, stride, groups=hid, name=p + ".dw")
            y = cbr(y, hid, c, 1, 1, act=False, name=p + ".project")
            if stride == 1 and cin == c:
                y = b.node("Add", [x, y], None, p + ".add")
            x, cin = y, c
            blk += 1
    x = cbr(x, cin, 1280, 1, 1, name=f"features.{blk}")
    x = b.node("GlobalAveragePool", [x], None, "avgpool")
    x = b.node("Flatten", [x], {"axis": 1}, "flatten")
    return b.finish(b.fc(x, 1280, num_classes, "classifier"))


# ---------------------------------------------------------- RepViT-style net

def _make_divisible(v, divisor=8):
    new_v = max(divisor, int(v + divisor / 2) // divisor * divisor)
    return new_v + divisor if new_v < 0.9 * v else new_v


def repvit(batch: int = 1, seed: int = 0, image: int = 224, num_classes: int = 1000,
           widths=(56, 112, 224, 448), depths=(2, 2, 14, 2)) -> Graph:
    """RepViT-M1.0-style reparameterised CNN.

    Stem: 3x3/2 conv (c/2) + GELU, 3x3/2 conv (c). Each block: a folded 3x3
    depthwise token mixer (one conv with bias), squeeze-excite (reduction 4,
    ``make_divisible(c/4, 8)``) on every other block, then
    ``x + conv1x1(GELU(conv1x1_expand2x(x)))``. Stage transitions: a stride-2
    depthwise conv then a 1x1 channel projection. Head: ReduceMean over H,W,
    Flatten, FC.
    """
    b = _Builder("repvit", seed)
    x = b.input("input", (batch, 3, image, image))

    def conv_bn(x, cin, cout, k, s=1, groups=1, gain=2.0, name=None):
        fan_in = (cin // groups) * k * k
        return b.bn(b.conv(x, cin, cout, k, s, k // 2, groups, name=name,
                           std=np.sqrt(gain / fan_in)), cout)

    c0 = widths[0]
    x = b.gelu(conv_bn(x, 3, c0 // 2, 3, 2, name="stem.0"))
    x = conv_bn(x, c0 // 2, c0, 3, 2, gain=1.0, name="stem.1")
    cin = c0
    blk = 0
    for si, (c, d) in enumerate(zip(widths, depths)):
        if si > 0:
            x = conv_bn(x, cin, cin, 3, 2, groups=cin, gain=1.0, name=f"stages.{si}.down.dw")
            x = conv_bn(x, cin, c, 1, 1, gain=1.0, name=f"stages.{si}.down.pw")
            cin = c
        for i in range(d):
            p = f"stages.{si}.blocks.{i}"
            # token mixer: reparameterised depthwise 3x3 (identity folded into the centre tap)
            x = b.conv(x, c, c, 3, 1, 1, groups=c, bias=True, name=p + ".mixer",
                       std=np.sqrt(1.0 / 9.0))
            if blk % 2 == 0:
                rd = _make_divisible(c * 0.25, 8)
                s = b.node("ReduceMean", [x], {"axes": [2, 3], "keepdims": 1}, p + ".se.pool")
                s = b.relu(b.conv(s, c, rd, 1, 1, 0, bias=True, name=p + ".se.fc1",
                                  std=np.sqrt(2.0 / c)))
                s = b.conv(s, rd, c, 1, 1, 0, bias=True, name=p + ".se.fc2", std=np.sqrt(1.0 / rd))
                s = b.node("Sigmoid", [s], None, p + ".se.gate")
                x = b.node("Mul", [x, s], None, p + ".se.mul")
            h = b.gelu(conv_bn(x, c, 2 * c, 1, name=p + ".mlp.fc1"))
            h = conv_bn(h, 2 * c, c, 1, gain=0.5, name=p + ".mlp.fc2")
            x = b.node("Add", [x, h], None, p + ".add")
            blk += 1
    x = b.node("ReduceMean", [x], {"axes": [2, 3], "keepdims": 1}, "head.pool")
    x = b.node("Flatten", [x], {"axis": 1}, "head.flatten")
    return b.finish(b.fc(x, cin, num_classes, "head.fc"))


BUILDERS = {"resnet18": resnet18, "mobilenetv2": mobilenetv2, "repvit": repvit,
            "conv_bn_relu": conv_bn_relu, "residual_block": residual_block, "mlp": mlp,
            "grouped_block": grouped_block}


def make_input(graph: Graph, seed: int = 0) -> dict:
    """Seeded N(0,1) feeds for every runtime input of ``graph``."""
    rng = np.random.default_rng(seed)
    return {name: rng.standard_normal(graph.info(name).shape).astype(np.float32)
            for name in graph.runtime_inputs}
