"""Node lists and seeded synthetic tensors of the path's workloads.

1. stem Conv+Relu:  X [1,3,224,224] U(-1,1); W [64,3,7,7] N(0, sqrt(2/147));
   bias [64] U(-0.1,0.1); stride 2, pad 3 (seed 0)
2. broadcast MatMul+Add+Relu: A [8,1,512,768] N(0,1); B [12,768,3072] N(0,1/sqrt(768));
   bias [3072] U(-0.1,0.1) (seed 1)
3. ResNet-18 v1, batch 32 (seed 2)
4. conv shape sweep, batch 128 (seed 3)
5. ResNet-50 v1.5, batch 256 (seed 4)

ResNet initialisation: conv weights Kaiming normal std = sqrt(2 / fan_in),
fan_in = C_in/group * kh * kw; BatchNormalization gamma = 1, beta = 0,
mean ~ N(0, 0.1), var ~ U(0.5, 1.5), eps = 1e-5; the final Gemm weight and bias
~ U(-1/sqrt(fan_in), 1/sqrt(fan_in)); input ~ N(0, 1).  All tensors come from
``synth`` keyed by (seed, tensor name).
"""
from __future__ import annotations

import math
from typing import Dict, List, Tuple

import numpy as np

from . import synth

Graph = Tuple[List[dict], Dict[str, np.ndarray], List[Tuple[str, List[int]]], List[str]]


def stem_conv(seed: int = 0, batch: int = 1) -> Graph:
    inits = {
        "W": synth.normal(seed, "W", (64, 3, 7, 7), 0.0, math.sqrt(2.0 / 147)),
        "B": synth.uniform(seed, "B", (64,), -0.1, 0.1),
    }
    nodes = [
        {"op": "Conv", "inputs": ["X", "W", "B"], "outputs": ["conv"],
         "attrs": {"kernel_shape": [7, 7], "strides": [2, 2], "pads": [3, 3, 3, 3]}},
        {"op": "Relu", "inputs": ["conv"], "outputs": ["Y"]},
    ]
    return nodes, inits, [("X", [batch, 3, 224, 224])], ["Y"]


def stem_input(seed: int = 0, batch: int = 1) -> np.ndarray:
    return synth.uniform(seed, "X", (batch, 3, 224, 224), -1.0, 1.0)


def broadcast_matmul(seed: int = 1):
    """Returns (A, B, bias) of the broadcast MatMul+Add+Relu workload."""
    a = synth.normal(seed, "A", (8, 1, 512, 768))
    b = synth.normal(seed, "B", (12, 768, 3072), 0.0, 1.0 / math.sqrt(768))
    bias = synth.uniform(seed, "bias", (3072,), -0.1, 0.1)
    return a, b, bias


def broadcast_matmul_graph(seed: int = 1) -> Graph:
    _, b, bias = broadcast_matmul(seed)
    nodes = [
        {"op": "MatMul", "inputs": ["A", "B"], "outputs": ["mm"]},
        {"op": "Add", "inputs": ["mm", "bias"], "outputs": ["sum"]},
        {"op": "Relu", "inputs": ["sum"], "outputs": ["Y"]},
    ]
    return nodes, {"B": b, "bias": bias}, [("A", [8, 1, 512, 768])], ["Y"]


# conv sweep: (name, C_in, C_out, H, kernel, pad, dilation, group)
SWEEP = [
    ("1x1_64_56", 64, 64, 56, 1, 0, 1, 1), ("3x3_64_56", 64, 64, 56, 3, 1, 1, 1),
    ("1x1_128_28", 128, 128, 28, 1, 0, 1, 1), ("3x3_128_28", 128, 128, 28, 3, 1, 1, 1),
    ("1x1_256_14", 256, 256, 14, 1, 0, 1, 1), ("3x3_256_14", 256, 256, 14, 3, 1, 1, 1),
    ("1x1_512_7", 512, 512, 7, 1, 0, 1, 1), ("3x3_512_7", 512, 512, 7, 3, 1, 1, 1),
    ("1x1_256to1024_14", 256, 1024, 14, 1, 0, 1, 1),
    ("3x3_g32_128_28", 128, 128, 28, 3, 1, 1, 32), ("3x3_g32_256_14", 256, 256, 14, 3, 1, 1, 32),
    ("3x3_g32_1024_7", 1024, 1024, 7, 3, 1, 1, 32),
    ("3x3_d2_256_28", 256, 256, 28, 3, 2, 2, 1),
]


def sweep_case(name: str, seed: int = 3, batch: int = 128):
    """(x, w, b, attrs) of one conv-sweep shape, bias+Relu epilogue."""
    _, ci, co, hw, k, p, d, g = next(s for s in SWEEP if s[0] == name)
    x = synth.normal(seed, name + "/X", (batch, ci, hw, hw))
    fan_in = ci // g * k * k
    w = synth.normal(seed, name + "/W", (co, ci // g, k, k), 0.0, math.sqrt(2.0 / fan_in))
    b = synth.uniform(seed, name + "/B", (co,), -0.1, 0.1)
    attrs = {"strides": [1, 1], "pads": [p, p, p, p], "dilations": [d, d], "group": g}
    return x, w, b, attrs


def sweep_flops(name: str, batch: int = 128) -> float:
    _, ci, co, hw, k, p, d, g = next(s for s in SWEEP if s[0] == name)
    return 2.0 * batch * co * hw * hw * (ci // g) * k * k


class _Builder:
    def __init__(self, seed: int):
        self.seed = seed
        self.nodes: List[dict] = []
        self.inits: Dict[str, np.ndarray] = {}
        self.n = 0
        self.conv_flops_per_image = 0.0

    def name(self, base: str) -> str:
        self.n += 1
        return f"{base}_{self.n}"

    def conv_bn(self, x: str, cin: int, cout: int, k: int, stride: int, pad: int, hw: int, relu: bool) -> Tuple[str, int]:
        w = self.name("W")
        fan_in = cin * k * k
        self.inits[w] = synth.normal(self.seed, w, (cout, cin, k, k), 0.0, math.sqrt(2.0 / fan_in))
        c = self.name("conv")
        self.nodes.append({"op": "Conv", "inputs": [x, w], "outputs": [c],
                           "attrs": {"kernel_shape": [k, k], "strides": [stride, stride], "pads": [pad] * 4}})
        ohw = (hw + 2 * pad - k) // stride + 1
        self.conv_flops_per_image += 2.0 * cout * ohw * ohw * cin * k * k
        g, b, m, v = (self.name(s) for s in ("gamma", "beta", "mean", "var"))
        self.inits[g] = np.ones(cout, np.float32)
        self.inits[b] = np.zeros(cout, np.float32)
        self.inits[m] = synth.normal(self.seed, m, (cout,), 0.0, 0.1)
        self.inits[v] = synth.uniform(self.seed, v, (cout,), 0.5, 1.5)
        y = self.name("bn")
        self.nodes.append({"op": "BatchNormalization", "inputs": [c, g, b, m, v], "outputs": [y],
                           "attrs": {"epsilon": 1e-5}})
        if relu:
            r = self.name("relu")
            self.nodes.append({"op": "Relu", "inputs": [y], "outputs": [r]})
            y = r
        return y, ohw

    def add_relu(self, a: str, b: str) -> str:
        s = self.name("add")
        self.nodes.append({"op": "Add", "inputs": [a, b], "outputs": [s]})
        r = self.name("relu")
        self.nodes.append({"op": "Relu", "inputs": [s], "outputs": [r]})
        return r

    def head(self, x: str, cin: int, classes: int = 1000) -> str:
        gap = self.name("gap")
        self.nodes.append({"op": "GlobalAveragePool", "inputs": [x], "outputs": [gap]})
        fl = self.name("flatten")
        self.nodes.append({"op": "Flatten", "inputs": [gap], "outputs": [fl], "attrs": {"axis": 1}})
        bound = 1.0 / math.sqrt(cin)
        self.inits["fc_W"] = synth.uniform(self.seed, "fc_W", (classes, cin), -bound, bound)
        self.inits["fc_B"] = synth.uniform(self.seed, "fc_B", (classes,), -bound, bound)
        self.nodes.append({"op": "Gemm", "inputs": [fl, "fc_W", "fc_B"], "outputs": ["logits"],
                           "attrs": {"alpha": 1.0, "beta": 1.0, "transB": 1}})
        return "logits"

    def stem(self, x: str) -> Tuple[str, int]:
        y, hw = self.conv_bn(x, 3, 64, 7, 2, 3, 224, relu=True)
        p = self.name("pool")
        self.nodes.append({"op": "MaxPool", "inputs": [y], "outputs": [p],
                           "attrs": {"kernel_shape": [3, 3], "strides": [2, 2], "pads": [1, 1, 1, 1]}})
        return p, (hw + 2 - 3) // 2 + 1


def resnet18(batch: int = 32, seed: int = 2) -> Graph:
    """ResNet-18 v1: BasicBlocks [2,2,2,2], widths 64..512, 1x1/2 conv+BN projection."""
    b = _Builder(seed)
    x, hw = b.stem("X")
    cin = 64
    for stage, width in enumerate((64, 128, 256, 512)):
        for blk in range(2):
            stride = 2 if (stage > 0 and blk == 0) else 1
            y, ohw = b.conv_bn(x, cin, width, 3, stride, 1, hw, relu=True)
            y, _ = b.conv_bn(y, width, width, 3, 1, 1, ohw, relu=False)
            sc = x
            if stride != 1 or cin != width:
                sc, _ = b.conv_bn(x, cin, width, 1, stride, 0, hw, relu=False)
            x = b.add_relu(y, sc)
            cin, hw = width, ohw
    out = b.head(x, 512)
    g = (b.nodes, b.inits, [("X", [batch, 3, 224, 224])], [out])
    resnet18.conv_flops_per_image = b.conv_flops_per_image
    return g


def resnet50(batch: int = 256, seed: int = 4) -> Graph:
    """ResNet-50 v1.5: Bottlenecks [3,4,6,3], widths 64..512, expansion 4, stride on the 3x3."""
    b = _Builder(seed)
    x, hw = b.stem("X")
    cin = 64
    for stage, (width, blocks) in enumerate(zip((64, 128, 256, 512), (3, 4, 6, 3))):
        for blk in range(blocks):
            stride = 2 if (stage > 0 and blk == 0) else 1
            y, _ = b.conv_bn(x, cin, width, 1, 1, 0, hw, relu=True)
            y, ohw = b.conv_bn(y, width, width, 3, stride, 1, hw, relu=True)
            y, _ = b.conv_bn(y, width, width * 4, 1, 1, 0, ohw, relu=False)
            sc = x
            if stride != 1 or cin != width * 4:
                sc, _ = b.conv_bn(x, cin, width * 4, 1, stride, 0, hw, relu=False)
            x = b.add_relu(y, sc)
            cin, hw = width * 4, ohw
    out = b.head(x, 2048)
    g = (b.nodes, b.inits, [("X", [batch, 3, 224, 224])], [out])
    resnet50.conv_flops_per_image = b.conv_flops_per_image
    return g


def resnet_input(seed: int, batch: int) -> np.ndarray:
    return synth.normal(seed, "X", (batch, 3, 224, 224))
