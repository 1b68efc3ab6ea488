"""Graph builders for the five benchmark workloads, through the public
Tensor / nn API with seeded synthetic data (numpy default_rng: seed 42 for
inputs, 43+i for layer i), so that every consumer (bench, smoke, tests) sees
identical bytes.

  mlp         Linear 784->256, ReLU, Linear 256->10, softmax(-1); x U(0,1), W N(0,1/fan_in), b 0
  fused       z = sigmoid(x*y + 0.5) - relu(x) on [rows, cols]; outputs row sum, mean, max of z
              and LayerNorm([cols])(z) (gamma 1, beta 0, eps 1e-5); x, y N(0,1)
  gemm_chain  out = Linear2(GELU(Linear1(A))), A [rows,4096] N(0,1), W1 [16384,4096] N(0,1/4096),
              W2 [4096,16384] N(0,1/16384), biases U(-0.01, 0.01)
  encoder     post-LN Transformer encoder block: x [B,S,768] N(0,1), 12-head self-attention,
              FFN 768->3072->768 with GELU; Linear weights N(0,0.02), biases 0
  convstack   Conv 3->64 k7 s2 p3 + BatchNorm(eval) + ReLU + MaxPool k3 s2 + 2x(Conv 64->64 k3 p1 + ReLU)
              + AdaptiveAvgPool(1) + Linear 64->1000; x U(0,1), He-normal weights, conv biases 0
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np

from . import nn
from .tensor import Tensor, from_numpy, gelu, relu, reset_graph, sigmoid, softmax


@dataclass
class Workload:
    name: str
    outputs: List[Tensor]
    inputs: Dict[str, Tensor]      # batch inputs (bound per step in the bench)
    samples: int                   # units of the throughput metric in one graph
    flops: float = 0.0             # algorithmic FLOPs per graph
    bytes: float = 0.0             # algorithmic HBM bytes per graph
    meta: dict = field(default_factory=dict)

    def graph(self):
        return self.outputs[0].graph()

    def output_ids(self) -> List[int]:
        return [t.node().id() for t in self.outputs]

    def weights(self) -> Dict[int, np.ndarray]:
        """Constant leaves a serving host keeps on the device (weights and
        biases), by node id: every payload-carrying leaf that is not a batch
        input, except constants whose elements are all equal, which the
        executor turns into scalar-table slots and never materialises."""
        g = self.graph()
        input_ids = {t.node().id() for t in self.inputs.values()}
        out = {}
        for n in g.topological_order([t.node() for t in self.outputs]):
            if n.is_operation() or n.id() in input_ids or not n.has_constant_data() or n.numel() <= 1:
                continue
            a = n.constant_data()
            if np.all(a == a.flat[0]):
                continue
            out[n.id()] = a
        return out


def _normal(seed, shape, std):
    return (np.random.default_rng(seed).standard_normal(shape) * std).astype(np.float32)


def mlp(batch: int = 64) -> Workload:
    reset_graph()
    x = Tensor.input(np.random.default_rng(42).random((batch, 784), dtype=np.float32), copy=False)
    with nn.deferred_init():
        l1, l2 = nn.Linear(784, 256), nn.Linear(256, 10)
    l1.set_parameter("weight", _normal(43, (256, 784), np.sqrt(1 / 784)))
    l2.set_parameter("weight", _normal(44, (10, 256), np.sqrt(1 / 256)))
    y = softmax(l2(relu(l1(x))), -1)
    flops = 2.0 * batch * (784 * 256 + 256 * 10)
    return Workload("mlp", [y], {"x": x}, batch, flops, batch * (784 + 10) * 4.0,
                    {"model": "MLP 784-256-10", "global_batch": batch})


def fused(rows: int = 8192, cols: int = 4096) -> Workload:
    reset_graph()
    x = Tensor.input(np.random.default_rng(42).standard_normal((rows, cols), dtype=np.float32), copy=False)
    y = Tensor.input(np.random.default_rng(43).standard_normal((rows, cols), dtype=np.float32), copy=False)
    z = sigmoid(x * y + 0.5) - relu(x)
    ln = nn.LayerNorm(cols)
    outs = [z.sum(1), z.mean(1), z.max(1), ln(z)]
    # per row: read x and y, write LayerNorm(z) and three row statistics
    return Workload("fused", outs, {"x": x, "y": y}, rows, 0.0, rows * (3 * cols * 4 + 3 * 4.0),
                    {"model": "fused elementwise+reduction", "rows": rows, "cols": cols})


def gemm_chain(rows: int = 8192, d: int = 4096, h: int = 16384) -> Workload:
    reset_graph()
    A = Tensor.input(np.random.default_rng(42).standard_normal((rows, d), dtype=np.float32), copy=False)
    with nn.deferred_init():
        l1, l2 = nn.Linear(d, h), nn.Linear(h, d)
    l1.set_parameter("weight", _normal(43, (h, d), np.sqrt(1 / d)))
    l1.set_parameter("bias", np.random.default_rng(44).uniform(-0.01, 0.01, h).astype(np.float32))
    l2.set_parameter("weight", _normal(45, (d, h), np.sqrt(1 / h)))
    l2.set_parameter("bias", np.random.default_rng(46).uniform(-0.01, 0.01, d).astype(np.float32))
    out = l2(gelu(l1(A)))
    return Workload("gemm_chain", [out], {"A": A}, rows, 2.0 * rows * (d * h + h * d), 0.0,
                    {"model": "Linear-GELU-Linear 4096-16384-4096", "rows": rows})


def encoder(batch: int = 32, seq: int = 512, d: int = 768, heads: int = 12, ff: int = 3072) -> Workload:
    reset_graph()
    x = Tensor.input(np.random.default_rng(42).standard_normal((batch, seq, d), dtype=np.float32), copy=False)
    with nn.deferred_init():
        blk = nn.TransformerEncoderLayer(d, heads, ff, dropout=0.0, activation="gelu", batch_first=True)
    blk.eval()
    seed = 43
    for name, p in list(blk.named_parameters()):
        if name.endswith("weight") and len(p.shape) == 2:
            blk.set_parameter(name, _normal(seed, p.shape, 0.02))
            seed += 1
    out = blk(x)
    per_seq = 2.0 * seq * (4 * d * d + 2 * d * ff) + 2.0 * 2 * seq * seq * d
    return Workload("encoder", [out], {"x": x}, batch, per_seq * batch, 0.0,
                    {"model": "post-LN encoder d768 h12 ff3072", "global_batch": batch, "seq_len": seq})


def convstack(batch: int = 256, hw: int = 224) -> Workload:
    reset_graph()
    x = Tensor.input(np.random.default_rng(42).random((batch, 3, hw, hw), dtype=np.float32), copy=False)
    with nn.deferred_init():
        c1 = nn.Conv2d(3, 64, 7, 2, 3)
        c2, c3 = nn.Conv2d(64, 64, 3, 1, 1), nn.Conv2d(64, 64, 3, 1, 1)
        fc = nn.Linear(64, 1000)
    bn = nn.BatchNorm2d(64)
    bn.eval()
    pool = nn.MaxPool2d(3, 2)
    gap = nn.AdaptiveAvgPool2d(1)
    c1.set_parameter("weight", _normal(43, (64, 3, 7, 7), np.sqrt(2 / 147)))
    c2.set_parameter("weight", _normal(44, (64, 64, 3, 3), np.sqrt(2 / 576)))
    c3.set_parameter("weight", _normal(45, (64, 64, 3, 3), np.sqrt(2 / 576)))
    fc.set_parameter("weight", _normal(46, (1000, 64), np.sqrt(2 / 64)))
    h = pool(relu(bn(c1(x))))
    h = relu(c3(relu(c2(h))))
    g = gap(h)
    out = fc(g.reshape([batch, 64]))
    o1 = (hw + 6 - 7) // 2 + 1
    o2 = (o1 - 3) // 2 + 1
    flops = 2.0 * batch * (o1 * o1 * 64 * 147 + 2 * o2 * o2 * 64 * 576 + 64 * 1000)
    return Workload("convstack", [out], {"x": x}, batch, flops, 0.0,
                    {"model": "conv stack 7x7/3x3", "global_batch": batch})


BUILDERS = {"mlp": mlp, "fused": fused, "gemm_chain": gemm_chain, "encoder": encoder, "convstack": convstack}
