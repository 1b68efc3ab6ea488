"""The Python front end emits the same IR as PyFlame's C++ producers.

oracle/_ref/ref_dump builds graphs with PyFlame's own Tensor API and nn
modules (linear.cpp, conv.cpp, normalization.cpp, pooling.cpp, attention.cpp)
and prints every node: type, op, shape, inputs and each attribute with its C++
type.  The same graphs are built here through pyflame_b200 and compared node
by node after relabelling both by a depth-first walk from the sinks (C++ may
evaluate operator arguments right to left, which numbers nodes differently).
"""
import subprocess

import numpy as np
import pytest

import pyflame_b200 as pf
from pyflame_b200 import autograd, ir, nn
from oracle import oracle as O

DUMP = O.HERE / "_ref" / "ref_dump"
pytestmark = pytest.mark.skipif(not DUMP.exists(), reason="PyFlame reference front end not built (oracle/_ref)")

ATTR_ORDER = ["dim", "keepdim", "new_shape", "dim0", "dim1", "start", "end", "stride", "padding", "dilation", "groups",
              "eps", "momentum", "training", "affine", "track_running_stats", "normalized_shape",
              "elementwise_affine", "kernel_size", "output_size", "target_shape"]
CT = {ir.A_INT: "int", ir.A_INT64: "int64", ir.A_FLOAT: "float", ir.A_DOUBLE: "double", ir.A_BOOL: "bool",
      ir.A_INT64_VEC: "vec64", ir.A_INT_VEC: "vec32"}


def fmt_attr(v, ct):
    t = CT[ct]
    if t in ("vec64", "vec32"):
        return f"{t}:" + "".join(f"{int(x)}," for x in v)
    if t == "bool":
        return f"bool:{1 if v else 0}"
    if t in ("float", "double"):
        return f"{t}:{v:g}"
    return f"{t}:{int(v)}"


def parse(text):
    nodes = {}
    for line in text.strip().splitlines():
        nid, typ, op, shape, ins, attrs = line.split("|")
        nodes[int(nid)] = dict(type=int(typ), op=int(op), shape=[int(s) for s in shape.split(",") if s],
                               inputs=[int(s) for s in ins.split(",") if s],
                               attrs=sorted(a for a in attrs.split(";") if a))
    return nodes


def python_nodes(g: ir.Graph):
    out = {}
    for n in g.all_nodes():
        attrs = sorted(f"{k}={fmt_attr(*n.attrs()[k])}" for k in ATTR_ORDER if n.has_attr(k))
        out[n.id()] = dict(type=int(n.type()), op=int(n.op_type()), shape=n.shape(),
                           inputs=[i.id() for i in n.inputs()], attrs=attrs)
    return out


def canonical(nodes):
    users = {k: 0 for k in nodes}
    for n in nodes.values():
        for i in n["inputs"]:
            users[i] += 1
    label, order = {}, []

    def visit(k):
        if k in label:
            return
        for i in nodes[k]["inputs"]:
            visit(i)
        label[k] = len(order)
        order.append(k)

    for k in sorted(nodes):
        if users[k] == 0:
            visit(k)
    return [(nodes[k]["type"], nodes[k]["op"], nodes[k]["shape"], [label[i] for i in nodes[k]["inputs"]],
             nodes[k]["attrs"]) for k in order]


def reference(kind):
    out = subprocess.run([str(DUMP), str(kind)], capture_output=True, text=True, check=True).stdout
    return parse(out.split("----")[0])


D = np.full(2 * 5 * 8 * 9 * 9, 0.25, np.float32)


def build(kind):
    pf.reset_graph()
    if kind == 0:
        x = pf.Tensor.from_data(D[:16], [2, 8])
        nn.Linear(8, 4)(x)
    elif kind == 1:
        x = pf.Tensor.from_data(D[:2 * 3 * 81], [2, 3, 9, 9])
        conv, bn, pool = nn.Conv2d(3, 4, 3, 2, 1), nn.BatchNorm2d(4), nn.MaxPool2d(3, 2)
        bn.eval()
        pool(pf.relu(bn(conv(x))))
    elif kind == 2:
        x = pf.Tensor.from_data(D[:16], [2, 8])
        pf.softmax(nn.LayerNorm(8)(x), -1)
    elif kind == 3:
        x = pf.Tensor.from_data(D[:80], [2, 5, 8])
        nn.MultiheadAttention(8, 2, 0.0, True, False, False, 0, 0, True)(x)
    elif kind == 4:
        x = pf.Tensor.from_data(D[:32], [4, 8])
        y = pf.Tensor.from_data(D[:32], [4, 8])
        z = pf.sigmoid(x * y + 0.5) - pf.relu(x)
        z.sum(1), z.mean(1), z.max(1)
    elif kind == 5:
        x = pf.Tensor.from_data(D[:2 * 3 * 64], [2, 3, 8, 8])
        nn.AdaptiveAvgPool2d(1)(nn.AvgPool2d(2)(x))
    elif kind == 6:
        x = pf.Tensor.from_data(D[:32], [4, 8])
        l1, l2 = nn.Linear(8, 6), nn.Linear(6, 3)
        autograd.backward(pf.softmax(l2(pf.relu(l1(x))), -1).sum())
    elif kind == 7:
        x = pf.Tensor.from_data(D[:32], [4, 8])
        y = pf.Tensor.from_data(D[:32], [4, 8])
        b = pf.Tensor.from_data(D[:8], [8])
        a = x * y + b
        h = pf.tanh(a) * pf.sigmoid(x) - pf.exp(y) / (pf.abs(x) + 1.0)
        z = pf.sqrt(h * h + 1.0).sum(1, True)
        autograd.backward((pf.log(z) + pf.sin(x).sum(1, True) * pf.cos(y).mean(1, True)).sum())
    return pf.get_current_graph()


@pytest.mark.parametrize("kind,what", [(0, "Linear"), (1, "Conv2d+BatchNorm2d+ReLU+MaxPool2d"),
                                       (2, "LayerNorm+softmax"), (3, "MultiheadAttention"),
                                       (4, "fused elementwise + row reductions"), (5, "AvgPool2d+AdaptiveAvgPool2d"),
                                       (6, "MLP loss + AutogradEngine::backward"),
                                       (7, "elementwise chain + AutogradEngine::backward")])
def test_same_ir_as_pyflame(kind, what):
    ref = canonical(reference(kind))
    ours = canonical(python_nodes(build(kind)))
    assert len(ref) == len(ours), f"{what}: {len(ref)} nodes in PyFlame's graph, {len(ours)} here"
    for i, (a, b) in enumerate(zip(ref, ours)):
        assert a == b, f"{what}: node {i} differs\n  PyFlame: {a}\n  here:    {b}"
