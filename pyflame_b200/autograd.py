"""Backward graphs for PyFlame's IR, evaluated by the CUDA executor.

PyFlame differentiates by graph construction: AutogradEngine::backward
(src/autograd/autograd.cpp:421-480) walks the forward graph in reverse
topological order from the output, asks the gradient registry
(autograd.cpp:41-397) for each operation's input gradients as NEW IR nodes in
the same graph, sums gradients that meet at one node with ADD, and attaches
the result to every PARAMETER and INPUT node as its "grad" attribute.
AutogradEngine::grad (autograd.cpp:482-548) returns the gradients of chosen
nodes instead.  Nothing is evaluated there: the backward graph is an
ordinary graph, so the executor evaluates it like any forward graph (the
GEMMs of MATMUL's gradient on the tensor cores, the rest as fused kernels).

This module builds node for node the graph PyFlame's engine builds (the
front-end IR test compares the two), including its conventions:
  - ones_like / zeros_like are full-size constants (grad_ops, :616-652);
  - broadcasting gradients are undone by sum_grad_for_broadcast (:567-614):
    a SUM over each added leading dim, then a keepdim SUM over each dim that
    was 1 in the input;
  - reduction gradients are BROADCAST nodes with a `target_shape` attribute
    (broadcast_grad_to_shape, :550-565), aligned by trailing dims as every
    broadcast here is, so they are exact for full reductions and keepdim
    reductions (the cases PyFlame's own shape rules make well-defined).
"""
from __future__ import annotations

import struct
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np

from . import ir
from .ir import DType, Graph, Node, OpType, TensorSpec
from .tensor import Tensor


def _spec(shape, like: Node) -> TensorSpec:
    return TensorSpec(list(shape), like.dtype())


def _op(g: Graph, op: OpType, ins: Sequence[Node], shape) -> Node:
    return g.create_op(op, list(ins), _spec(shape, ins[0]))


def reduction_shape(shape: Sequence[int], dim: Optional[int], keepdim: bool) -> List[int]:
    """infer_reduction_shape (shape_inference.hpp:72-107)."""
    if dim is None:
        return [1] * len(shape) if keepdim else []
    d = dim + len(shape) if dim < 0 else dim
    if not 0 <= d < len(shape):
        raise ValueError("Reduction dimension out of range")
    out = []
    for i, s in enumerate(shape):
        if i != d:
            out.append(int(s))
        elif keepdim:
            out.append(1)
    return out


# ---- grad_ops (autograd.cpp:546-652) ---------------------------------------------

def ones_like(n: Node, g: Graph) -> Node:
    return g.create_constant(_spec(n.shape(), n), np.ones(n.shape(), np.float32))


def zeros_like(n: Node, g: Graph) -> Node:
    return g.create_constant(_spec(n.shape(), n), np.zeros(n.shape(), np.float32))


def broadcast_grad_to_shape(grad: Node, target: Sequence[int], g: Graph) -> Node:
    if grad.shape() == list(target):
        return grad
    r = g.create_op(OpType.BROADCAST, [grad], _spec(target, grad))
    r.set_attr("target_shape", [int(s) for s in target], ir.A_INT64_VEC)
    return r


def sum_grad_for_broadcast(grad: Node, in_shape: Sequence[int], out_shape: Sequence[int], g: Graph) -> Node:
    in_shape, out_shape = list(in_shape), list(out_shape)
    if in_shape == out_shape:
        return grad
    if not in_shape or in_shape == [1]:
        return g.create_op(OpType.SUM, [grad], _spec(in_shape, grad))
    r = grad
    for _ in range(len(out_shape) - len(in_shape)):
        r2 = g.create_op(OpType.SUM, [r], _spec(reduction_shape(r.shape(), 0, False), r))
        r2.set_attr("dim", 0, ir.A_INT)
        r2.set_attr("keepdim", False, ir.A_BOOL)
        r = r2
    rs = r.shape()
    for i in range(len(in_shape) - 1, -1, -1):
        if in_shape[i] == 1 and rs[i] != 1:
            r2 = g.create_op(OpType.SUM, [r], _spec(reduction_shape(r.shape(), i, True), r))
            r2.set_attr("dim", i, ir.A_INT)
            r2.set_attr("keepdim", True, ir.A_BOOL)
            r = r2
    return r


# ---- the gradient registry (autograd.cpp:41-397) ------------------------------------
# fn(grad_out, inputs, node, graph) -> list of input gradients (None: no gradient)

GradFn = Callable[[Node, List[Node], Node, Graph], List[Optional[Node]]]
REGISTRY: Dict[OpType, GradFn] = {}


def _register(op: OpType):
    def deco(fn: GradFn) -> GradFn:
        REGISTRY[op] = fn
        return fn
    return deco


@_register(OpType.ADD)
def _add(go, ins, n, g):
    return [sum_grad_for_broadcast(go, ins[0].shape(), go.shape(), g),
            sum_grad_for_broadcast(go, ins[1].shape(), go.shape(), g)]


@_register(OpType.SUB)
def _sub(go, ins, n, g):
    ga = sum_grad_for_broadcast(go, ins[0].shape(), go.shape(), g)
    neg = _op(g, OpType.NEG, [go], go.shape())
    return [ga, sum_grad_for_broadcast(neg, ins[1].shape(), go.shape(), g)]


@_register(OpType.MUL)
def _mul(go, ins, n, g):
    ma = _op(g, OpType.MUL, [go, ins[1]], go.shape())
    ga = sum_grad_for_broadcast(ma, ins[0].shape(), go.shape(), g)
    mb = _op(g, OpType.MUL, [go, ins[0]], go.shape())
    return [ga, sum_grad_for_broadcast(mb, ins[1].shape(), go.shape(), g)]


@_register(OpType.DIV)
def _div(go, ins, n, g):
    a, b = ins
    d = _op(g, OpType.DIV, [go, b], go.shape())
    ga = sum_grad_for_broadcast(d, a.shape(), go.shape(), g)
    neg = _op(g, OpType.NEG, [go], go.shape())
    ma = _op(g, OpType.MUL, [neg, a], go.shape())
    bsq = g.create_op(OpType.MUL, [b, b], _spec(b.shape(), b))
    db = _op(g, OpType.DIV, [ma, bsq], go.shape())
    return [ga, sum_grad_for_broadcast(db, b.shape(), go.shape(), g)]


@_register(OpType.NEG)
def _neg(go, ins, n, g):
    return [_op(g, OpType.NEG, [go], go.shape())]


@_register(OpType.ABS)
def _abs(go, ins, n, g):
    x = ins[0]
    zero = zeros_like(x, g)
    gt = g.create_op(OpType.GT, [x, zero], _spec(x.shape(), x))
    lt = g.create_op(OpType.LT, [x, zero], _spec(x.shape(), x))
    sign = g.create_op(OpType.SUB, [gt, lt], _spec(x.shape(), x))
    return [_op(g, OpType.MUL, [go, sign], go.shape())]


@_register(OpType.SQRT)
def _sqrt(go, ins, n, g):
    # grad / (2 * sqrt(x)) with a scalar 2 (autograd.cpp:137-158); PyFlame
    # also builds a data-less scalar and an output*output product that
    # nothing reads, kept here so the graphs stay node for node the same
    g.create_constant(TensorSpec([], go.dtype()))
    g.create_op(OpType.MUL, [n, n], _spec(n.shape(), n))
    two = g.create_constant(TensorSpec([], go.dtype()), np.array(2.0, np.float32))
    tt = g.create_op(OpType.MUL, [two, n], _spec(n.shape(), n))
    return [_op(g, OpType.DIV, [go, tt], go.shape())]


@_register(OpType.EXP)
def _exp(go, ins, n, g):
    return [_op(g, OpType.MUL, [go, n], go.shape())]


@_register(OpType.LOG)
def _log(go, ins, n, g):
    return [_op(g, OpType.DIV, [go, ins[0]], go.shape())]


@_register(OpType.SIN)
def _sin(go, ins, n, g):
    c = g.create_op(OpType.COS, [ins[0]], _spec(ins[0].shape(), ins[0]))
    return [_op(g, OpType.MUL, [go, c], go.shape())]


@_register(OpType.COS)
def _cos(go, ins, n, g):
    s = g.create_op(OpType.SIN, [ins[0]], _spec(ins[0].shape(), ins[0]))
    ns = g.create_op(OpType.NEG, [s], _spec(ins[0].shape(), ins[0]))
    return [_op(g, OpType.MUL, [go, ns], go.shape())]


@_register(OpType.TANH)
def _tanh(go, ins, n, g):
    one = ones_like(n, g)
    sq = g.create_op(OpType.MUL, [n, n], _spec(n.shape(), n))
    om = g.create_op(OpType.SUB, [one, sq], _spec(n.shape(), n))
    return [_op(g, OpType.MUL, [go, om], go.shape())]


@_register(OpType.RELU)
def _relu(go, ins, n, g):
    x = ins[0]
    zero = zeros_like(x, g)
    mask = g.create_op(OpType.GT, [x, zero], _spec(x.shape(), x))
    return [_op(g, OpType.MUL, [go, mask], go.shape())]


@_register(OpType.SIGMOID)
def _sigmoid(go, ins, n, g):
    one = ones_like(n, g)
    om = g.create_op(OpType.SUB, [one, n], _spec(n.shape(), n))
    yom = g.create_op(OpType.MUL, [n, om], _spec(n.shape(), n))
    return [_op(g, OpType.MUL, [go, yom], go.shape())]


@_register(OpType.SOFTMAX)
def _softmax(go, ins, n, g):
    dim = int(n.get_attr("dim", -1))
    nd = len(go.shape())
    if dim < 0:
        dim += nd
    gy = _op(g, OpType.MUL, [go, n], go.shape())
    s = g.create_op(OpType.SUM, [gy], _spec(reduction_shape(gy.shape(), dim, True), gy))
    s.set_attr("dim", dim, ir.A_INT)
    s.set_attr("keepdim", True, ir.A_BOOL)
    gm = _op(g, OpType.SUB, [go, s], go.shape())
    return [_op(g, OpType.MUL, [n, gm], go.shape())]


@_register(OpType.SUM)
def _sum(go, ins, n, g):
    return [broadcast_grad_to_shape(go, ins[0].shape(), g)]


@_register(OpType.MEAN)
def _mean(go, ins, n, g):
    # As autograd.cpp:163-207: the `dim` attribute defaults to -1 and is
    # normalised before the full-reduction test, so a full MEAN over a tensor
    # of rank >= 1 is scaled by 1/(last dim), not 1/numel (PyFlame's result,
    # kept).
    shape = ins[0].shape()
    dim = int(n.get_attr("dim", -1))
    nd = len(shape)
    if dim < 0:
        dim += nd
    cnt = ins[0].numel() if (dim < 0 or dim >= nd) else shape[dim]
    if cnt == 0:
        return [g.create_constant(_spec(shape, go))]
    inv = g.create_constant(TensorSpec([], go.dtype()),
                            np.frombuffer(struct.pack("<f", np.float32(1.0) / np.float32(cnt)), np.float32).reshape(()))
    scaled = _op(g, OpType.MUL, [go, inv], go.shape())
    return [broadcast_grad_to_shape(scaled, shape, g)]


@_register(OpType.MATMUL)
def _matmul(go, ins, n, g):
    a, b = ins
    bt = g.create_op(OpType.TRANSPOSE, [b], _spec([b.shape()[1], b.shape()[0]], b))
    bt.set_attr("dim0", 0, ir.A_INT)
    bt.set_attr("dim1", 1, ir.A_INT)
    at = g.create_op(OpType.TRANSPOSE, [a], _spec([a.shape()[1], a.shape()[0]], a))
    at.set_attr("dim0", 0, ir.A_INT)
    at.set_attr("dim1", 1, ir.A_INT)
    ga = g.create_op(OpType.MATMUL, [go, bt], _spec(a.shape(), a))
    gb = g.create_op(OpType.MATMUL, [at, go], _spec(b.shape(), b))
    return [ga, gb]


@_register(OpType.TRANSPOSE)
def _transpose(go, ins, n, g):
    r = g.create_op(OpType.TRANSPOSE, [go], _spec(ins[0].shape(), go))
    r.set_attr("dim0", int(n.get_attr("dim0")), ir.A_INT)
    r.set_attr("dim1", int(n.get_attr("dim1")), ir.A_INT)
    return [r]


@_register(OpType.RESHAPE)
def _reshape(go, ins, n, g):
    r = g.create_op(OpType.RESHAPE, [go], _spec(ins[0].shape(), go))
    r.set_attr("new_shape", list(ins[0].shape()), ir.A_INT64_VEC)
    return [r]


@_register(OpType.VIEW)
def _view(go, ins, n, g):
    return [g.create_op(OpType.VIEW, [go], _spec(ins[0].shape(), go))]


# ---- AutogradEngine (autograd.cpp:398-548) --------------------------------------------

def reverse_topological_sort(outputs: Sequence[Node]) -> List[Node]:
    """Post-order depth-first walk over inputs from the outputs, reversed."""
    result, seen = [], set()
    for out in outputs:
        stack = [(out, 0)]
        while stack:
            node, i = stack.pop()
            if i == 0:
                if node.id() in seen:
                    continue
                seen.add(node.id())
            if i < len(node.inputs()):
                stack.append((node, i + 1))
                stack.append((node.inputs()[i], 0))
            else:
                result.append(node)
    result.reverse()
    return result


def _propagate(grad_map: Dict[int, Node], outputs: Sequence[Node], g: Graph) -> None:
    for node in reverse_topological_sort(outputs):
        if not node.is_operation():
            continue
        go = grad_map.get(node.id())
        if go is None:
            continue
        fn = REGISTRY.get(node.op_type())
        if fn is None:
            continue  # no gradient for this op (comparisons and the like)
        grads = fn(go, node.inputs(), node, g)
        for i, gi in enumerate(grads[:len(node.inputs())]):
            if gi is None:
                continue
            iid = node.inputs()[i].id()
            prev = grad_map.get(iid)
            grad_map[iid] = gi if prev is None else g.create_op(OpType.ADD, [prev, gi], _spec(gi.shape(), gi))


def backward(output: Tensor, grad_output: Optional[Tensor] = None) -> Dict[int, Tensor]:
    """AutogradEngine::backward: extends the output's graph with its backward
    graph and records on every PARAMETER and INPUT node the node holding its
    gradient (node.grad_node).  Returns {leaf node id: gradient Tensor}."""
    g = output.graph()
    go = grad_output.node() if grad_output is not None else ones_like(output.node(), g)
    grad_map = {output.node().id(): go}
    _propagate(grad_map, [output.node()], g)
    out = {}
    for nid, gn in grad_map.items():
        node = g.node(nid)
        if node is not None and (node.is_parameter() or node.is_input()):
            node.grad_node = gn
            out[nid] = Tensor(g, gn)
    return out


def grad(outputs: Sequence[Tensor], inputs: Sequence[Tensor],
         grad_outputs: Optional[Sequence[Optional[Tensor]]] = None) -> List[Optional[Tensor]]:
    """AutogradEngine::grad: gradients of `outputs` (seeded with ones, or
    `grad_outputs`) with respect to any nodes `inputs`, or None where no
    gradient reaches."""
    g = outputs[0].graph()
    grad_map = {}
    for i, o in enumerate(outputs):
        go = grad_outputs[i] if grad_outputs is not None and i < len(grad_outputs) else None
        grad_map[o.node().id()] = go.node() if go is not None else ones_like(o.node(), g)
    _propagate(grad_map, [o.node() for o in outputs], g)
    res = []
    for t in inputs:
        gn = grad_map.get(t.node().id())
        res.append(Tensor(g, gn) if gn is not None else None)
    return res
