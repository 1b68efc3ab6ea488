"""Lazy Tensor API mirroring PyFlame's `Tensor` (src/core/tensor.cpp,
src/core/tensor_impl.cpp): every operation adds a node to the thread's
current graph (src/core/context.cpp:7-18) with the same op type, output spec
and attributes as PyFlame; `eval()` / `numpy()` evaluate the node's subgraph
on the selected CUDA device through the executor boundary.
"""
from __future__ import annotations

import threading
from typing import List, Optional, Sequence, Union

import numpy as np

from . import ir
from .ir import DType, Graph, Node, OpType, TensorSpec

_tls = threading.local()


def get_current_graph() -> Graph:
    """context.cpp:7-18: one graph per thread."""
    g = getattr(_tls, "graph", None)
    if g is None:
        g = Graph()
        _tls.graph = g
    return g


def reset_graph() -> None:
    _tls.graph = Graph()


_rng = np.random.default_rng(0)


def manual_seed(seed: int) -> None:
    global _rng
    _rng = np.random.default_rng(seed)


Scalar = Union[int, float]


class Tensor:
    """A handle to one node of a lazy graph (core/tensor.hpp:22-175)."""

    __slots__ = ("_graph", "_node", "_data", "__weakref__")

    def __init__(self, graph: Graph, node: Node):
        self._graph = graph
        self._node = node
        self._data: Optional[np.ndarray] = node.constant_data() if node.is_constant() else None

    # ---- factories (tensor.cpp:40-66, tensor_impl.hpp:47-101) -------------
    @staticmethod
    def from_data(data, shape: Optional[Sequence[int]] = None, dtype: DType = DType.float32) -> "Tensor":
        arr = np.asarray(data, dtype=ir.numpy_dtype(dtype))
        if shape is not None:
            arr = arr.reshape(shape)
        g = get_current_graph()
        return Tensor(g, g.create_constant(TensorSpec(arr.shape, dtype), arr))

    @staticmethod
    def input(data: np.ndarray, copy: bool = True) -> "Tensor":
        """An INPUT node (graph.hpp:53-64) carrying per-call data: its payload
        is uploaded on every evaluation instead of being kept on the device."""
        arr = np.asarray(data)
        dtype = ir.from_numpy_dtype(arr.dtype)
        g = get_current_graph()
        n = g.create_input(TensorSpec(arr.shape, dtype))
        n.set_constant_data(arr, copy=copy)
        return Tensor(g, n)

    @staticmethod
    def zeros(shape, dtype: DType = DType.float32) -> "Tensor":
        return Tensor.from_data(np.zeros(shape, ir.numpy_dtype(dtype)), dtype=dtype)

    @staticmethod
    def ones(shape, dtype: DType = DType.float32) -> "Tensor":
        return Tensor.from_data(np.ones(shape, ir.numpy_dtype(dtype)), dtype=dtype)

    @staticmethod
    def full(shape, value: float, dtype: DType = DType.float32) -> "Tensor":
        return Tensor.from_data(np.full(shape, value, ir.numpy_dtype(dtype)), dtype=dtype)

    @staticmethod
    def randn(shape, dtype: DType = DType.float32) -> "Tensor":
        return Tensor.from_data(_rng.standard_normal(shape).astype(ir.numpy_dtype(dtype)), dtype=dtype)

    @staticmethod
    def rand(shape, dtype: DType = DType.float32) -> "Tensor":
        return Tensor.from_data(_rng.random(shape).astype(ir.numpy_dtype(dtype)), dtype=dtype)

    @staticmethod
    def arange(start: int, end: int, step: int = 1, dtype: DType = DType.float32) -> "Tensor":
        return Tensor.from_data(np.arange(start, end, step).astype(ir.numpy_dtype(dtype)), dtype=dtype)

    # ---- properties --------------------------------------------------------
    @property
    def shape(self) -> List[int]:
        return self._node.shape()

    def size(self, dim: int) -> int:
        s = self.shape
        d = dim + len(s) if dim < 0 else dim
        return s[d] if 0 <= d < len(s) else 0

    def numel(self) -> int:
        return self._node.numel()

    @property
    def dtype(self) -> DType:
        return self._node.dtype()

    @property
    def ndim(self) -> int:
        return self._node.ndim()

    def node(self) -> Node:
        return self._node

    def graph(self) -> Graph:
        return self._graph

    def is_evaluated(self) -> bool:
        return self._data is not None

    # ---- graph construction helpers (tensor_impl.cpp:467-582) -------------
    def _unary(self, op: OpType) -> "Tensor":
        g = self._graph
        n = g.create_op(op, [self._node], TensorSpec(self.shape, self.dtype), f"{ir.op_type_name(op)}_{g.num_nodes()}")
        return Tensor(g, n)

    def _binary(self, op: OpType, other: "Tensor") -> "Tensor":
        g = self._graph
        spec = ir.infer_binary_op_spec(self._node.output_spec(), other._node.output_spec())
        n = g.create_op(op, [self._node, other._node], spec, f"{ir.op_type_name(op)}_{g.num_nodes()}")
        return Tensor(g, n)

    def _scalar(self, v: Scalar) -> "Tensor":
        # tensor.cpp:452-466: a scalar becomes a full-size constant
        return Tensor.full(self.shape, float(v), self.dtype)

    def _reduction(self, op: OpType, dim: Optional[int], keepdim: bool) -> "Tensor":
        g = self._graph
        spec = ir.infer_reduction_spec(self._node.output_spec(), dim, keepdim)
        n = g.create_op(op, [self._node], spec, f"{ir.op_type_name(op)}_{g.num_nodes()}")
        if dim is not None:
            n.set_attr("dim", int(dim), ir.A_INT)
        n.set_attr("keepdim", bool(keepdim), ir.A_BOOL)
        return Tensor(g, n)

    # ---- arithmetic (tensor.cpp:427-466) ----------------------------------
    def __add__(self, o):
        return self._binary(OpType.ADD, o if isinstance(o, Tensor) else self._scalar(o))

    def __sub__(self, o):
        return self._binary(OpType.SUB, o if isinstance(o, Tensor) else self._scalar(o))

    def __mul__(self, o):
        return self._binary(OpType.MUL, o if isinstance(o, Tensor) else self._scalar(o))

    def __truediv__(self, o):
        return self._binary(OpType.DIV, o if isinstance(o, Tensor) else self._scalar(o))

    def __radd__(self, o):
        return self._scalar(o)._binary(OpType.ADD, self)

    def __rsub__(self, o):
        return self._scalar(o)._binary(OpType.SUB, self)

    def __rmul__(self, o):
        return self._scalar(o)._binary(OpType.MUL, self)

    def __rtruediv__(self, o):
        return self._scalar(o)._binary(OpType.DIV, self)

    def __neg__(self):
        return self._unary(OpType.NEG)

    def __matmul__(self, o):
        return matmul(self, o)

    # comparisons (tensor.cpp:546-574) produce 0/1 float tensors
    def __eq__(self, o):  # type: ignore[override]
        return self._binary(OpType.EQ, o if isinstance(o, Tensor) else self._scalar(o))

    def __ne__(self, o):  # type: ignore[override]
        return self._binary(OpType.NE, o if isinstance(o, Tensor) else self._scalar(o))

    def __lt__(self, o):
        return self._binary(OpType.LT, o if isinstance(o, Tensor) else self._scalar(o))

    def __le__(self, o):
        return self._binary(OpType.LE, o if isinstance(o, Tensor) else self._scalar(o))

    def __gt__(self, o):
        return self._binary(OpType.GT, o if isinstance(o, Tensor) else self._scalar(o))

    def __ge__(self, o):
        return self._binary(OpType.GE, o if isinstance(o, Tensor) else self._scalar(o))

    __hash__ = object.__hash__

    # ---- reductions (tensor.cpp:517-540) -----------------------------------
    def sum(self, dim: Optional[int] = None, keepdim: bool = False):
        return self._reduction(OpType.SUM, dim, keepdim)

    def mean(self, dim: Optional[int] = None, keepdim: bool = False):
        return self._reduction(OpType.MEAN, dim, keepdim)

    def max(self, dim: Optional[int] = None, keepdim: bool = False):
        return self._reduction(OpType.MAX, dim, keepdim)

    def min(self, dim: Optional[int] = None, keepdim: bool = False):
        return self._reduction(OpType.MIN, dim, keepdim)

    def prod(self, dim: Optional[int] = None, keepdim: bool = False):
        return self._reduction(OpType.PROD, dim, keepdim)

    # ---- shape ops (tensor.cpp:176-311) ------------------------------------
    def reshape(self, new_shape: Sequence[int]) -> "Tensor":
        g = self._graph
        new_shape = [int(s) for s in new_shape]
        spec = ir.infer_reshape_spec(self._node.output_spec(), new_shape)
        n = g.create_op(OpType.RESHAPE, [self._node], spec, f"reshape_{g.num_nodes()}")
        n.set_attr("new_shape", new_shape, ir.A_INT64_VEC)
        return Tensor(g, n)

    view = reshape

    def transpose(self, dim0: int, dim1: int) -> "Tensor":
        g = self._graph
        spec = ir.infer_transpose_spec(self._node.output_spec(), dim0, dim1)
        n = g.create_op(OpType.TRANSPOSE, [self._node], spec, f"transpose_{g.num_nodes()}")
        n.set_attr("dim0", int(dim0), ir.A_INT)
        n.set_attr("dim1", int(dim1), ir.A_INT)
        return Tensor(g, n)

    def t(self) -> "Tensor":
        if self.ndim != 2:
            raise RuntimeError("t() expects a 2D tensor")
        return self.transpose(0, 1)

    def squeeze(self, dim: int = -1) -> "Tensor":
        s = self.shape
        if dim == -1:
            ns = [d for d in s if d != 1]
        else:
            dim = dim + len(s) if dim < 0 else dim
            ns = [d for i, d in enumerate(s) if not (i == dim and d == 1)]
        return self.reshape(ns)

    def unsqueeze(self, dim: int) -> "Tensor":
        s = self.shape
        dim = dim + len(s) + 1 if dim < 0 else dim
        ns = []
        for i in range(len(s) + 1):
            if i == dim:
                ns.append(1)
            if i < len(s):
                ns.append(s[i])
        return self.reshape(ns)

    def contiguous(self) -> "Tensor":
        return self

    def clone(self) -> "Tensor":
        return self

    def slice(self, dim: int, start: int, end: int) -> "Tensor":
        g = self._graph
        spec = ir.infer_slice_spec(self._node.output_spec(), dim, start, end)
        nd = self.ndim
        dim = dim + nd if dim < 0 else dim
        size = self.shape[dim]
        start = start + size if start < 0 else start
        end = end + size if end < 0 else end
        start, end = max(0, min(start, size)), max(0, min(end, size))
        n = g.create_op(OpType.SLICE, [self._node], spec, f"slice_{g.num_nodes()}")
        n.set_attr("dim", int(dim), ir.A_INT)
        n.set_attr("start", int(start), ir.A_INT64)
        n.set_attr("end", int(end), ir.A_INT64)
        return Tensor(g, n)

    def __getitem__(self, idx: int) -> "Tensor":
        s = self.shape
        if not s:
            raise RuntimeError("Cannot index a scalar tensor")
        if idx < 0:
            idx += s[0]
        if idx < 0 or idx >= s[0]:
            raise IndexError(f"Index {idx} out of bounds for dimension of size {s[0]}")
        sl = self.slice(0, idx, idx + 1)
        return sl.squeeze(0) if len(s) > 1 else sl

    # ---- evaluation ---------------------------------------------------------
    def eval(self) -> "Tensor":
        if self._data is None:
            from . import device
            self._data = device.evaluate([self])[0]
        return self

    def numpy(self) -> np.ndarray:
        self.eval()
        return np.array(self._data, copy=True)

    def data(self) -> np.ndarray:
        return self.numpy()

    def to(self, dtype: DType) -> "Tensor":
        """tensor.cpp:324-421: evaluate, convert on the host, new constant."""
        if dtype == self.dtype:
            return self
        return Tensor.from_data(self.numpy().astype(ir.numpy_dtype(dtype)), dtype=dtype)

    def __repr__(self):
        return f"Tensor(shape={self.shape}, dtype={ir.dtype_name(self.dtype)})"


# ---- free functions (tensor.cpp:624-849) --------------------------------------

def tensor(data, dtype: DType = DType.float32) -> Tensor:
    return Tensor.from_data(data, dtype=dtype)


def from_numpy(arr: np.ndarray, dtype: Optional[DType] = None) -> Tensor:
    return Tensor.from_data(arr, dtype=dtype if dtype is not None else ir.from_numpy_dtype(arr.dtype))


zeros, ones, full, randn, rand, arange = (Tensor.zeros, Tensor.ones, Tensor.full, Tensor.randn, Tensor.rand,
                                          Tensor.arange)


def matmul(a: Tensor, b: Tensor) -> Tensor:
    g = a.graph()
    spec = ir.infer_matmul_spec(a.node().output_spec(), b.node().output_spec())
    return Tensor(g, g.create_op(OpType.MATMUL, [a.node(), b.node()], spec, f"matmul_{g.num_nodes()}"))


def relu(x: Tensor) -> Tensor:
    return x._unary(OpType.RELU)


def sigmoid(x: Tensor) -> Tensor:
    return x._unary(OpType.SIGMOID)


def tanh(x: Tensor) -> Tensor:
    return x._unary(OpType.TANH)


def gelu(x: Tensor) -> Tensor:
    return x._unary(OpType.GELU)


def silu(x: Tensor) -> Tensor:
    return x._unary(OpType.SILU)


def abs(x: Tensor) -> Tensor:  # noqa: A001 - PyFlame's name
    return x._unary(OpType.ABS)


def sqrt(x: Tensor) -> Tensor:
    return x._unary(OpType.SQRT)


def exp(x: Tensor) -> Tensor:
    return x._unary(OpType.EXP)


def log(x: Tensor) -> Tensor:
    return x._unary(OpType.LOG)


def sin(x: Tensor) -> Tensor:
    return x._unary(OpType.SIN)


def cos(x: Tensor) -> Tensor:
    return x._unary(OpType.COS)


def _softmax_like(x: Tensor, dim: int, op: OpType, name: str) -> Tensor:
    g = x.graph()
    n = g.create_op(op, [x.node()], TensorSpec(x.shape, x.dtype), f"{name}_{g.num_nodes()}")
    n.set_attr("dim", int(dim), ir.A_INT)
    return Tensor(g, n)


def softmax(x: Tensor, dim: int = -1) -> Tensor:
    return _softmax_like(x, dim, OpType.SOFTMAX, "softmax")


def log_softmax(x: Tensor, dim: int = -1) -> Tensor:
    return _softmax_like(x, dim, OpType.LOG_SOFTMAX, "log_softmax")


def pow(base: Tensor, exponent) -> Tensor:  # noqa: A001
    e = exponent if isinstance(exponent, Tensor) else Tensor.full(base.shape, float(exponent), base.dtype)
    return base._binary(OpType.POW, e)


def clamp(x: Tensor, min_val: float, max_val: float) -> Tensor:
    """tensor.cpp:749-767 (composite of comparisons and arithmetic)."""
    lo = Tensor.full(x.shape, min_val, x.dtype)
    hi = Tensor.full(x.shape, max_val, x.dtype)
    below, above = x < lo, x > hi
    in_range = (x >= lo) * (x <= hi)
    return x * in_range + lo * below + hi * above


def maximum(a: Tensor, b: Tensor) -> Tensor:
    """tensor.cpp:769-775."""
    return a * (a >= b) + b * (a < b)


def minimum(a: Tensor, b: Tensor) -> Tensor:
    """tensor.cpp:777-783."""
    return a * (a <= b) + b * (a > b)


def cat(tensors: Sequence[Tensor], dim: int = 0) -> Tensor:
    g = tensors[0].graph()
    spec = ir.infer_concat_spec([t.node().output_spec() for t in tensors], dim)
    n = g.create_op(OpType.CONCAT, [t.node() for t in tensors], spec, f"concat_{g.num_nodes()}")
    n.set_attr("dim", int(dim), ir.A_INT)
    return Tensor(g, n)


def stack(tensors: Sequence[Tensor], dim: int = 0) -> Tensor:
    return cat([t.unsqueeze(dim) for t in tensors], dim)


def broadcast_to(x: Tensor, shape: Sequence[int]) -> Tensor:
    return x.reshape(shape)  # tensor.cpp:845-849
