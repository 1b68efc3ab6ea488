"""PyFlame's lazy IR, mirrored in Python: OpType, NodeType, DType, TensorSpec,
Node and Graph with the same values, names and behaviour as
include/pyflame/ir/{op_type,node,graph,shape_inference}.hpp and
include/pyflame/core/dtype.hpp.  Graphs built here are what the CUDA executor
evaluates; their node structure and attributes follow PyFlame's producers so
that a graph built by PyFlame's own C++ front end and one built here are the
same input to the executor.
"""
from __future__ import annotations

import enum
import itertools
from typing import Any, Dict, List, Optional, Sequence

import numpy as np


class OpType(enum.IntEnum):
    """op_type.hpp:9-124 (values are the interface)."""
    NONE = 0
    ADD = 100; SUB = 101; MUL = 102; DIV = 103; POW = 104; MAX_BINARY = 105; MIN_BINARY = 106
    NEG = 200; ABS = 201; SQRT = 202; EXP = 203; LOG = 204; SIN = 205; COS = 206; TANH = 207
    RELU = 300; SIGMOID = 301; GELU = 302; SILU = 303; SOFTMAX = 304; LOG_SOFTMAX = 305
    SUM = 400; MEAN = 401; MAX = 402; MIN = 403; PROD = 404
    MATMUL = 500; TRANSPOSE = 501; BATCH_MATMUL = 502
    CONV1D = 510; CONV2D = 511; CONV3D = 512; CONV_TRANSPOSE2D = 513
    MAX_POOL1D = 520; MAX_POOL2D = 521; MAX_POOL3D = 522; AVG_POOL1D = 523; AVG_POOL2D = 524
    AVG_POOL3D = 525; ADAPTIVE_AVG_POOL2D = 526; ADAPTIVE_AVG_POOL1D = 527
    BATCH_NORM = 530; LAYER_NORM = 531; GROUP_NORM = 532; INSTANCE_NORM = 533
    DROPOUT = 540; EMBEDDING = 545; GATHER = 546
    RESHAPE = 600; VIEW = 601; SQUEEZE = 602; UNSQUEEZE = 603; SLICE = 604; CONCAT = 605; STACK = 606
    BROADCAST = 607
    COPY = 700; CONTIGUOUS = 701; LAYOUT_TRANSFORM = 702
    EQ = 800; NE = 801; LT = 802; LE = 803; GT = 804; GE = 805; LESS = 806
    WHERE = 810; MAXIMUM = 811; MINIMUM = 812; CLAMP = 813
    NLL_LOSS = 850; CROSS_ENTROPY_LOSS = 851; MSE_LOSS = 852; L1_LOSS = 853; BCE_LOSS = 854
    BCE_WITH_LOGITS_LOSS = 855; KL_DIV_LOSS = 856; SMOOTH_L1_LOSS = 857
    CONSTANT = 900; INPUT = 901; PARAMETER = 902


def op_type_name(op: OpType) -> str:
    return OpType(op).name.lower()


def is_elementwise(op: OpType) -> bool:  # op_type.hpp:216-219
    v = int(op)
    return (100 <= v < 400) or (800 <= v < 900)


def is_reduction(op: OpType) -> bool:  # op_type.hpp:222-225
    return 400 <= int(op) < 500


class NodeType(enum.IntEnum):  # node.hpp:22-27
    CONSTANT = 0
    INPUT = 1
    PARAMETER = 2
    OPERATION = 3


class DType(enum.IntEnum):  # dtype.hpp:11-21
    float32 = 0
    float16 = 1
    bfloat16 = 2
    int32 = 3
    int16 = 4
    int8 = 5
    bool_ = 6
    float64 = 7
    int64 = 8


_NP = {DType.float32: np.float32, DType.float16: np.float16, DType.int32: np.int32, DType.int16: np.int16,
       DType.int8: np.int8, DType.bool_: np.uint8, DType.float64: np.float64, DType.int64: np.int64}
_SIZE = {DType.float32: 4, DType.float16: 2, DType.bfloat16: 2, DType.int32: 4, DType.int16: 2, DType.int8: 1,
         DType.bool_: 1, DType.float64: 8, DType.int64: 8}


def dtype_size(d: DType) -> int:
    return _SIZE[DType(d)]


def dtype_name(d: DType) -> str:
    return DType(d).name.rstrip("_")


def numpy_dtype(d: DType):
    if DType(d) == DType.bfloat16:
        raise TypeError("bfloat16 has no numpy dtype")
    return _NP[DType(d)]


def from_numpy_dtype(dt) -> DType:
    dt = np.dtype(dt)
    for k, v in _NP.items():
        if np.dtype(v) == dt and k != DType.bool_:
            return k
    if dt == np.bool_:
        return DType.bool_
    raise TypeError(f"unsupported numpy dtype {dt}")


MAX_TENSOR_DIMS = 8  # safe_math.hpp:144-147
MAX_TENSOR_NUMEL = 1 << 40


class TensorSpec:
    """node.hpp:30-68: shape + dtype (the Cerebras MeshLayout is not used)."""

    __slots__ = ("shape", "dtype")

    def __init__(self, shape: Sequence[int] = (), dtype: DType = DType.float32):
        self.shape = [int(s) for s in shape]
        self.dtype = DType(dtype)
        if any(s < 0 for s in self.shape):
            raise ValueError(f"negative dimension in shape {self.shape}")

    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n

    def size_bytes(self) -> int:
        return self.numel() * dtype_size(self.dtype)

    def ndim(self) -> int:
        return len(self.shape)

    def __eq__(self, o):
        return isinstance(o, TensorSpec) and self.shape == o.shape and self.dtype == o.dtype

    def __repr__(self):
        return f"TensorSpec({self.shape}, {dtype_name(self.dtype)})"


# C++ attribute value types (include/pyflame_cuda.h pfc_attr_type)
A_INT, A_INT64, A_FLOAT, A_DOUBLE, A_BOOL, A_INT64_VEC, A_INT_VEC, A_FLOAT_VEC = range(8)

_ids = itertools.count(1)


class Node:
    """node.hpp:74-229.  Attributes keep the C++ type the producer stored."""

    def __init__(self, nid: int, ntype: NodeType, name: str = ""):
        self._id = nid
        self._type = NodeType(ntype)
        self.name = name
        self._spec = TensorSpec()
        self._inputs: List["Node"] = []
        self._users: List["Node"] = []
        self._op = OpType.NONE
        self._attrs: Dict[str, tuple] = {}
        self._data: Optional[np.ndarray] = None
        self._data_key = 0

    # accessors mirroring node.hpp:82-96
    def id(self) -> int:
        return self._id

    def type(self) -> NodeType:
        return self._type

    def output_spec(self) -> TensorSpec:
        return self._spec

    def set_output_spec(self, s: TensorSpec):
        self._spec = s

    def shape(self) -> List[int]:
        return list(self._spec.shape)

    def dtype(self) -> DType:
        return self._spec.dtype

    def numel(self) -> int:
        return self._spec.numel()

    def ndim(self) -> int:
        return self._spec.ndim()

    def inputs(self) -> List["Node"]:
        return self._inputs

    def users(self) -> List["Node"]:
        return self._users

    def op_type(self) -> OpType:
        return self._op

    def set_op_type(self, op: OpType):
        self._op = OpType(op)

    def set_attr(self, key: str, value: Any, ctype: Optional[int] = None):
        """Store an attribute with the C++ type a PyFlame producer uses.  When
        `ctype` is omitted: bool -> bool, int -> int, float -> float,
        list of ints -> std::vector<int64_t>."""
        if ctype is None:
            if isinstance(value, (bool, np.bool_)):
                ctype = A_BOOL
            elif isinstance(value, (int, np.integer)):
                ctype = A_INT
            elif isinstance(value, (float, np.floating)):
                ctype = A_FLOAT
            elif isinstance(value, (list, tuple)):
                ctype = A_INT64_VEC if all(isinstance(v, (int, np.integer)) for v in value) else A_FLOAT_VEC
            else:
                raise TypeError(f"unsupported attribute value {value!r}")
        self._attrs[key] = (value if not isinstance(value, tuple) else list(value), ctype)

    def get_attr(self, key: str, default: Any = ...):
        if key not in self._attrs:
            if default is ...:
                raise RuntimeError(f"Attribute not found: {key}")
            return default
        return self._attrs[key][0]

    def has_attr(self, key: str) -> bool:
        return key in self._attrs

    def attrs(self) -> Dict[str, tuple]:
        return dict(self._attrs)

    def is_constant(self) -> bool:
        return self._type == NodeType.CONSTANT

    def is_input(self) -> bool:
        return self._type == NodeType.INPUT

    def is_parameter(self) -> bool:
        return self._type == NodeType.PARAMETER

    def is_operation(self) -> bool:
        return self._type == NodeType.OPERATION

    def set_constant_data(self, data: np.ndarray, copy: bool = True):
        """node.hpp:175-177.  By default the array is copied and frozen; with
        copy=False the caller's C-contiguous array is used in place (an
        INPUT node's per-call buffer, e.g. pinned host memory)."""
        if copy:
            arr = np.ascontiguousarray(np.array(data, dtype=numpy_dtype(self.dtype()), copy=True)).reshape(self.shape())
            arr.setflags(write=False)
        else:
            arr = data
            if not (isinstance(arr, np.ndarray) and arr.flags.c_contiguous and arr.dtype == numpy_dtype(self.dtype())
                    and list(arr.shape) == self.shape()):
                raise ValueError("copy=False needs a C-contiguous array of the node's shape and dtype")
        self._data = arr
        self._data_key = next(_ids)

    def constant_data(self) -> Optional[np.ndarray]:
        return self._data

    def has_constant_data(self) -> bool:
        return self._data is not None and self._data.size > 0

    def __repr__(self):
        if self.is_operation():
            ins = ", ".join(f"%{i.id()}" for i in self._inputs)
            return f"%{self._id} = {op_type_name(self._op)}({ins}) : {self._spec}"
        return f"%{self._id} = {self._type.name.lower()} : {self._spec}"


class Graph:
    """graph.hpp:17-215.  Ids count up from 0 per graph."""

    def __init__(self):
        self._next_id = 0
        self._nodes: List[Node] = []
        self._map: Dict[int, Node] = {}
        self._inputs: List[Node] = []
        self._outputs: List[Node] = []
        self._params: List[Node] = []
        self.version = 0

    def _add(self, n: Node) -> Node:
        self._nodes.append(n)
        self._map[n.id()] = n
        self.version += 1
        return n

    def create_constant(self, spec: TensorSpec, data=None, name: str = "") -> Node:
        n = Node(self._next_id, NodeType.CONSTANT, name)
        self._next_id += 1
        n.set_output_spec(spec)
        n.set_op_type(OpType.CONSTANT)
        if data is not None:
            n.set_constant_data(data)
        return self._add(n)

    def create_input(self, spec: TensorSpec, name: str = "") -> Node:
        n = Node(self._next_id, NodeType.INPUT, name)
        self._next_id += 1
        n.set_output_spec(spec)
        n.set_op_type(OpType.INPUT)
        self._inputs.append(n)
        return self._add(n)

    def create_parameter(self, spec: TensorSpec, name: str = "") -> Node:
        n = Node(self._next_id, NodeType.PARAMETER, name)
        self._next_id += 1
        n.set_output_spec(spec)
        n.set_op_type(OpType.PARAMETER)
        self._params.append(n)
        return self._add(n)

    def create_op(self, op_type: OpType, inputs: Sequence[Node], output_spec: TensorSpec, name: str = "") -> Node:
        n = Node(self._next_id, NodeType.OPERATION, name)
        self._next_id += 1
        n.set_output_spec(output_spec)
        n.set_op_type(op_type)
        n._inputs = list(inputs)
        for i in inputs:
            i._users.append(n)
        return self._add(n)

    def node(self, nid: int) -> Optional[Node]:
        return self._map.get(nid)

    get_node = node

    def mark_output(self, n: Node):
        if n not in self._outputs:
            self._outputs.append(n)
            self.version += 1

    def all_nodes(self) -> List[Node]:
        return list(self._nodes)

    nodes = all_nodes

    def inputs(self) -> List[Node]:
        return list(self._inputs)

    def outputs(self) -> List[Node]:
        return list(self._outputs)

    def parameters(self) -> List[Node]:
        return list(self._params)

    def num_nodes(self) -> int:
        return len(self._nodes)

    def num_ops(self) -> int:
        return sum(1 for n in self._nodes if n.is_operation())

    def topological_order(self, roots: Optional[Sequence[Node]] = None) -> List[Node]:
        """graph.hpp:136-164: DFS from the outputs (or every node), inputs first."""
        seen, order = set(), []
        starts = list(roots) if roots is not None else (self._outputs or self._nodes)
        for s in starts:
            stack = [(s, 0)]
            if s.id() in seen:
                continue
            seen.add(s.id())
            while stack:
                n, i = stack.pop()
                if i < len(n._inputs):
                    stack.append((n, i + 1))
                    c = n._inputs[i]
                    if c.id() not in seen:
                        seen.add(c.id())
                        stack.append((c, 0))
                else:
                    order.append(n)
        return order

    def estimated_memory_bytes(self) -> int:
        return sum(n.output_spec().size_bytes() for n in self._nodes)

    def clear(self):
        self.__init__()

    def __repr__(self):
        lines = ["Graph {"] + [f"  {n!r}" for n in self.topological_order()] + ["}"]
        return "\n".join(lines)


# ---------------------------------------------------------------------------
# shape inference (shape_inference.hpp)
# ---------------------------------------------------------------------------

def broadcast_shapes(a: Sequence[int], b: Sequence[int]) -> List[int]:
    """shape_inference.hpp:16-42."""
    n = max(len(a), len(b))
    out = [0] * n
    for i in range(n):
        da = a[len(a) - 1 - i] if i < len(a) else 1
        db = b[len(b) - 1 - i] if i < len(b) else 1
        if da == db:
            out[n - 1 - i] = da
        elif da == 1:
            out[n - 1 - i] = db
        elif db == 1:
            out[n - 1 - i] = da
        else:
            raise RuntimeError(f"Shapes are not broadcastable: dimension {da} vs {db}")
    return out


def infer_binary_op_spec(a: TensorSpec, b: TensorSpec) -> TensorSpec:
    if a.dtype != b.dtype:
        raise RuntimeError("Binary operation requires matching dtypes")
    return TensorSpec(broadcast_shapes(a.shape, b.shape), a.dtype)


def infer_reduction_spec(x: TensorSpec, dim: Optional[int], keepdim: bool) -> TensorSpec:
    """shape_inference.hpp:109-143."""
    if dim is None:
        return TensorSpec([1] * len(x.shape) if keepdim else [], x.dtype)
    d = dim + len(x.shape) if dim < 0 else dim
    if d < 0 or d >= len(x.shape):
        raise RuntimeError("Reduction dimension out of range")
    shape = []
    for i, s in enumerate(x.shape):
        if i == d:
            if keepdim:
                shape.append(1)
        else:
            shape.append(s)
    return TensorSpec(shape, x.dtype)


def infer_matmul_spec(a: TensorSpec, b: TensorSpec) -> TensorSpec:
    """shape_inference.hpp:146-217."""
    if not a.shape or not b.shape:
        raise RuntimeError("matmul requires non-scalar inputs")
    if a.dtype != b.dtype:
        raise RuntimeError("matmul requires matching dtypes")
    if len(a.shape) == 1 and len(b.shape) == 1:
        if a.shape[0] != b.shape[0]:
            raise RuntimeError("matmul: incompatible shapes for dot product")
        return TensorSpec([], a.dtype)
    if len(a.shape) == 2 and len(b.shape) == 2:
        if a.shape[1] != b.shape[0]:
            raise RuntimeError(f"matmul: shapes not aligned: {a.shape[1]} vs {b.shape[0]}")
        return TensorSpec([a.shape[0], b.shape[1]], a.dtype)
    if len(a.shape) == 1 and len(b.shape) == 2:
        if a.shape[0] != b.shape[0]:
            raise RuntimeError("matmul: shapes not aligned")
        return TensorSpec([b.shape[1]], a.dtype)
    if len(a.shape) == 2 and len(b.shape) == 1:
        if a.shape[1] != b.shape[0]:
            raise RuntimeError("matmul: shapes not aligned")
        return TensorSpec([a.shape[0]], a.dtype)
    batch = broadcast_shapes(a.shape[:-2], b.shape[:-2])
    if a.shape[-1] != b.shape[-2]:
        raise RuntimeError("matmul: inner dimensions don't match")
    return TensorSpec(batch + [a.shape[-2], b.shape[-1]], a.dtype)


def infer_transpose_spec(x: TensorSpec, d0: int, d1: int) -> TensorSpec:
    n = len(x.shape)
    d0 = d0 + n if d0 < 0 else d0
    d1 = d1 + n if d1 < 0 else d1
    if not (0 <= d0 < n and 0 <= d1 < n):
        raise RuntimeError("transpose: dimension out of range")
    s = list(x.shape)
    s[d0], s[d1] = s[d1], s[d0]
    return TensorSpec(s, x.dtype)


def infer_reshape_spec(x: TensorSpec, new_shape: Sequence[int]) -> TensorSpec:
    """shape_inference.hpp:242-280."""
    numel = x.numel()
    out, neg, known = list(new_shape), -1, 1
    for i, s in enumerate(new_shape):
        if s == -1:
            if neg >= 0:
                raise RuntimeError("reshape: only one -1 allowed")
            neg = i
        elif s < 0:
            raise RuntimeError("reshape: invalid dimension")
        else:
            known *= s
    if neg >= 0:
        if known == 0 or numel % known != 0:
            raise RuntimeError("reshape: cannot infer -1 dimension")
        out[neg] = numel // known
    elif known != numel:
        raise RuntimeError("reshape: total elements must match")
    return TensorSpec(out, x.dtype)


def infer_concat_spec(specs: Sequence[TensorSpec], dim: int) -> TensorSpec:
    if not specs:
        raise RuntimeError("concat: requires at least one input")
    f = specs[0]
    n = len(f.shape)
    d = dim + n if dim < 0 else dim
    if not 0 <= d < n:
        raise RuntimeError("concat: dimension out of range")
    out = list(f.shape)
    for s in specs[1:]:
        if s.dtype != f.dtype:
            raise RuntimeError("concat: all inputs must have same dtype")
        if len(s.shape) != n:
            raise RuntimeError("concat: all inputs must have same number of dimensions")
        for k in range(n):
            if k == d:
                out[d] += s.shape[k]
            elif s.shape[k] != f.shape[k]:
                raise RuntimeError("concat: shapes don't match on non-concat dimension")
    return TensorSpec(out, f.dtype)


def infer_slice_spec(x: TensorSpec, dim: int, start: int, end: int) -> TensorSpec:
    """shape_inference.hpp:336-368."""
    n = len(x.shape)
    d = dim + n if dim < 0 else dim
    if not 0 <= d < n:
        raise RuntimeError("slice: dimension out of range")
    size = x.shape[d]
    start = start + size if start < 0 else start
    end = end + size if end < 0 else end
    start = max(0, min(start, size))
    end = max(0, min(end, size))
    if end <= start:
        raise RuntimeError("slice: end must be greater than start")
    s = list(x.shape)
    s[d] = end - start
    return TensorSpec(s, x.dtype)
