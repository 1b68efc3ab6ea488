"""ORACLE — test infrastructure, not product code.

Python access to the two CPU checkers:

* `run(graph, ids, precision)`: the C++ restatement (oracle.cpp, built into
  oracle/liboracle.so) evaluating a pyflame_b200.ir.Graph in float (PyFlame's
  fp32 arithmetic order) or double (fp64 shadow).
* `Reference`: PyFlame's own code compiled from its sources
  (oracle/_ref/libpyflame_ref.so): the CPU reference executor
  (src/backend/executor.cpp:205-524), the scalar kernels ops::*_cpu, and
  graphs built by PyFlame's own nn front end.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Dict, Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libpyflame_ref.so"

_lib = None
_ref = None


def build(with_reference: bool = True, reference_tree: str = "") -> None:
    """Compile liboracle.so, and the reference shim when a PyFlame source
    tree is given (`reference_tree`, else the PYFLAME_REFERENCE environment
    variable) and present."""
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)
    tree = reference_tree or os.environ.get("PYFLAME_REFERENCE", "")
    if with_reference and tree and Path(tree, "src").exists():
        subprocess.run(["make", "-s", "-j8", "-C", str(HERE), "ref", f"REF={tree}"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build(with_reference=False)
        L = C.CDLL(str(LIB))
        L.orc_graph_create.restype = C.c_void_p
        L.orc_graph_destroy.argtypes = [C.c_void_p]
        L.orc_last_error.restype = C.c_char_p
        L.orc_add_node.argtypes = [C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.POINTER(C.c_int64), C.c_int, C.POINTER(C.c_uint64)]
        L.orc_set_attr.argtypes = [C.c_void_p, C.c_uint64, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
        L.orc_set_constant.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_size_t]
        L.orc_execute.argtypes = [C.c_void_p, C.POINTER(C.c_uint64), C.c_int, C.POINTER(C.c_void_p), C.c_int]
        _lib = L
    return _lib


def _attr_buf(val, ct):
    if ct == 0:
        return C.c_int32(int(val)), 1
    if ct == 1:
        return C.c_int64(int(val)), 1
    if ct == 2:
        return C.c_float(float(val)), 1
    if ct == 3:
        return C.c_double(float(val)), 1
    if ct == 4:
        return C.c_uint8(1 if val else 0), 1
    if ct == 5:
        return (C.c_int64 * max(1, len(val)))(*map(int, val)), len(val)
    if ct == 6:
        return (C.c_int32 * max(1, len(val)))(*map(int, val)), len(val)
    return (C.c_float * max(1, len(val)))(*map(float, val)), len(val)


def _fill(graph, ids, add, set_attr, set_const):
    roots = [graph.node(i) for i in ids]
    keep = []
    for n in graph.topological_order(roots):
        shape = (C.c_int64 * max(1, n.ndim()))(*n.shape())
        ins = (C.c_uint64 * max(1, len(n.inputs())))(*[i.id() for i in n.inputs()])
        add(n.id(), int(n.type()), int(n.op_type()), int(n.dtype()), n.ndim(), shape, len(n.inputs()), ins)
        for k, (v, ct) in n.attrs().items():
            buf, cnt = _attr_buf(v, ct)
            keep.append(buf)
            set_attr(n.id(), k.encode(), ct, C.byref(buf), cnt)
        if n.has_constant_data():
            arr = np.ascontiguousarray(n.constant_data())
            keep.append(arr)
            set_const(n.id(), arr.ctypes.data, arr.nbytes)
    return keep


def run(graph, output_ids: Sequence[int], precision: str = "f32") -> Dict[int, np.ndarray]:
    """Evaluate `output_ids` of a pyflame_b200.ir.Graph on the CPU."""
    L = lib()
    g = L.orc_graph_create()
    try:
        keep = _fill(graph, output_ids,
                     lambda *a: L.orc_add_node(g, *a),
                     lambda *a: L.orc_set_attr(g, *a),
                     lambda nid, p, n: L.orc_set_constant(g, nid, p, n))
        dt = np.float32 if precision == "f32" else np.float64
        outs = [np.empty(graph.node(i).shape(), dtype=dt) for i in output_ids]
        ids = (C.c_uint64 * len(output_ids))(*output_ids)
        ptrs = (C.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
        if L.orc_execute(g, ids, len(outs), ptrs, 0 if precision == "f32" else 1) != 0:
            raise RuntimeError("oracle: " + L.orc_last_error().decode())
        del keep
        return dict(zip(output_ids, outs))
    finally:
        L.orc_graph_destroy(g)


def num_threads() -> int:
    L = lib()
    L.orc_num_threads.restype = C.c_int
    return L.orc_num_threads()


def set_threads(n: int) -> None:
    """Worker threads of later oracle calls made from the calling Python
    thread (0 restores the default: ORACLE_THREADS or every host thread)."""
    L = lib()
    L.orc_set_threads.argtypes = [C.c_int]
    L.orc_set_threads(int(n))


class Reference:
    """PyFlame's own CPU code (oracle/_ref/libpyflame_ref.so)."""

    def __init__(self):
        global _ref
        if _ref is None:
            if not REF_LIB.exists():
                raise FileNotFoundError(f"{REF_LIB} not built (needs the PyFlame sources: make -C oracle ref)")
            L = C.CDLL(str(REF_LIB))
            L.ref_graph_create.restype = C.c_void_p
            L.ref_graph_destroy.argtypes = [C.c_void_p]
            L.ref_last_error.restype = C.c_char_p
            L.ref_add_node.argtypes = [C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.POINTER(C.c_int64), C.c_int, C.POINTER(C.c_uint64)]
            L.ref_set_attr.argtypes = [C.c_void_p, C.c_uint64, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
            L.ref_set_constant.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_size_t]
            L.ref_execute_cpu.argtypes = [C.c_void_p, C.POINTER(C.c_uint64), C.c_int, C.POINTER(C.c_void_p)]
            f = C.POINTER(C.c_float)
            L.ref_unary.argtypes = [C.c_int, f, f, C.c_int64]
            L.ref_binary.argtypes = [C.c_int, f, f, f, C.c_int64]
            L.ref_softmax.argtypes = [f, f, C.c_int64, C.c_int64]
            L.ref_log_softmax.argtypes = [f, f, C.c_int64, C.c_int64]
            L.ref_reduce_dim.argtypes = [C.c_int, f, f, C.c_int64, C.c_int64, C.c_int]
            L.ref_matmul.argtypes = [f, f, f, C.c_int64, C.c_int64, C.c_int64]
            L.ref_batch_matmul.argtypes = [f, f, f, C.c_int64, C.c_int64, C.c_int64, C.c_int64]
            L.ref_matmul_a_bt.argtypes = [f, f, f, C.c_int64, C.c_int64, C.c_int64]
            L.ref_build.argtypes = [C.c_int, C.c_char_p, C.c_size_t]
            _ref = L
        self.L = _ref

    @staticmethod
    def available() -> bool:
        return REF_LIB.exists()

    def execute_cpu(self, graph, output_ids: Sequence[int]) -> Dict[int, np.ndarray]:
        """backend::Executor{Backend::CPU}.execute on the same graph."""
        L = self.L
        g = L.ref_graph_create()
        try:
            keep = _fill(graph, output_ids,
                         lambda *a: L.ref_add_node(g, *a),
                         lambda *a: L.ref_set_attr(g, *a),
                         lambda nid, p, n: L.ref_set_constant(g, nid, p, n))
            outs = [np.empty(graph.node(i).shape(), dtype=np.float32) for i in output_ids]
            ids = (C.c_uint64 * len(output_ids))(*output_ids)
            ptrs = (C.c_void_p * len(outs))(*[o.ctypes.data for o in outs])
            if L.ref_execute_cpu(g, ids, len(outs), ptrs) != 0:
                raise RuntimeError("reference executor: " + L.ref_last_error().decode())
            del keep
            return dict(zip(output_ids, outs))
        finally:
            L.ref_graph_destroy(g)

    @staticmethod
    def _p(a):
        return a.ctypes.data_as(C.POINTER(C.c_float))

    UNARY = {"relu": 0, "sigmoid": 1, "tanh": 2, "gelu": 3, "silu": 4, "exp": 5, "log": 6, "sqrt": 7}
    BINARY = {"add": 0, "sub": 1, "mul": 2, "div": 3}
    REDUCE = {"sum": 0, "mean": 1, "max": 2, "min": 3}

    def unary(self, name: str, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.L.ref_unary(self.UNARY[name], self._p(x), self._p(out), x.size)
        return out

    def binary(self, name: str, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty_like(a)
        self.L.ref_binary(self.BINARY[name], self._p(a), self._p(b), self._p(out), a.size)
        return out

    def softmax(self, x: np.ndarray, log: bool = False) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        f = self.L.ref_log_softmax if log else self.L.ref_softmax
        f(self._p(x), self._p(out), x.shape[0], x.shape[1])
        return out

    def reduce_dim(self, name: str, x: np.ndarray, dim: int) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(x.shape[1 - dim], np.float32)
        self.L.ref_reduce_dim(self.REDUCE[name], self._p(x), self._p(out), x.shape[0], x.shape[1], dim)
        return out

    def matmul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        out = np.empty((a.shape[0], b.shape[1]), np.float32)
        self.L.ref_matmul(self._p(a), self._p(b), self._p(out), a.shape[0], a.shape[1], b.shape[1])
        return out

    def batch_matmul(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        B, M, K = a.shape
        N = b.shape[2]
        out = np.empty((B, M, N), np.float32)
        self.L.ref_batch_matmul(self._p(a), self._p(b), self._p(out), B, M, K, N)
        return out

    def matmul_a_bt(self, a: np.ndarray, bt: np.ndarray) -> np.ndarray:
        a = np.ascontiguousarray(a, np.float32)
        bt = np.ascontiguousarray(bt, np.float32)
        out = np.empty((a.shape[0], bt.shape[0]), np.float32)
        self.L.ref_matmul_a_bt(self._p(a), self._p(bt), self._p(out), a.shape[0], a.shape[1], bt.shape[0])
        return out

    @staticmethod
    def build(kind: int) -> str:
        """Graph made by PyFlame's own front end, one line per node
        (run in a separate process: oracle/_ref/ref_dump)."""
        r = subprocess.run([str(HERE / "_ref" / "ref_dump"), str(kind)], capture_output=True, text=True, check=True)
        return r.stdout.split("----")[0]
