"""PyFlame's executor boundary with a CUDA backend.

Mirrors `pyflame::backend::Executor` (src/backend/executor.cpp:137-194):
`Backend`, `ExecutorConfig`, `ExecutionResult`, `Executor.execute(graph,
output_ids)`, and the backend class `CudaExecutor` shaped like
`rocm::ROCmExecutor` (include/pyflame/backend/rocm/rocm_executor.hpp:37-194),
plus the device functions of rocm_backend.hpp:119-139 as `cuda_*`.

Graphs are handed to libpyflame_cuda.so through its C ABI; evaluation happens
only on the GPU.  `Backend.CPU` is PyFlame's own reference executor and is not
part of this package: selecting it returns a failed ExecutionResult.
"""
from __future__ import annotations

import ctypes as C
import enum
import threading
import weakref
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _native as N
from .ir import A_BOOL, A_DOUBLE, A_FLOAT, A_FLOAT_VEC, A_INT, A_INT64, A_INT64_VEC, A_INT_VEC, Graph, Node, \
    NodeType, numpy_dtype

PFC_CONST_RESIDENT = 0x2
PRECISIONS = {"tf32x3": 0, "bf16": 1}


class Backend(enum.Enum):
    """executor.cpp:138-145 with CUDA in place of ROCM."""
    CPU = "cpu"
    SIMULATOR = "cerebras:simulator"
    HARDWARE = "cerebras"
    CUDA = "cuda"


@dataclass
class ExecutorConfig:
    """executor.cpp:163-168 plus the CUDA executor's options."""
    backend: Backend = Backend.CUDA
    enable_profiling: bool = False
    cache_compiled_kernels: bool = True
    device_address: str = "localhost:9000"
    device_id: int = 0
    precision: str = "tf32x3"
    use_cuda_graph: bool = True


@dataclass
class ExecutionResult:
    """executor.cpp:148-160; outputs map node id -> numpy array."""
    success: bool = False
    error_message: str = ""
    compile_time_ms: float = 0.0
    transfer_time_ms: float = 0.0
    compute_time_ms: float = 0.0
    total_time_ms: float = 0.0
    outputs: Dict[int, np.ndarray] = field(default_factory=dict)
    kernel_launches: int = 0
    h2d_bytes: int = 0   # host->device bytes the call copied (inputs, constants not yet resident)
    d2h_bytes: int = 0   # device->host bytes the call copied (outputs)


@dataclass
class DeviceInfo:
    """rocm_backend.hpp:100-109."""
    device_id: int
    name: str
    architecture: str
    total_memory: int
    free_memory: int
    compute_units: int
    max_threads_per_block: int
    warp_size: int


@dataclass
class MemoryStats:
    """rocm_memory.hpp:14-21 (+ bytes of device-resident constants)."""
    total_allocated: int
    peak_allocated: int
    total_allocations: int
    total_deallocations: int
    cache_hits: int
    cache_misses: int
    resident_constant_bytes: int


# ---------------------------------------------------------------------------
# device functions (bindings.cpp:430-463 as cuda_*)
# ---------------------------------------------------------------------------

def cuda_is_available() -> bool:
    try:
        return bool(N.lib().pfc_cuda_is_available())
    except RuntimeError:
        return False


def cuda_device_count() -> int:
    n = C.c_int(0)
    N.check(N.lib().pfc_cuda_get_device_count(C.byref(n)))
    return n.value


def cuda_get_device() -> int:
    d = C.c_int(-1)
    N.check(N.lib().pfc_cuda_get_device(C.byref(d)))
    return d.value


def cuda_set_device(device_id: int) -> None:
    N.check(N.lib().pfc_cuda_set_device(int(device_id)))


def cuda_synchronize() -> None:
    N.check(N.lib().pfc_cuda_synchronize())


def _info(i: N.DeviceInfo) -> DeviceInfo:
    return DeviceInfo(i.device_id, i.name.decode(), i.architecture.decode(), i.total_memory, i.free_memory,
                      i.compute_units, i.max_threads_per_block, i.warp_size)


def cuda_get_device_info(device_id: int = 0) -> DeviceInfo:
    i = N.DeviceInfo()
    N.check(N.lib().pfc_cuda_get_device_info(int(device_id), C.byref(i)))
    return _info(i)


# ---------------------------------------------------------------------------
# graph -> C ABI
# ---------------------------------------------------------------------------

class NativeGraph:
    """A pfc_graph holding the ancestors of `roots` (ids, types, ops, specs,
    edges, typed attributes, constant payloads)."""

    def __init__(self, graph: Graph, roots: Sequence[Node]):
        L = N.lib()
        h = C.c_void_p()
        N.check(L.pfc_graph_create(C.byref(h)))
        self.handle = h
        self._keep = []
        self._fin = weakref.finalize(self, L.pfc_graph_destroy, h)
        for n in graph.topological_order(roots):
            shape = (C.c_int64 * max(1, n.ndim()))(*n.shape())
            ins = (C.c_uint64 * max(1, len(n.inputs())))(*[i.id() for i in n.inputs()])
            N.check(L.pfc_graph_add_node(h, n.id(), int(n.type()), int(n.op_type()), int(n.dtype()), n.ndim(),
                                         shape, len(n.inputs()), ins))
            for key, (val, ct) in n.attrs().items():
                self._set_attr(n.id(), key, val, ct)
            if n.has_constant_data():
                # constants and parameters are immutable: keep them on the device;
                # an INPUT node's payload is runtime data (node.hpp:24), uploaded per call
                arr = n.constant_data()
                self._keep.append(arr)
                flags = 0 if n.type() == NodeType.INPUT else PFC_CONST_RESIDENT
                N.check(L.pfc_graph_set_constant(h, n.id(), arr.ctypes.data, arr.nbytes, flags, n._data_key))

    def _set_attr(self, nid: int, key: str, val, ct: int):
        L = N.lib()
        k = key.encode()
        if ct == A_INT:
            v, cnt = C.c_int32(int(val)), 1
        elif ct == A_INT64:
            v, cnt = C.c_int64(int(val)), 1
        elif ct == A_BOOL:
            v, cnt = C.c_uint8(1 if val else 0), 1
        elif ct == A_FLOAT:
            v, cnt = C.c_float(float(val)), 1
        elif ct == A_DOUBLE:
            v, cnt = C.c_double(float(val)), 1
        elif ct == A_INT64_VEC:
            v, cnt = (C.c_int64 * max(1, len(val)))(*[int(x) for x in val]), len(val)
        elif ct == A_INT_VEC:
            v, cnt = (C.c_int32 * max(1, len(val)))(*[int(x) for x in val]), len(val)
        elif ct == A_FLOAT_VEC:
            v, cnt = (C.c_float * max(1, len(val)))(*[float(x) for x in val]), len(val)
        else:
            raise TypeError(f"attribute {key}: unknown C type {ct}")
        N.check(L.pfc_graph_set_attr(self.handle, nid, k, ct, C.byref(v), cnt))


_native_lock = threading.Lock()


def native_graph(graph: Graph, output_ids: Sequence[int]) -> NativeGraph:
    """Build (or reuse) the native description of the subgraph for
    `output_ids`.  Descriptions of the graph's current version are kept per
    output set (up to 8), so callers that evaluate several subgraphs of one
    graph in turn, or from several threads, reuse theirs."""
    with _native_lock:
        cache = graph.__dict__.setdefault("_native_cache", {})
        key = (graph.version, tuple(output_ids))
        ng = cache.get(key)
        if ng is None:
            roots = []
            for i in output_ids:
                n = graph.node(i)
                if n is None:
                    raise KeyError(f"output id {i} is not in the graph")
                roots.append(n)
            ng = NativeGraph(graph, roots)
            for k in [k for k in cache if k[0] != graph.version]:
                del cache[k]
            while len(cache) >= 8:
                del cache[next(iter(cache))]
            cache[key] = ng
        return ng


# ---------------------------------------------------------------------------
# executors
# ---------------------------------------------------------------------------

class CudaExecutor:
    """B200 graph executor (rocm_executor.hpp:37-194 shape)."""

    @dataclass
    class Config:
        """rocm_executor.hpp:40-47 plus precision, CUDA graphs and fault injection."""
        device_id: int = 0
        enable_profiling: bool = False
        sync_after_launch: bool = False
        workspace_size_mb: int = 256
        precision: str = "tf32x3"
        use_cuda_graph: bool = True
        fail_after_n_allocations: int = 0

    def __init__(self, config: Optional["CudaExecutor.Config"] = None):
        self.config = config or CudaExecutor.Config()
        L = N.lib()
        c = N.ExecutorConfigC()
        L.pfc_executor_config_default(C.byref(c))
        c.device_id = self.config.device_id
        c.enable_profiling = int(self.config.enable_profiling)
        c.sync_after_launch = int(self.config.sync_after_launch)
        c.workspace_size_mb = self.config.workspace_size_mb
        c.precision = PRECISIONS[self.config.precision]
        c.use_cuda_graph = int(self.config.use_cuda_graph)
        c.fail_after_n_allocations = self.config.fail_after_n_allocations
        h = C.c_void_p()
        N.check(L.pfc_executor_create(C.byref(c), C.byref(h)))
        self.handle = h
        self._fin = weakref.finalize(self, L.pfc_executor_destroy, h)

    def close(self):
        self._fin()

    def execute(self, graph: Graph, output_ids: Sequence[int], out: Optional[Sequence[np.ndarray]] = None
                ) -> ExecutionResult:
        """ROCmExecutor::execute (rocm_executor.cpp:66-161): never raises; a
        failure comes back as success=False with the message.  `out`
        optionally supplies the host arrays to write (e.g. pinned memory)."""
        res = ExecutionResult()
        try:
            output_ids = [int(i) for i in output_ids]
            ng = native_graph(graph, output_ids)
            outs, ptrs, sizes = [], [], []
            for k, i in enumerate(output_ids):
                n = graph.node(i)
                if out is not None:
                    arr = out[k]
                    if list(arr.shape) != n.shape() or not arr.flags.c_contiguous:
                        raise ValueError(f"output buffer {k} does not match node {i}")
                else:
                    arr = np.empty(n.shape(), dtype=numpy_dtype(n.dtype()))
                outs.append(arr)
                ptrs.append(arr.ctypes.data)
                sizes.append(arr.nbytes)
            k = len(output_ids)
            ids = (C.c_uint64 * max(1, k))(*output_ids)
            pa = (C.c_void_p * max(1, k))(*ptrs)
            sa = (C.c_size_t * max(1, k))(*sizes)
            r = N.ExecutionResultC()
            rc = N.lib().pfc_executor_execute(self.handle, ng.handle, ids, k, pa, sa, C.byref(r))
            res.compile_time_ms, res.transfer_time_ms = r.compile_time_ms, r.transfer_time_ms
            res.compute_time_ms, res.total_time_ms = r.compute_time_ms, r.total_time_ms
            res.kernel_launches = r.kernel_launches
            res.h2d_bytes, res.d2h_bytes = r.h2d_bytes, r.d2h_bytes
            if rc != 0:
                res.success = False
                res.error_message = r.error_message.decode(errors="replace")
                return res
            res.success = True
            res.outputs = dict(zip(output_ids, outs))
        except Exception as e:  # noqa: BLE001 - the boundary reports, never raises
            res.success = False
            res.error_message = str(e)
        return res

    def execute_device(self, graph: Graph, inputs: Dict[int, int], output_ids: Sequence[int],
                       outputs: Sequence[int], stream: int = 0) -> ExecutionResult:
        """Device-resident execution: `inputs` maps leaf node id -> device
        pointer (dense row-major); `outputs` are device pointers for
        `output_ids`.  Issued on `stream` (0 = the executor's own stream) and
        not synchronised.  Raises on failure."""
        # a loop of calls with the same arguments (serving, the bench) reuses
        # the ctypes argument block of the previous call
        key = (id(graph), graph.version, tuple(inputs.items()), tuple(output_ids), tuple(outputs), stream)
        cached = self.__dict__.get("_dev_args")
        if cached is not None and cached[0] == key:
            args = cached[1]
        else:
            output_ids = [int(i) for i in output_ids]
            ng = native_graph(graph, output_ids)
            ins = list(inputs.items())
            k_in, k_out = len(ins), len(output_ids)
            args = (ng, (C.c_uint64 * max(1, k_in))(*[i for i, _ in ins]), k_in,
                    (C.c_void_p * max(1, k_in))(*[p for _, p in ins]), (C.c_uint64 * max(1, k_out))(*output_ids),
                    k_out, (C.c_void_p * max(1, k_out))(*outputs), C.c_void_p(stream or None))
            self._dev_args = (key, args)
        ng, in_ids, k_in, in_p, out_ids, k_out, out_p, sp = args
        r = N.ExecutionResultC()
        N.check(N.lib().pfc_executor_execute_device(self.handle, ng.handle, in_ids, k_in, in_p, out_ids, k_out,
                                                    out_p, sp, C.byref(r)))
        return ExecutionResult(True, "", r.compile_time_ms, 0.0, 0.0, r.total_time_ms, {}, r.kernel_launches,
                               r.h2d_bytes, r.d2h_bytes)

    def execute_streamed(self, chunk_graph: Graph, inputs: Dict[int, np.ndarray], output_ids: Sequence[int],
                         outputs: Sequence[np.ndarray]) -> ExecutionResult:
        """Host-buffer execution of a batch in chunks, with the copies of
        neighbouring chunks overlapping each chunk's compute.  `chunk_graph`
        computes one chunk of rows; `inputs` maps each of its leaf node ids to
        a host array holding all chunks back to back along dim 0, `outputs`
        are host arrays for `output_ids` laid out the same way.  Valid when
        rows are independent (as for batch sharding).  Pinned arrays (e.g.
        torch `pin_memory()` views) let the copies overlap.  Raises on
        failure."""
        output_ids = [int(i) for i in output_ids]
        ng = native_graph(chunk_graph, output_ids)
        items = list(inputs.items())
        n_chunks = None
        for nid, arr in items:
            per = chunk_graph.node(nid).numel() * 4
            if arr.nbytes % per or not arr.flags.c_contiguous:
                raise ValueError(f"input {nid}: {arr.nbytes} bytes is not a whole number of {per}-byte chunks")
            n = arr.nbytes // per
            if n_chunks not in (None, n):
                raise ValueError("inputs hold different numbers of chunks")
            n_chunks = n
        for oid, arr in zip(output_ids, outputs):
            per = chunk_graph.node(oid).numel() * 4
            if not arr.flags.c_contiguous or arr.nbytes != per * (n_chunks or 0):
                raise ValueError(f"output {oid}: expected {n_chunks} chunks of {per} bytes")
        k_in, k_out = len(items), len(output_ids)
        in_ids = (C.c_uint64 * max(1, k_in))(*[i for i, _ in items])
        in_p = (C.c_void_p * max(1, k_in))(*[a.ctypes.data for _, a in items])
        out_ids = (C.c_uint64 * max(1, k_out))(*output_ids)
        out_p = (C.c_void_p * max(1, k_out))(*[a.ctypes.data for a in outputs])
        r = N.ExecutionResultC()
        N.check(N.lib().pfc_executor_execute_streamed(self.handle, ng.handle, in_ids, k_in, in_p, out_ids, k_out,
                                                      out_p, int(n_chunks or 0), C.byref(r)))
        return ExecutionResult(True, "", r.compile_time_ms, r.transfer_time_ms, r.compute_time_ms, r.total_time_ms,
                               {}, r.kernel_launches, r.h2d_bytes, r.d2h_bytes)

    def get_device_info(self) -> DeviceInfo:
        i = N.DeviceInfo()
        N.check(N.lib().pfc_executor_get_device_info(self.handle, C.byref(i)))
        return _info(i)

    def get_memory_stats(self) -> MemoryStats:
        s = N.MemoryStatsC()
        N.check(N.lib().pfc_executor_get_memory_stats(self.handle, C.byref(s)))
        return MemoryStats(s.total_allocated, s.peak_allocated, s.total_allocations, s.total_deallocations,
                           s.cache_hits, s.cache_misses, s.resident_constant_bytes)

    def release_constants(self):
        N.check(N.lib().pfc_executor_release_constants(self.handle))

    def set_resident(self, node: Node, device_ptr: int):
        """Use device memory at `device_ptr` (caller-owned, same bytes as the
        node's payload) as the resident copy of `node`'s constant payload, e.g.
        a weight broadcast over NCCL.  It must stay valid and unchanged while
        this executor may run graphs holding the node."""
        if not node.has_constant_data():
            raise ValueError(f"node {node.id()} has no constant payload")
        N.check(N.lib().pfc_executor_set_resident(self.handle, node._data_key, device_ptr,
                                                  node.constant_data().nbytes))

    def describe_plan(self, graph: Graph, output_ids: Sequence[int]) -> str:
        output_ids = [int(i) for i in output_ids]
        ng = native_graph(graph, output_ids)
        buf = C.create_string_buffer(1 << 16)
        ids = (C.c_uint64 * max(1, len(output_ids)))(*output_ids)
        N.check(N.lib().pfc_executor_describe_plan(self.handle, ng.handle, ids, len(output_ids), buf, len(buf)))
        return buf.value.decode()

    def last_profile(self) -> List[tuple]:
        cap = 256
        names = (C.c_char * 64 * cap)()
        ms = (C.c_double * cap)()
        cnt = C.c_int(0)
        N.check(N.lib().pfc_executor_last_profile(self.handle, names, ms, cap, C.byref(cnt)))
        return [(bytes(names[i]).split(b"\0")[0].decode(), ms[i]) for i in range(min(cnt.value, cap))]


class Executor:
    """executor.cpp:171-194: dispatch on ExecutorConfig.backend."""

    def __init__(self, config: Optional[ExecutorConfig] = None):
        self.config = config or ExecutorConfig()
        self._cuda: Optional[CudaExecutor] = None

    def execute(self, graph: Graph, output_ids: Sequence[int]) -> ExecutionResult:
        b = self.config.backend
        if b == Backend.CUDA:
            return self._execute_cuda(graph, output_ids)
        if b in (Backend.SIMULATOR, Backend.HARDWARE):
            return ExecutionResult(False, "CSL execution requires Cerebras SDK (not available)")
        return ExecutionResult(False, "Backend.CPU is PyFlame's reference executor; this package evaluates "
                                      "graphs with Backend.CUDA only")

    def _execute_cuda(self, graph, output_ids):
        # executor.cpp:557-582 (execute_rocm) shape: availability gate, lazy executor
        if not cuda_is_available():
            return ExecutionResult(False, "CUDA backend requested but no compatible sm_100 GPU found.")
        if self._cuda is None:
            try:
                self._cuda = CudaExecutor(CudaExecutor.Config(
                    device_id=self.config.device_id, enable_profiling=self.config.enable_profiling,
                    precision=self.config.precision, use_cuda_graph=self.config.use_cuda_graph))
            except Exception as e:  # noqa: BLE001
                return ExecutionResult(False, str(e))
        return self._cuda.execute(graph, output_ids)

    @property
    def cuda_executor(self) -> Optional[CudaExecutor]:
        return self._cuda
