"""Batched inference on the CUDA executor, over one or several local GPUs.

Mirrors PyFlame's serving API (python/pyflame/serving/inference.py:15-383):
`InferenceConfig`, `InferenceStats`, `LRUCache` and `InferenceEngine` with
`warmup`, `infer`, `batch_infer`, `stats`, `reset_stats`, `clear_cache` and
`get_info`.  PyFlame's engine calls the model and returns the lazy result;
this one also evaluates it: the batch is split along dim 0 over the
configured devices (one CudaExecutor per device, each driven by its own host
thread), every device evaluates the same graph structure on its rows with
the weights resident on it after the first call, and each device's outputs
are copied into its rows of one host result.  Samples are independent in
every graph PyFlame's inference models build (BatchNorm runs with running
statistics), which is what makes the split exact.
"""
from __future__ import annotations

import threading
import time
from collections import OrderedDict
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Optional, Sequence

import numpy as np

from . import backend as B
from .distributed import shard_range
from .ir import TensorSpec
from .tensor import Tensor, get_current_graph


@dataclass
class InferenceConfig:
    """inference.py:15-33, plus the devices to split batches over and the
    contraction precision."""
    max_batch_size: int = 32
    enable_caching: bool = False
    cache_size: int = 1000
    warmup_iterations: int = 10
    timeout_ms: int = 30000
    num_threads: int = 1
    devices: Optional[List[int]] = None   # None: every visible GPU
    precision: str = "tf32x3"


@dataclass
class InferenceStats:
    """inference.py:36-83."""
    total_inferences: int = 0
    total_time_ms: float = 0.0
    cache_hits: int = 0
    cache_misses: int = 0

    @property
    def average_time_ms(self) -> float:
        return self.total_time_ms / self.total_inferences if self.total_inferences else 0.0

    @property
    def throughput(self) -> float:
        return self.total_inferences / (self.total_time_ms / 1000) if self.total_time_ms else 0.0

    @property
    def cache_hit_rate(self) -> float:
        total = self.cache_hits + self.cache_misses
        return self.cache_hits / total if total else 0.0

    def to_dict(self) -> Dict[str, Any]:
        return {"total_inferences": self.total_inferences, "total_time_ms": self.total_time_ms,
                "average_time_ms": self.average_time_ms, "throughput_per_second": self.throughput,
                "cache_hits": self.cache_hits, "cache_misses": self.cache_misses,
                "cache_hit_rate": self.cache_hit_rate}


class LRUCache:
    """inference.py:86-138: least-recently-used output cache."""

    def __init__(self, max_size: int = 1000):
        self.max_size = max_size
        self._d: "OrderedDict[int, Any]" = OrderedDict()
        self._lock = threading.Lock()

    def get(self, key: int) -> Optional[Any]:
        with self._lock:
            if key not in self._d:
                return None
            self._d.move_to_end(key)
            return self._d[key]

    def put(self, key: int, value: Any):
        with self._lock:
            self._d[key] = value
            self._d.move_to_end(key)
            while len(self._d) > self.max_size:
                self._d.popitem(last=False)

    def clear(self):
        with self._lock:
            self._d.clear()

    def __len__(self) -> int:
        return len(self._d)


class ShardedExecutor:
    """Evaluates a graph builder on a batch split over several local GPUs.

    `build(x) -> Tensor` maps an input Tensor of a given row count to the
    model's output; one graph is built per distinct shard shape and reused.
    Each device has its own CudaExecutor (weights become resident on it on
    first use); the shards run concurrently from one host thread per device,
    each writing its rows of the shared host output."""

    def __init__(self, build: Callable[[Tensor], Tensor], devices: Sequence[int], precision: str = "tf32x3",
                 graph=None):
        if not devices:
            raise ValueError("no devices to run on")
        self.build = build
        self.graph = graph  # the graph holding the model's weights (None: the current graph)
        self.devices = list(devices)
        self.executors = [B.CudaExecutor(B.CudaExecutor.Config(device_id=d, precision=precision)) for d in devices]
        self._graphs: Dict[tuple, tuple] = {}
        self._pool = ThreadPoolExecutor(max_workers=len(devices))
        self._lock = threading.Lock()

    def _graph_for(self, shape: tuple):
        """(input node, output tensor) of the model on an input of `shape`,
        built once per shape in the model's graph, so every shape shares the
        model's weight constants and each device uploads a weight once.  The
        input is an INPUT node bound to the caller's rows on every call."""
        with self._lock:
            ent = self._graphs.get(shape)
            if ent is None:
                g = self.graph or get_current_graph()
                x = Tensor(g, g.create_input(TensorSpec(list(shape))))
                out = self.build(x)
                ent = (x.node(), out)
                self._graphs[shape] = ent
            return ent

    def run(self, batch: np.ndarray) -> np.ndarray:
        batch = np.ascontiguousarray(batch, np.float32)
        n, k = batch.shape[0], len(self.devices)
        spans = [(i, s, e) for i, (s, e) in enumerate(shard_range(n, r, k) for r in range(k)) if e > s]
        ents = {e - s: self._graph_for((e - s,) + batch.shape[1:]) for _, s, e in spans}
        out = np.empty([n] + ents[spans[0][2] - spans[0][1]][1].shape[1:], np.float32)

        def one(i, s, e):
            node, res_t = ents[e - s]
            # host rows in, host rows out: the input is bound per call, the graph is not changed
            return self.executors[i].execute_streamed(res_t.graph(), {node.id(): batch[s:e]}, [res_t.node().id()],
                                                      [out[s:e]])

        futs = [self._pool.submit(one, i, s, e) for i, s, e in spans]
        errors = []
        for f in futs:
            try:
                f.result()
            except Exception as e:  # noqa: BLE001 - collect every device's failure
                errors.append(f"device {self.devices[futs.index(f)]}: {e}")
        if errors:
            raise RuntimeError("; ".join(errors))
        return out

    def close(self):
        self._pool.shutdown(wait=True)
        for ex in self.executors:
            ex.close()


class InferenceEngine:
    """inference.py:141-383 on the CUDA executor: `infer` evaluates the model
    on the batch (split over `config.devices`) and returns the result as an
    evaluated Tensor; `batch_infer` stacks inputs into batches of
    `max_batch_size` and unbatches the results."""

    def __init__(self, model, config: Optional[InferenceConfig] = None):
        self.model = model
        self.config = config or InferenceConfig()
        self._stats = InferenceStats()
        self._cache: Optional[LRUCache] = LRUCache(self.config.cache_size) if self.config.enable_caching else None
        self._lock = threading.Lock()
        self._warmed_up = False
        if hasattr(self.model, "eval"):
            self.model.eval()
        devices = self.config.devices
        if devices is None:
            devices = list(range(B.cuda_device_count()))
        params = self.model.parameters() if hasattr(self.model, "parameters") else []
        self._runner = ShardedExecutor(self._forward, devices, self.config.precision,
                                       graph=params[0].graph() if params else None)

    def _forward(self, x: Tensor) -> Tensor:
        return self.model(x)

    @staticmethod
    def _as_array(inputs) -> np.ndarray:
        if isinstance(inputs, Tensor):
            if not inputs.is_evaluated() and inputs.node().has_constant_data():
                return np.asarray(inputs.node().constant_data(), np.float32)
            return np.asarray(inputs.numpy(), np.float32)
        return np.asarray(inputs, np.float32)

    def warmup(self, example_input, num_iterations: Optional[int] = None):
        for _ in range(num_iterations or self.config.warmup_iterations):
            self._runner.run(self._as_array(example_input))
        self._warmed_up = True

    def infer(self, inputs, return_time: bool = False):
        arr = self._as_array(inputs)
        key = None
        if self._cache is not None:
            key = self._compute_cache_key(arr)
            cached = self._cache.get(key)
            if cached is not None:
                self._stats.cache_hits += 1
                return (cached, 0.0) if return_time else cached
            self._stats.cache_misses += 1
        t0 = time.perf_counter()
        out = self._runner.run(arr)
        ms = (time.perf_counter() - t0) * 1000
        with self._lock:
            self._stats.total_inferences += 1
            self._stats.total_time_ms += ms
        res = Tensor.from_data(out)
        res._data = out
        if self._cache is not None:
            self._cache.put(key, res)
        return (res, ms) if return_time else res

    def batch_infer(self, inputs: Sequence, batch_size: Optional[int] = None) -> List[Tensor]:
        bs = batch_size or self.config.max_batch_size
        results: List[Tensor] = []
        for i in range(0, len(inputs), bs):
            batch = np.stack([self._as_array(x) for x in inputs[i:i + bs]], 0)
            out = self.infer(batch)._data
            for j in range(out.shape[0]):
                t = Tensor.from_data(out[j])
                t._data = out[j]
                results.append(t)
        return results

    @staticmethod
    def _compute_cache_key(arr: np.ndarray) -> int:
        return hash((arr.shape, arr.tobytes()))

    @property
    def stats(self) -> InferenceStats:
        return self._stats

    def reset_stats(self):
        with self._lock:
            self._stats = InferenceStats()

    def clear_cache(self):
        if self._cache is not None:
            self._cache.clear()

    def get_info(self) -> Dict[str, Any]:
        return {"config": {"max_batch_size": self.config.max_batch_size, "enable_caching": self.config.enable_caching,
                           "cache_size": self.config.cache_size, "devices": self._runner.devices},
                "stats": self._stats.to_dict(), "warmed_up": self._warmed_up,
                "cache_entries": len(self._cache) if self._cache else 0}

    def close(self):
        self._runner.close()
