"""Device selection and whole-subgraph evaluation for the Tensor API.

Mirrors python/pyflame/__init__.py:451-600 (`Backend`, `set_device`,
`get_device`, `device_info`, `synchronize`) with 'cuda[:N]' in place of
'rocm[:N]'.  Unlike PyFlame's single-node CPU `materialize`
(tensor_impl.cpp:10-36), `eval` hands the tensor's whole subgraph to the CUDA
executor.
"""
from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np

from . import backend as B

_current = {"backend": "cuda", "device_id": 0, "precision": "tf32x3"}
_executors: Dict[tuple, B.CudaExecutor] = {}


def set_device(device: str) -> None:
    d = device.lower().strip()
    if d == "cpu":
        _current.update(backend="cpu", device_id=0)
        return
    if d.startswith("cuda"):
        if not B.cuda_is_available():
            raise RuntimeError("CUDA backend requested but not available: no sm_100 GPU is visible")
        dev = 0
        if ":" in d:
            try:
                dev = int(d.split(":")[1])
            except ValueError:
                raise ValueError(f"Invalid CUDA device specification: {device}")
            if dev >= B.cuda_device_count():
                raise ValueError(f"CUDA device {dev} requested but only {B.cuda_device_count()} devices available")
        B.cuda_set_device(dev)
        _current.update(backend="cuda", device_id=dev)
        return
    raise ValueError(f"Unknown device: {device}. Valid options: 'cpu', 'cuda', 'cuda:N'")


def get_device() -> str:
    return "cpu" if _current["backend"] == "cpu" else f"cuda:{_current['device_id']}"


def set_precision(p: str) -> None:
    if p not in B.PRECISIONS:
        raise ValueError(f"precision must be one of {list(B.PRECISIONS)}")
    _current["precision"] = p


def executor() -> B.CudaExecutor:
    key = (_current["device_id"], _current["precision"])
    ex = _executors.get(key)
    if ex is None:
        ex = B.CudaExecutor(B.CudaExecutor.Config(device_id=key[0], precision=key[1]))
        _executors[key] = ex
    return ex


def evaluate(tensors: Sequence) -> List[np.ndarray]:
    if _current["backend"] != "cuda":
        raise RuntimeError("pyflame_b200 evaluates graphs on CUDA devices; call set_device('cuda')")
    g = tensors[0].graph()
    ids = [t.node().id() for t in tensors]
    res = executor().execute(g, ids)
    if not res.success:
        raise RuntimeError(res.error_message)
    return [res.outputs[i] for i in ids]


def eval(*tensors):  # noqa: A001 - PyFlame's name
    """Evaluate several tensors with one executor call (shared subgraphs run once)."""
    todo = [t for t in tensors if not t.is_evaluated()]
    if todo:
        for t, a in zip(todo, evaluate(todo)):
            t._data = a
    return tensors[0] if len(tensors) == 1 else tensors


def device_info() -> dict:
    if _current["backend"] == "cpu":
        import os
        import platform
        return {"type": "cpu", "name": platform.processor() or "Unknown CPU", "cores": os.cpu_count() or 1}
    i = B.cuda_get_device_info(_current["device_id"])
    return {"type": "cuda", **i.__dict__}


def synchronize() -> None:
    if _current["backend"] == "cuda":
        B.cuda_synchronize()
