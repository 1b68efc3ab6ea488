"""Batch-sharded inference across GPUs: one process per GPU over
torch.distributed (NCCL on GPUs, gloo on CPU for tests).

Graph evaluation is independent per sample (no op in the supported graphs
reduces across the batch dimension; BatchNorm runs with running statistics),
so a batch splits into contiguous row shards, one per rank.  Weights are
broadcast once from rank 0; outputs may be gathered back to one rank.  No
other collective is involved.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Tuple

import numpy as np


def shard_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, end) of `n` rows for `rank` of `world`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def broadcast_weights(arrays: Dict[int, np.ndarray], device=None, src: int = 0):
    """Broadcast rank `src`'s arrays (node id -> array) to every rank; returns
    node id -> torch tensor on `device` (rank != src passes arrays of the right
    shape and dtype; their contents are ignored)."""
    import torch
    import torch.distributed as dist
    out = {}
    for nid in sorted(arrays):
        a = arrays[nid]
        t = torch.from_numpy(np.ascontiguousarray(a)).to(device) if dist.get_rank() == src else \
            torch.empty(a.shape, dtype=torch.float32, device=device)
        dist.broadcast(t, src=src)
        out[nid] = t
    return out


def gather_rows(local, world: int, dst: int = 0):
    """Gather per-rank row shards (possibly of different lengths) to `dst`,
    concatenated in rank order.  Returns the full tensor on `dst`, None
    elsewhere."""
    import torch
    import torch.distributed as dist
    n = torch.tensor([local.shape[0]], device=local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    rows = [int(s.item()) for s in sizes]
    m = max(rows)
    pad = torch.zeros((m,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    if dist.get_rank() != dst:
        return None
    return torch.cat([p[:r] for p, r in zip(parts, rows)], 0)


def shard_batch(x: np.ndarray, rank: int, world: int) -> np.ndarray:
    s, e = shard_range(x.shape[0], rank, world)
    return x[s:e]


def split_even(n: int, world: int) -> List[int]:
    return [shard_range(n, r, world)[1] - shard_range(n, r, world)[0] for r in range(world)]


def init(backend: str = "nccl", timeout_s: int = 120, device: Optional[int] = None):
    """Initialise the process group from the torchrun environment (short
    timeout so ranks waiting on a lost peer fail with an error)."""
    import datetime

    import torch.distributed as dist
    kw = {}
    if backend == "nccl" and device is not None:
        import torch
        kw["device_id"] = torch.device("cuda", device)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.get_rank(), dist.get_world_size()


# ---------------------------------------------------------------------------
# Failure handling for the multi-process path
# ---------------------------------------------------------------------------

class CollectiveError(RuntimeError):
    """A collective of the multi-GPU path failed or missed its deadline."""


class ShardResult:
    """Outcome of one rank's part of a sharded evaluation (never raised)."""

    def __init__(self, success: bool, error_message: str = "", output=None):
        self.success, self.error_message, self.output = success, error_message, output

    def __repr__(self):
        return f"ShardResult(success={self.success}, error_message={self.error_message!r})"


def run_sharded(evaluate, batch: np.ndarray, weights: Dict[int, np.ndarray], *, backend: str = "nccl",
                timeout_s: float = 60.0, device: Optional[int] = None, release=None, fail_at: str = "") -> ShardResult:
    """One rank of batch-sharded inference with failure handling: join the
    process group, receive rank 0's weights (broadcast once), evaluate this
    rank's rows, gather every rank's rows to rank 0.

    `evaluate(weights, shard) -> np.ndarray` runs the graph on this rank's
    device (a CudaExecutor call); `release()` frees the executor's device
    memory and runs on every failure.  Every collective is bounded by
    `timeout_s` (the process group's timeout): a rank that fails, exits or
    never arrives makes the others' next collective end with an error, the
    group is aborted (ProcessGroupNCCL::abort, i.e. ncclCommAbort, for NCCL)
    so no rank stays blocked, and each rank returns success=False with the
    reason.  `fail_at` injects a host-side failure on this rank at "init",
    "broadcast", "evaluate" or "gather" (test hook: nothing faults a GPU).
    Returns the gathered output on rank 0, this rank's rows elsewhere."""
    import torch
    import torch.distributed as dist

    joined = False

    def fail(msg: str) -> ShardResult:
        if release is not None:
            try:
                release()
            except Exception as e:  # noqa: BLE001 - report both failures
                msg += f"; release failed: {e}"
        if joined:
            try:
                from torch.distributed.distributed_c10d import _abort_process_group
                _abort_process_group()
            except Exception:  # noqa: BLE001 - already torn down
                try:
                    dist.destroy_process_group()
                except Exception:  # noqa: BLE001
                    pass
        return ShardResult(False, msg)

    try:
        if fail_at == "init":
            raise CollectiveError("injected failure before joining the process group")
        init(backend, timeout_s=int(max(1, timeout_s)), device=device)
        joined = True
        rank, world = dist.get_rank(), dist.get_world_size()
        if fail_at == "broadcast":
            raise CollectiveError("injected failure before the weight broadcast")
        dev = torch.device("cuda", device) if backend == "nccl" else None
        bw = broadcast_weights(weights, device=dev)
        local = {k: (v.cpu().numpy() if v.device.type != "cpu" else v.numpy()) for k, v in bw.items()}
        if fail_at == "evaluate":
            raise CollectiveError("injected failure while evaluating the shard")
        ys = evaluate(local, shard_batch(batch, rank, world))
        if fail_at == "gather":
            raise CollectiveError("injected failure before the output gather")
        t = torch.from_numpy(np.ascontiguousarray(ys))
        full = gather_rows(t.to(dev) if dev is not None else t, world)
        out = full.cpu().numpy() if full is not None else ys
        dist.barrier()
        dist.destroy_process_group()
        return ShardResult(True, "", out)
    except Exception as e:  # noqa: BLE001 - the boundary reports, never raises
        return fail(f"{type(e).__name__}: {e}")
