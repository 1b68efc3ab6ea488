"""Parity on the exact path bench.py times, at the benchmark layer widths.

A serving host (and every rank after the NCCL weight broadcast) keeps the
weights in its own device buffers and registers them with
CudaExecutor.set_resident; batches then arrive either as device pointers
(execute_device) or from pinned host memory in chunks whose copies overlap
compute (execute_streamed).  These tests run gemm_chain, the encoder block,
the conv stack and the MLP that way, on reduced batches with the real layer
widths, and compare with the oracle on the same batch.  They also check the
copy accounting the bench relies on: registered weights are never uploaded,
and a repeated host-buffer call copies only its inputs and outputs.
"""
import numpy as np
import pytest

from pyflame_b200 import workloads
from tests.helpers import RTOL_GEMM_TF32X3, close_rows

pytestmark = pytest.mark.gpu

# (workload, reduced batch at the benchmark widths, batch input, chunks of the streamed run)
CASES = [
    ("gemm_chain", dict(rows=128), "A", 2),
    ("encoder", dict(batch=2, seq=512), "x", 2),
    ("convstack", dict(batch=2), "x", 2),
    ("mlp", dict(batch=64), "x", 4),
]
BATCH_KEY = {"gemm_chain": "rows", "encoder": "batch", "convstack": "batch", "mlp": "batch"}

_ref_cache = {}


def _oracle(oracle_mod, name, kw):
    """Oracle output of the workload at this batch (computed once per case)."""
    key = (name, tuple(sorted(kw.items())))
    if key not in _ref_cache:
        w = workloads.BUILDERS[name](**kw)
        _ref_cache[key] = oracle_mod.run(w.graph(), w.output_ids())[w.output_ids()[0]]
    return _ref_cache[key]


def _register(ex, w, dev):
    """set_resident for every weight of `w`, from the device copies in `dev`
    (keyed by weight order, so a second graph of the same workload reuses
    the same buffers, as each rank's executor does after the broadcast)."""
    for k, nid in enumerate(sorted(w.weights())):
        ex.set_resident(w.graph().node(nid), dev[k].data_ptr())


@pytest.mark.parametrize("name,kw,key,chunks", CASES, ids=[c[0] for c in CASES])
def test_resident_weights_device_and_streamed(native, oracle_mod, name, kw, key, chunks):
    import torch
    from pyflame_b200.backend import CudaExecutor

    ref = _oracle(oracle_mod, name, kw)
    w = workloads.BUILDERS[name](**kw)
    g, ids = w.graph(), w.output_ids()
    weights = w.weights()
    assert weights, "the workload has weights to keep resident"
    dev = [torch.from_numpy(np.ascontiguousarray(weights[nid])).cuda() for nid in sorted(weights)]
    x = w.inputs[key].node().constant_data()
    xd = torch.from_numpy(x.copy()).cuda()
    torch.cuda.synchronize()
    ex = CudaExecutor(CudaExecutor.Config())
    try:
        _register(ex, w, dev)
        # device-resident: the call the bench's `value` times
        out = torch.full(tuple(w.outputs[0].shape), float("nan"), device="cuda")
        r1 = ex.execute_device(g, {w.inputs[key].node().id(): xd.data_ptr()}, ids, [out.data_ptr()])
        r2 = ex.execute_device(g, {w.inputs[key].node().id(): xd.data_ptr()}, ids, [out.data_ptr()])
        torch.cuda.synchronize()
        # registered weights are never copied from the host: at most the
        # splat-value table (a few floats) on the first call, nothing after
        assert r1.h2d_bytes < 4096, r1.h2d_bytes
        assert r2.h2d_bytes == 0 and r2.d2h_bytes == 0, (r2.h2d_bytes, r2.d2h_bytes)
        # the second call skips the once-only operand preparation of the weights
        assert 0 < r2.kernel_launches <= r1.kernel_launches
        got = out.cpu().numpy()
        close_rows(got.reshape(-1, got.shape[-1]), ref.reshape(-1, ref.shape[-1]), RTOL_GEMM_TF32X3,
                   what=f"{name} execute_device with resident weights")

        # streamed host buffers: the call the bench's `e2e` times
        bk = BATCH_KEY[name]
        cw = workloads.BUILDERS[name](**{**kw, bk: kw[bk] // chunks})
        _register(ex, cw, dev)
        xin = torch.from_numpy(x.copy()).pin_memory()
        outs = torch.full(tuple(w.outputs[0].shape), float("nan")).pin_memory()
        for _ in range(2):  # the second call replays the captured plan
            rs = ex.execute_streamed(cw.graph(), {cw.inputs[key].node().id(): xin.numpy()}, cw.output_ids(),
                                     [outs.numpy()])
        assert rs.h2d_bytes == x.nbytes, (rs.h2d_bytes, x.nbytes)
        assert rs.d2h_bytes == outs.numpy().nbytes
        got = outs.numpy()
        close_rows(got.reshape(-1, got.shape[-1]), ref.reshape(-1, ref.shape[-1]), RTOL_GEMM_TF32X3,
                   what=f"{name} execute_streamed ({chunks} chunks) with resident weights")
    finally:
        ex.close()


@pytest.mark.parametrize("name,kw,key,chunks", CASES[:1] + CASES[2:3], ids=["gemm_chain", "convstack"])
def test_repeat_host_call_uploads_inputs_only(native, oracle_mod, name, kw, key, chunks):
    """Without set_resident the first execute uploads the weights once; every
    later call copies only the batch input in and the output out."""
    from pyflame_b200.backend import CudaExecutor

    ref = _oracle(oracle_mod, name, kw)
    w = workloads.BUILDERS[name](**kw)
    g, ids = w.graph(), w.output_ids()
    wbytes = sum(a.nbytes for a in w.weights().values())
    x = w.inputs[key].node().constant_data()
    ex = CudaExecutor(CudaExecutor.Config())
    try:
        r1 = ex.execute(g, ids)
        r2 = ex.execute(g, ids)
        r3 = ex.execute(g, ids)
        assert r1.success and r2.success and r3.success, (r1.error_message, r2.error_message, r3.error_message)
        assert r1.h2d_bytes >= wbytes + x.nbytes, (r1.h2d_bytes, wbytes)
        assert r2.h2d_bytes == x.nbytes and r3.h2d_bytes == x.nbytes, (r2.h2d_bytes, r3.h2d_bytes, x.nbytes)
        assert r3.d2h_bytes == ref.nbytes
        assert ex.get_memory_stats().resident_constant_bytes >= wbytes
        for r in (r1, r3):
            got = r.outputs[ids[0]]
            close_rows(got.reshape(-1, got.shape[-1]), ref.reshape(-1, ref.shape[-1]), RTOL_GEMM_TF32X3,
                       what=f"{name} repeated execute")
    finally:
        ex.close()


def test_resident_buffer_replaced_in_place(native, oracle_mod):
    """A registered weight buffer is read on every call, not copied: new
    values written into it (e.g. a fresh broadcast) show up in the next
    call's result once the prepared operands are rebuilt by re-registering."""
    import torch
    from pyflame_b200.backend import CudaExecutor

    w = workloads.gemm_chain(rows=64, d=512, h=1024)
    g, ids = w.graph(), w.output_ids()
    weights = w.weights()
    dev = [torch.from_numpy(np.ascontiguousarray(weights[nid])).cuda() for nid in sorted(weights)]
    xd = torch.from_numpy(w.inputs["A"].node().constant_data().copy()).cuda()
    out = torch.empty(tuple(w.outputs[0].shape), device="cuda")
    ex = CudaExecutor(CudaExecutor.Config())
    try:
        _register(ex, w, dev)
        ex.execute_device(g, {w.inputs["A"].node().id(): xd.data_ptr()}, ids, [out.data_ptr()])
        torch.cuda.synchronize()
        first = out.cpu().numpy()
        ref = oracle_mod.run(g, ids)[ids[0]]
        close_rows(first, ref, RTOL_GEMM_TF32X3, what="before")
        # scale the second layer's weight by 2 on the device, re-register it
        nid2 = max(n for n in weights if weights[n].ndim == 2)
        k2 = sorted(weights).index(nid2)
        dev[k2].mul_(2.0)
        torch.cuda.synchronize()
        _register(ex, w, dev)
        ex.execute_device(g, {w.inputs["A"].node().id(): xd.data_ptr()}, ids, [out.data_ptr()])
        torch.cuda.synchronize()
        g.node(nid2).set_constant_data(np.ascontiguousarray(weights[nid2] * np.float32(2.0)))
        ref2 = oracle_mod.run(g, ids)[ids[0]]
        close_rows(out.cpu().numpy(), ref2, RTOL_GEMM_TF32X3, what="after re-registering")
    finally:
        ex.close()
