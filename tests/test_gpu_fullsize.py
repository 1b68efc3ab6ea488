"""The benchmark graphs at their full sizes, checked through a size-independent
property: samples are independent (no op reduces across the batch dimension;
BatchNorm runs in eval mode), so any sample of the full-batch GPU result must
equal the oracle's result for a graph holding just that sample.  The fused
graph is small enough for the oracle at full size and is compared whole."""
import numpy as np
import pytest

from pyflame_b200 import workloads
from tests.helpers import RTOL_GEMM_TF32X3, close, close_rows, close_sum

pytestmark = pytest.mark.gpu


def _gpu(ex, w):
    g = w.outputs[0].graph()
    ids = [t.node().id() for t in w.outputs]
    res = ex.execute(g, ids)
    assert res.success, res.error_message
    return [res.outputs[i] for i in ids]


def _oracle(oracle_mod, w):
    g = w.outputs[0].graph()
    ids = [t.node().id() for t in w.outputs]
    ref = oracle_mod.run(g, ids)
    return [ref[i] for i in ids]


def test_fused_full_size(cuda_executor, oracle_mod):
    w = workloads.fused(8192, 4096)
    gpu = _gpu(cuda_executor, w)
    ref = _oracle(oracle_mod, w)
    z = w.outputs[0].node().inputs()[0]
    zabs = np.abs(oracle_mod.run(w.outputs[0].graph(), [z.id()])[z.id()]).sum(1)
    close_sum(gpu[0], ref[0], zabs, what="sum")
    close_sum(gpu[1], ref[1], zabs / 4096, what="mean")
    close(gpu[2], ref[2], rtol=1e-5, atol=1e-6, what="max")
    close_rows(gpu[3], ref[3], 1e-5, what="layernorm")


@pytest.mark.parametrize("name,key,full,pick", [
    ("mlp", "x", dict(batch=64), [0, 31, 63]),
    ("gemm_chain", "A", dict(rows=8192), [0, 1, 4095, 8191]),
    ("encoder", "x", dict(batch=32, seq=512), [31]),
    ("convstack", "x", dict(batch=256), [0, 255]),
])
def test_full_batch_rows_match_single_sample_oracle(cuda_executor, oracle_mod, name, key, full, pick):
    build = workloads.BUILDERS[name]
    w = build(**full)
    x = w.inputs[key].node().constant_data()
    (gpu,) = _gpu(cuda_executor, w)
    small = dict(full)
    small["batch" if "batch" in full else "rows"] = len(pick)
    ws = build(**small)
    ws.inputs[key].node().set_constant_data(np.ascontiguousarray(x[pick]))
    (ref,) = _oracle(oracle_mod, ws)
    g = ws.outputs[0].graph()
    oid = ws.outputs[0].node().id()
    ref64 = oracle_mod.run(g, [oid], "f64")[oid]
    got = gpu[pick].reshape(len(pick), -1)
    ref = ref.reshape(len(pick), -1)
    ref64 = ref64.reshape(len(pick), -1)
    # Long contractions (K = 16384) carry the fp32 reference's own rounding
    # (sequential fp32 sums): the GPU is held to 1e-4 of the exact (fp64)
    # result, and to 1e-4 plus the reference's own deviation from it.
    close_rows(got, ref64, RTOL_GEMM_TF32X3, what=f"{name} full batch vs fp64")
    own = np.abs(ref.astype(np.float64) - ref64)
    close(got, ref, rtol=RTOL_GEMM_TF32X3, atol=RTOL_GEMM_TF32X3 * np.sqrt(np.mean(ref64 ** 2, axis=1, keepdims=True)) + own,
          what=f"{name} full batch vs fp32 reference")
