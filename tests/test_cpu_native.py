"""CPU-only checks of the C ABI library: it loads without a GPU, exports every
entry point include/pyflame_cuda.h declares, compiles the plan and every
generated kernel for sm_100a without a device, and reports malformed graphs
through status codes (never by crashing)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import pyflame_b200 as pf
from pyflame_b200 import backend as B
from pyflame_b200 import workloads as W

HEADER = Path(__file__).resolve().parent.parent / "include" / "pyflame_cuda.h"


def declared_symbols():
    return sorted(set(re.findall(r"PFC_API\s+[\w\s\*]+?\b(pf[ck]_\w+)\s*\(", HEADER.read_text())))


def test_library_exports_every_declared_symbol(native):
    L = native.lib()
    syms = declared_symbols()
    assert len(syms) >= 30
    for s in syms:
        assert hasattr(L, s), f"{s} not exported"
    assert L.pfc_abi_version() == 1
    assert set(syms) == set(native.SIGNATURES), "ctypes signature table out of sync with the header"


def compile_check(outs, precision=0):
    g = outs[0].graph()
    ids = [t.node().id() for t in outs]
    ng = B.native_graph(g, ids)
    buf = C.create_string_buffer(1 << 20)
    rc = B.N.lib().pfc_compile_check(ng.handle, (C.c_uint64 * len(ids))(*ids), len(ids), precision, buf, len(buf))
    return rc, (buf.value.decode() if rc == 0 else B.N.lib().pfc_last_error().decode())


@pytest.mark.parametrize("name,kw", [("mlp", {}), ("fused", dict(rows=64, cols=4096)),
                                     ("gemm_chain", dict(rows=64, d=512, h=1024)),
                                     ("encoder", dict(batch=2, seq=16, d=64, heads=4, ff=256)),
                                     ("convstack", dict(batch=2, hw=64))])
@pytest.mark.parametrize("precision", [0, 1])
def test_workload_plans_compile(native, name, kw, precision):
    w = W.BUILDERS[name](**kw)
    rc, desc = compile_check(w.outputs, precision)
    assert rc == 0, desc
    if name == "fused":
        assert desc.count("row kernel") == 1 and "fused elementwise" not in desc
    if name == "mlp":
        # Linear, ReLU, Linear and softmax of a 64-sample batch: one launch
        assert "small mlp [64x256x784 -> 10] +softmax" in desc and "row kernel" not in desc, desc
    if name == "convstack":
        assert "fold batch_norm" in desc and desc.count("conv gemm") == 3


def test_graph_errors_are_reported(native):
    L = native.lib()
    g = C.c_void_p()
    assert L.pfc_graph_create(C.byref(g)) == 0
    shape = (C.c_int64 * 1)(4)
    # a cycle: 1 <- 2 <- 1
    assert L.pfc_graph_add_node(g, 1, 3, 200, 0, 1, shape, 1, (C.c_uint64 * 1)(2)) == 0
    assert L.pfc_graph_add_node(g, 2, 3, 200, 0, 1, shape, 1, (C.c_uint64 * 1)(1)) == 0
    buf = C.create_string_buffer(4096)
    rc = L.pfc_compile_check(g, (C.c_uint64 * 1)(1), 1, 0, buf, len(buf))
    assert rc == -6 and b"cycle" in L.pfc_last_error()
    # duplicate ids, bad payload size, unknown output
    assert L.pfc_graph_add_node(g, 1, 0, 900, 0, 1, shape, 0, None) == -1
    assert L.pfc_graph_add_node(g, 3, 0, 900, 0, 1, shape, 0, None) == 0
    data = np.zeros(3, np.float32)
    assert L.pfc_graph_set_constant(g, 3, data.ctypes.data, data.nbytes, 0, 0) == -1
    L.pfc_graph_destroy(g)
    g2 = C.c_void_p()
    assert L.pfc_graph_create(C.byref(g2)) == 0
    assert L.pfc_graph_add_node(g2, 3, 0, 900, 0, 1, shape, 0, None) == 0
    assert L.pfc_compile_check(g2, (C.c_uint64 * 1)(99), 1, 0, buf, len(buf)) == -1
    L.pfc_graph_destroy(g2)


def test_unsupported_op_is_reported(native):
    a = pf.tensor(np.ones((4, 4), np.float32))
    g = a.graph()
    bad = g.create_op(pf.OpType.CONV3D, [a.node()], pf.TensorSpec([4, 4]))
    rc, msg = compile_check([pf.Tensor(g, bad)])
    assert rc == -2 and "Unsupported" in msg


def test_no_device_is_a_clean_error(native):
    if B.cuda_is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(Exception) as e:
        B.CudaExecutor()
    assert "no CUDA device" in str(e.value) or "no device" in str(e.value)
    r = pf.Executor(pf.ExecutorConfig(backend=pf.Backend.CUDA)).execute(pf.tensor([1.0]).graph(), [0])
    assert not r.success and "CUDA" in r.error_message
    r = pf.Executor(pf.ExecutorConfig(backend=pf.Backend.CPU)).execute(pf.tensor([1.0]).graph(), [0])
    assert not r.success
