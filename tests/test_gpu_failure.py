"""The device failure path without a fault: a bounded wait that must give up.

pfk_check_bounded_wait runs a kernel whose mbarrier wait can never complete,
through the wait helper the GEMM and attention kernels use; it has to record
PFC_ERR_TIMEOUT in the error flag and return, and the context has to stay
usable for the next graph."""
import ctypes as C

import numpy as np
import pytest

import pyflame_b200 as pf
from tests.helpers import RTOL_GEMM_TF32X3, close_rows

pytestmark = pytest.mark.gpu

PFC_ERR_TIMEOUT = -8


def test_bounded_wait_gives_up_and_context_survives(native, oracle_mod, rng):
    import torch
    lib = native.lib()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.pfk_check_bounded_wait(C.c_void_p(err.data_ptr()), 50_000, None) == 0, lib.pfc_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == PFC_ERR_TIMEOUT
    # a flag that already holds an error is left as is
    err.fill_(-3)
    assert lib.pfk_check_bounded_wait(C.c_void_p(err.data_ptr()), 1_000, None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == -3
    # the context still runs graphs
    ex = pf.CudaExecutor()
    a = rng.standard_normal((96, 200)).astype(np.float32)
    b = rng.standard_normal((200, 72)).astype(np.float32)
    out = pf.matmul(pf.tensor(a), pf.tensor(b))
    res = ex.execute(out.graph(), [out.node().id()])
    assert res.success, res.error_message
    ref = oracle_mod.run(out.graph(), [out.node().id()])
    close_rows(res.outputs[out.node().id()], ref[out.node().id()], RTOL_GEMM_TF32X3)
    ex.close()


def test_bounded_wait_rejects_bad_arguments(native):
    lib = native.lib()
    assert lib.pfk_check_bounded_wait(None, 1000, None) != 0
