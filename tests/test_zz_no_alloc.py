"""pfk_matmul_tf32x3_static (the matmul entry point that allocates nothing)
against the allocating pair pfk_split_tf32 + pfk_gemm on the same inputs,
through the C ABI, on two calls in a row (the second reuses the shared
scratch array with a different shape).  Named to be collected last; it also
passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

from tests.helpers import RTOL_GEMM_TF32X3

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(native):
    from pyflame_b200.backend import cuda_is_available
    if not cuda_is_available():
        pytest.fail("GPU test collected but no sm_100 GPU is visible")
    return native.lib()


def _allocating(lib, a, b, stream):
    """C = A @ B through the existing entry points with caller-owned buffers."""
    import torch
    M, K = a.shape
    N = b.shape[1]
    kpad = (K + 31) // 32 * 32
    a_hi = torch.empty((M, kpad), dtype=torch.float32, device="cuda")
    a_lo = torch.empty_like(a_hi)
    b_hi = torch.empty((N, kpad), dtype=torch.float32, device="cuda")
    b_lo = torch.empty_like(b_hi)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    c = torch.empty((M, N), dtype=torch.float32, device="cuda")
    assert lib.pfk_split_tf32(a.data_ptr(), 1, M, K, 0, K, 1, a_hi.data_ptr(), a_lo.data_ptr(), kpad, stream) == 0
    assert lib.pfk_split_tf32(b.data_ptr(), 1, N, K, 0, 1, N, b_hi.data_ptr(), b_lo.data_ptr(), kpad, stream) == 0
    assert lib.pfk_gemm(0, a_hi.data_ptr(), a_lo.data_ptr(), 0, b_hi.data_ptr(), b_lo.data_ptr(), 0, 1, M, N, K,
                        kpad, c.data_ptr(), 0, N, 1, None, err.data_ptr(), stream) == 0
    return c, err


def test_static_scratch_matmul_matches_allocating_path(lib):
    import torch
    stream = torch.cuda.Stream()
    sp = C.c_void_p(stream.cuda_stream)
    rng = np.random.default_rng(42)
    for M, N, K in ((300, 200, 100), (1024, 768, 1536)):  # two calls in a row, different shapes
        a_np = rng.standard_normal((M, K)).astype(np.float32)
        b_np = rng.standard_normal((K, N)).astype(np.float32)
        a = torch.from_numpy(a_np).cuda()
        b = torch.from_numpy(b_np).cuda()
        torch.cuda.synchronize()
        c = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        err = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        with torch.cuda.stream(stream):
            rc = lib.pfk_matmul_tf32x3_static(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, err.data_ptr(), sp)
            assert rc == 0, lib.pfc_last_error().decode()
            ref, ref_err = _allocating(lib, a, b, sp)
        stream.synchronize()
        assert int(err.item()) == 0 and int(ref_err.item()) == 0
        got, want = c.cpu().numpy(), ref.cpu().numpy()
        exact = a_np.astype(np.float64) @ b_np.astype(np.float64)
        scale = np.sqrt(np.mean(exact ** 2))
        assert np.all(np.isfinite(got))
        assert np.max(np.abs(got - want)) <= RTOL_GEMM_TF32X3 * scale, "differs from pfk_split_tf32 + pfk_gemm"
        assert np.max(np.abs(got - exact)) <= RTOL_GEMM_TF32X3 * scale, "differs from the fp64 product"


def test_static_scratch_matmul_rejects_oversize(lib):
    M = N = K = 2048  # needs 64 MiB + 256 B of scratch
    rc = lib.pfk_matmul_tf32x3_static(None, None, None, M, N, K, None, None)
    assert rc == -1  # PFC_ERR_INVALID_ARGUMENT
    assert b"maximum" in lib.pfc_last_error()
