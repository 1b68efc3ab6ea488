"""PyFlame's own Python module evaluating on the B200.

oracle/_ref/py/_pyflame_cpp.so is PyFlame's pybind11 module compiled from
PyFlame's sources (python/bindings.cpp, nn_bindings.cpp, pyflame_core),
unmodified, with the CUDA backend wired in as a PyFlame maintainer would: a
`_pyflame_cuda` module with cuda_* device functions and set_device("cuda"),
and TensorImpl::materialize routed to libpyflame_cuda.so while a CUDA
device is selected (oracle/pyflame_cuda_ext.cpp).  Models are built with
PyFlame's own Tensor API and nn modules; `.numpy()` evaluates the whole
graph on the GPU.  The expected values come from the same weights (read
back through PyFlame's CPU path) in float64 numpy/torch.
"""
import importlib.machinery
import importlib.util
from pathlib import Path

import numpy as np
import pytest

from tests.helpers import RTOL_GEMM_TF32X3, close_rows

EXT = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "py" / "_pyflame_cpp.so"
pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not EXT.exists(), reason="PyFlame's Python module not built (make -C oracle pyext)")]


def _load(name):
    loader = importlib.machinery.ExtensionFileLoader(name, str(EXT))
    spec = importlib.util.spec_from_file_location(name, str(EXT), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def pyflame():
    cuda = _load("_pyflame_cuda")  # first: it makes PyFlame's module importable (see pyflame_cuda_ext.cpp)
    pf = _load("_pyflame_cpp")
    yield pf, cuda
    cuda.set_device("cpu")


def test_device_functions(pyflame):
    pf, cuda = pyflame
    assert cuda.cuda_is_available() and cuda.cuda_device_count() >= 1
    cuda.set_device("cuda:0")
    assert cuda.get_device() == "cuda:0"
    info = cuda.cuda_get_device_info(0)
    assert info["architecture"].startswith("sm_10") and info["compute_units"] > 0
    with pytest.raises(ValueError):
        cuda.set_device("rocm")
    cuda.set_device("cpu")
    assert cuda.get_device() == "cpu"


def test_mlp_numpy_evaluates_on_the_gpu(pyflame):
    pf, cuda = pyflame
    cuda.set_device("cpu")
    rng = np.random.default_rng(42)
    xn = rng.random((64, 784), dtype=np.float32)
    x = pf.Tensor.from_numpy(xn)
    l1, l2 = pf.nn.Linear(784, 256), pf.nn.Linear(256, 10)
    # the weights as PyFlame initialised them, read back through its CPU path
    w1, b1, w2, b2 = (t.numpy().astype(np.float64) for t in (l1.weight, l1.bias, l2.weight, l2.bias))
    h = np.maximum(xn.astype(np.float64) @ w1.T + b1, 0.0)
    z = h @ w2.T + b2
    ref = np.exp(z - z.max(1, keepdims=True))
    ref /= ref.sum(1, keepdims=True)
    cuda.set_device("cuda")
    y = pf.softmax(l2(pf.relu(l1(x))), -1)
    before = cuda.routed_count()
    out = y.numpy()
    assert cuda.routed_count() == before + 1, "the output was not evaluated by the CUDA executor"
    close_rows(out, ref, RTOL_GEMM_TF32X3, what="PyFlame MLP on the GPU")


def test_conv_block_numpy_evaluates_on_the_gpu(pyflame):
    import torch
    import torch.nn.functional as F
    pf, cuda = pyflame
    cuda.set_device("cpu")
    rng = np.random.default_rng(43)
    xn = rng.random((4, 3, 32, 32), dtype=np.float32)
    x = pf.Tensor.from_numpy(xn)
    conv = pf.nn.Conv2d(3, 16, [3, 3], [1, 1], [1, 1])
    bn = pf.nn.BatchNorm2d(16)
    bn.eval()
    pool = pf.nn.MaxPool2d(2)
    w = conv.weight.numpy().astype(np.float64)
    cuda.set_device("cuda")
    y = pool(pf.relu(bn(conv(x))))
    out = y.numpy()
    # conv bias zeros; BatchNorm(eval) with its initial statistics (mean 0, var 1, gamma 1, beta 0)
    t = F.conv2d(torch.from_numpy(xn).double(), torch.from_numpy(w), padding=1) / np.sqrt(1.0 + 1e-5)
    ref = F.max_pool2d(torch.relu(t), 2).numpy()
    close_rows(out.reshape(4, -1), ref.reshape(4, -1), RTOL_GEMM_TF32X3, what="PyFlame conv block on the GPU")
