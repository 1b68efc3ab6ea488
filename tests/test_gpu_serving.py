"""InferenceEngine (PyFlame's serving API) on the CUDA executor: batches are
split over devices (one executor per device, one host thread each) and
gathered into one host result; checked against the oracle on the whole
batch.  With one GPU visible the split runs as two executors on that GPU."""
import numpy as np
import pytest

import pyflame_b200 as pf
from pyflame_b200 import nn
from pyflame_b200.serving import InferenceConfig, InferenceEngine
from tests.helpers import RTOL_GEMM_TF32X3, close_rows

pytestmark = pytest.mark.gpu


class MLP(nn.Module):
    def __init__(self, rng):
        super().__init__()
        with nn.deferred_init():
            self.l1 = self.register_module("l1", nn.Linear(784, 256))
            self.l2 = self.register_module("l2", nn.Linear(256, 10))
        self.set_parameter("l1.weight", (rng.standard_normal((256, 784)) / 28).astype(np.float32))
        self.set_parameter("l1.bias", (rng.standard_normal(256) * 0.1).astype(np.float32))
        self.set_parameter("l2.weight", (rng.standard_normal((10, 256)) / 16).astype(np.float32))

    def forward(self, x):
        return pf.softmax(self.l2(pf.relu(self.l1(x))), -1)


def _devices():
    n = pf.cuda_device_count()
    return [0, 1] if n >= 2 else [0, 0]


def _oracle(oracle_mod, model, x):
    pf_x = pf.tensor(x)
    out = model(pf_x)
    return oracle_mod.run(out.graph(), [out.node().id()])[out.node().id()]


def test_infer_split_over_devices(native, oracle_mod, rng):
    model = MLP(rng)
    eng = InferenceEngine(model, InferenceConfig(devices=_devices(), enable_caching=True))
    try:
        x = rng.random((67, 784), dtype=np.float32)  # uneven split: 34 + 33 rows
        eng.warmup(x, num_iterations=2)
        y = eng.infer(x)
        ref = _oracle(oracle_mod, model, x)
        close_rows(y.numpy(), ref, RTOL_GEMM_TF32X3, what="infer over two executors")
        y2, ms = eng.infer(x, return_time=True)
        assert ms == 0.0 and eng.stats.cache_hits == 1
        np.testing.assert_array_equal(y2.numpy(), y.numpy())
        assert eng.stats.total_inferences == 1 and eng.get_info()["warmed_up"]
    finally:
        eng.close()


def test_batch_infer_unbatches(native, oracle_mod, rng):
    model = MLP(rng)
    eng = InferenceEngine(model, InferenceConfig(devices=_devices(), max_batch_size=32))
    try:
        xs = [rng.random(784, dtype=np.float32) for _ in range(70)]  # batches of 32, 32, 6
        ys = eng.batch_infer(xs)
        assert len(ys) == 70
        ref = _oracle(oracle_mod, model, np.stack(xs))
        close_rows(np.stack([t.numpy() for t in ys]), ref, RTOL_GEMM_TF32X3, what="batch_infer")
        assert eng.stats.total_inferences == 3
    finally:
        eng.close()


def test_conv_model_through_engine(native, oracle_mod, rng):
    with nn.deferred_init():
        conv = nn.Conv2d(3, 16, 3, 1, 1)
    conv.set_parameter("weight", (rng.standard_normal((16, 3, 3, 3)) * 0.3).astype(np.float32))
    conv.set_parameter("bias", (rng.standard_normal(16) * 0.1).astype(np.float32))
    pool = nn.MaxPool2d(2, 2)

    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            self.register_module("conv", conv)

        def forward(self, x):
            return pool(pf.relu(conv(x)))

    net = Net()
    eng = InferenceEngine(net, InferenceConfig(devices=_devices()))
    try:
        x = rng.random((6, 3, 20, 20), dtype=np.float32)
        y = eng.infer(x).numpy()
        ref = _oracle(oracle_mod, net, x)
        close_rows(y.reshape(6, -1), ref.reshape(6, -1), RTOL_GEMM_TF32X3, what="conv net")
    finally:
        eng.close()
