"""Backward graphs on the CUDA executor.

pyflame_b200.autograd builds, node for node, the backward graph PyFlame's
AutogradEngine builds (tests/test_frontend_ir.py pins that against PyFlame's
own C++ engine).  Here the forward+backward graph is evaluated by the CUDA
executor and compared with the oracle on the same graph, and with torch's
autograd in float64 as an independent check of the derivatives themselves.
"""
import numpy as np
import pytest
import torch

import pyflame_b200 as pf
from pyflame_b200 import autograd, nn
from tests.helpers import RTOL_GEMM_TF32X3, close, close_rows

pytestmark = pytest.mark.gpu

T64 = torch.float64


def _run(ex, oracle_mod, tensors):
    g = tensors[0].graph()
    ids = [t.node().id() for t in tensors]
    res = ex.execute(g, ids)
    assert res.success, res.error_message
    ref = oracle_mod.run(g, ids)
    return [res.outputs[i] for i in ids], [ref[i] for i in ids]


@pytest.mark.parametrize("batch,d_in,d_h,d_out", [(16, 32, 24, 5), (64, 784, 256, 10)])
def test_mlp_gradients(cuda_executor, oracle_mod, rng, batch, d_in, d_h, d_out):
    x = rng.random((batch, d_in), dtype=np.float32)
    t = rng.random((batch, d_out), dtype=np.float32)
    w1 = (rng.standard_normal((d_h, d_in)) / np.sqrt(d_in)).astype(np.float32)
    b1 = (rng.standard_normal(d_h) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((d_out, d_h)) / np.sqrt(d_h)).astype(np.float32)
    b2 = (rng.standard_normal(d_out) * 0.1).astype(np.float32)
    # keep every pre-activation at least 1e-3 from ReLU's kink, where fp32
    # rounding could flip the mask between implementations
    pre = x.astype(np.float64) @ w1.T.astype(np.float64)
    for _ in range(100):
        near = np.abs(pre + b1) < 1e-3
        if not near.any():
            break
        b1[near.any(0)] += np.float32(3e-3)
    assert not (np.abs(pre + b1) < 1e-3).any()
    with nn.deferred_init():
        l1, l2 = nn.Linear(d_in, d_h), nn.Linear(d_h, d_out)
    for m, w, b in ((l1, w1, b1), (l2, w2, b2)):
        m.set_parameter("weight", w)
        m.set_parameter("bias", b)
    xt = pf.tensor(x)
    loss = (pf.softmax(l2(pf.relu(l1(xt))), -1) * pf.tensor(t)).sum()
    wrt = [l1.p("weight"), l1.p("bias"), l2.p("weight"), l2.p("bias"), xt]
    grads = autograd.grad([loss], wrt)
    assert all(gr is not None for gr in grads)
    gpu, ref = _run(cuda_executor, oracle_mod, [loss] + grads)
    close(gpu[0], ref[0], rtol=1e-4, atol=0, what="loss")
    for name, a, b in zip(("dW1", "db1", "dW2", "db2", "dx"), gpu[1:], ref[1:]):
        close_rows(a.reshape(a.shape[0], -1), b.reshape(b.shape[0], -1), RTOL_GEMM_TF32X3, what=name)
    # independent check of the derivatives: torch autograd in float64
    tw = [torch.tensor(a, dtype=T64, requires_grad=True) for a in (w1, b1, w2, b2, x)]
    h = torch.relu(tw[4] @ tw[0].T + tw[1])
    lt = (torch.softmax(h @ tw[2].T + tw[3], -1) * torch.tensor(t, dtype=T64)).sum()
    lt.backward()
    for name, a, tt in zip(("dW1", "db1", "dW2", "db2", "dx"), gpu[1:], tw):
        want = tt.grad.numpy()
        close_rows(a.reshape(a.shape[0], -1), want.reshape(want.shape[0], -1), RTOL_GEMM_TF32X3, what=f"{name} vs torch")


def test_elementwise_chain_gradients(cuda_executor, oracle_mod, rng):
    """The backward graph of an elementwise chain with a broadcast bias, abs,
    division, sqrt, log, sin/cos and keepdim row reductions."""
    x = rng.standard_normal((64, 96)).astype(np.float32)
    y = rng.standard_normal((64, 96)).astype(np.float32)
    b = rng.standard_normal(96).astype(np.float32)
    xt, yt, bt = pf.tensor(x), pf.tensor(y), pf.tensor(b)
    a = xt * yt + bt
    h = pf.tanh(a) * pf.sigmoid(xt) - pf.exp(yt) / (pf.abs(xt) + 1.0)
    z = pf.sqrt(h * h + 1.0).sum(1, True)
    loss = (pf.log(z) + pf.sin(xt).sum(1, True) * pf.cos(yt).mean(1, True)).sum()
    grads = autograd.grad([loss], [xt, yt, bt])
    gpu, ref = _run(cuda_executor, oracle_mod, [loss] + grads)
    close(gpu[0], ref[0], rtol=1e-5, atol=0, what="loss")
    for name, g_, r_ in zip(("dx", "dy", "db"), gpu[1:], ref[1:]):
        close_rows(g_.reshape(1, -1) if g_.ndim == 1 else g_, r_.reshape(1, -1) if r_.ndim == 1 else r_, 1e-5,
                   what=name)
    tx, ty, tb = (torch.tensor(v, dtype=T64, requires_grad=True) for v in (x, y, b))
    ta = tx * ty + tb
    th = torch.tanh(ta) * torch.sigmoid(tx) - torch.exp(ty) / (torch.abs(tx) + 1.0)
    tz = torch.sqrt(th * th + 1.0).sum(1, keepdim=True)
    tl = (torch.log(tz) + torch.sin(tx).sum(1, keepdim=True) * torch.cos(ty).mean(1, keepdim=True)).sum()
    tl.backward()
    for name, g_, tt in zip(("dx", "dy", "db"), gpu[1:], (tx, ty, tb)):
        want = tt.grad.numpy()
        close_rows(g_.reshape(1, -1) if g_.ndim == 1 else g_, want.reshape(1, -1) if want.ndim == 1 else want,
                   1e-4, what=f"{name} vs torch")


def test_backward_records_leaf_gradients(cuda_executor, oracle_mod, rng):
    """backward() attaches each INPUT/PARAMETER leaf's gradient node, as
    PyFlame's engine sets the leaf's "grad" attribute."""
    g = pf.get_current_graph()
    x = pf.Tensor(g, g.create_input(pf.TensorSpec([8, 16])))
    x.node().set_constant_data(rng.standard_normal((8, 16)).astype(np.float32))
    w = pf.Tensor(g, g.create_parameter(pf.TensorSpec([16, 4])))
    w.node().set_constant_data(rng.standard_normal((16, 4)).astype(np.float32))
    loss = pf.tanh(pf.matmul(x, w)).sum()
    grads = autograd.backward(loss)
    assert set(grads) == {x.node().id(), w.node().id()}
    assert x.node().grad_node is grads[x.node().id()].node()
    gpu, ref = _run(cuda_executor, oracle_mod, [grads[w.node().id()], grads[x.node().id()]])
    for a, b_ in zip(gpu, ref):
        close_rows(a, b_, RTOL_GEMM_TF32X3)
