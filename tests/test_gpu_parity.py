"""CUDA executor vs the oracle on the same seeded graphs.

Every case builds a graph with the PyFlame-mirroring front end, evaluates it
through libpyflame_cuda.so (CudaExecutor.execute -> pfc_executor_execute)
and compares with the CPU restatement (oracle/oracle.cpp), which itself is
pinned to PyFlame's own executor and kernels by tests/test_oracle_pinned.py.
"""
import numpy as np
import pytest

import pyflame_b200 as pf
from pyflame_b200 import nn
from tests.helpers import (RTOL_GEMM_BF16, RTOL_GEMM_TF32X3, bitexact, close, close_rows, close_sum)

pytestmark = pytest.mark.gpu


def run(ex, outs, oracle_mod, precision="f32"):
    g = outs[0].graph()
    ids = [t.node().id() for t in outs]
    res = ex.execute(g, ids)
    assert res.success, res.error_message
    assert res.kernel_launches >= 0
    ref = oracle_mod.run(g, ids, precision)
    return [res.outputs[i] for i in ids], [ref[i] for i in ids]


# ---- known-answer tests from PyFlame's tests/cpp/test_operations.cpp ---------------

def test_kat_operations(cuda_executor, oracle_mod):
    x = pf.tensor([-2.0, -1.0, 0.0, 1.0, 2.0])
    s = pf.tensor([1.0, 2.0, 3.0, 4.0])
    outs = [pf.relu(x), pf.sigmoid(pf.tensor([0.0])), pf.exp(pf.tensor([0.0, 1.0])),
            pf.log(pf.tensor([1.0, float(np.exp(np.float32(1.0)))])), pf.sqrt(pf.tensor([1.0, 4.0, 9.0])),
            pf.abs(pf.tensor([-3.0, -1.0, 0.0, 1.0, 3.0])), s.sum(), s.mean(), pf.tensor([1.0, 5.0, 3.0, 2.0]).max(),
            pf.tensor([5.0, 1.0, 3.0, 2.0]).min(), (pf.ones([10]) + pf.full([10], 2.0)) * 3.0 - 1.0,
            pf.matmul(pf.tensor([[1.0, 2.0], [3.0, 4.0]]), pf.tensor([[5.0, 6.0], [7.0, 8.0]])),
            pf.matmul(pf.tensor([[1.0, 2.0, 3.0]]), pf.tensor([[1.0], [2.0], [3.0]])),
            pf.arange(1, 11).sum(), pf.arange(1, 11).mean()]
    gpu, _ = run(cuda_executor, outs, oracle_mod)
    expect = [[0, 0, 0, 1, 2], [0.5], [1, np.e], [0, 1], [1, 2, 3], [3, 1, 0, 1, 3], 10.0, 2.5, 5.0, 1.0, [8.0] * 10,
              [[19, 22], [43, 50]], [[14]], 55.0, 5.5]
    for g_, e in zip(gpu, expect):
        np.testing.assert_allclose(g_, np.asarray(e, np.float32), rtol=1e-5, atol=1e-5)


# ---- elementwise --------------------------------------------------------------------

SPECIAL = np.array([0.0, -0.0, 1.0, -1.0, 1e-30, -1e-30, 1e30, -1e30, np.inf, -np.inf, np.nan, 88.0, -88.0,
                    20.0, -20.0], np.float32)


@pytest.mark.parametrize("fn", ["neg", "abs", "sqrt", "exp", "log", "sin", "cos", "tanh", "relu", "sigmoid",
                                "gelu", "silu"])
def test_unary(cuda_executor, oracle_mod, rng, fn):
    data = np.concatenate([rng.standard_normal(1021).astype(np.float32) * 4, SPECIAL])
    x = pf.tensor(data)
    f = {"neg": lambda t: -t}.get(fn, getattr(pf, fn, None))
    (g,), (r,) = run(cuda_executor, [f(x)], oracle_mod)
    close(g, r, rtol=2e-6 if fn in ("relu", "neg", "abs") else 1e-5, atol=1e-6, what=fn)
    if fn in ("neg", "abs", "relu"):
        bitexact(g, r)


FLT_MIN = float(np.finfo(np.float32).tiny)

# Inputs per function over which the output spans its whole normal range.
# Sigmoid/SiLU stop short of -88.72, where the reference's exp(-x) overflows
# (its semantics there are checked separately below).
_REL_DOMAIN = {
    "sigmoid": (-88.70, 40.0), "silu": (-88.70, 40.0), "exp": (-87.3, 88.7), "tanh": (-12.0, 12.0),
    "log": (1e-37, 3e38), "sqrt": (1e-37, 3e38), "sin": (-200.0, 200.0), "cos": (-200.0, 200.0),
}
_F64 = {"sigmoid": lambda x: 1.0 / (1.0 + np.exp(-x)), "silu": lambda x: x / (1.0 + np.exp(-x)), "exp": np.exp,
        "tanh": np.tanh, "log": np.log, "sqrt": np.sqrt, "sin": np.sin, "cos": np.cos}


@pytest.mark.parametrize("fn", sorted(_REL_DOMAIN))
def test_unary_relative_over_normal_range(cuda_executor, oracle_mod, rng, fn):
    """1e-5 relative, with no absolute floor, against the exact (fp64) value
    and against the fp32 reference, for every output at or above FLT_MIN;
    outputs below FLT_MIN within FLT_MIN.  Covers the tails where a fast
    exp loses accuracy (sigmoid and SiLU for x in [-88.7, -20])."""
    lo, hi = _REL_DOMAIN[fn]
    if lo > 0:  # log-spaced positive inputs
        data = np.exp(rng.uniform(np.log(lo), np.log(hi), 8192))
    else:
        data = np.concatenate([np.linspace(lo, hi, 8192), rng.uniform(lo, hi, 4096)])
    if fn in ("sigmoid", "silu"):
        data = np.concatenate([data, rng.uniform(-88.7, -20.0, 4096), np.linspace(-88.7, -87.0, 1024)])
    if fn == "tanh":
        data = np.concatenate([data, np.exp(rng.uniform(np.log(1e-30), 0.0, 1024))])
    data = data.astype(np.float32)
    f = getattr(pf, fn)
    (g,), (r,) = run(cuda_executor, [f(pf.tensor(data))], oracle_mod)
    exact = _F64[fn](data.astype(np.float64))
    for what, want in (("fp64", exact), ("reference fp32", r.astype(np.float64))):
        got = g.astype(np.float64)
        normal = np.abs(exact) >= FLT_MIN
        rel = np.abs(got[normal] - want[normal]) / np.abs(want[normal])
        assert rel.max() <= 1e-5, f"{fn} vs {what}: max rel {rel.max():.3g} at x={data[normal][rel.argmax()]!r}"
        assert np.all(np.abs(got[~normal] - want[~normal]) <= FLT_MIN), f"{fn} vs {what}: sub-FLT_MIN outputs"


def test_sigmoid_silu_past_exp_overflow(cuda_executor, oracle_mod):
    """Below x = -88.72 the reference's exp(-x) is +inf, so sigmoid is +0 and
    SiLU is -0 (x / inf); the device gives the same values, bit for bit.
    Between -88.72 and -87.34 SiLU's outputs are still normal numbers."""
    x = np.concatenate([np.linspace(-200.0, -88.75, 512), [-1e30, -np.inf]]).astype(np.float32)
    (gs, gl), (rs, rl) = run(cuda_executor, [pf.sigmoid(pf.tensor(x)), pf.silu(pf.tensor(x))], oracle_mod)
    assert np.all(np.abs(gs) <= FLT_MIN) and np.all(np.abs(rs) <= FLT_MIN)
    bitexact(gl, rl)
    near = np.linspace(-88.7, -87.34, 256).astype(np.float32)
    (g,), (r,) = run(cuda_executor, [pf.silu(pf.tensor(near))], oracle_mod)
    assert np.all(np.abs(r) >= FLT_MIN)
    np.testing.assert_allclose(g, r, rtol=1e-5, atol=0)


@pytest.mark.parametrize("shapes", [((37, 129), (37, 129)), ((64, 256), (256,)), ((64, 256), (64, 1)),
                                    ((2, 5, 7, 3), (1, 5, 1, 1)), ((3, 1, 8), (4, 1)), ((1000,), ())])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_binary_broadcast(cuda_executor, oracle_mod, rng, shapes, op):
    a = pf.tensor(rng.standard_normal(shapes[0]).astype(np.float32))
    b = pf.tensor(rng.standard_normal(shapes[1]).astype(np.float32))
    out = {"add": a + b, "sub": a - b, "mul": a * b, "div": a / b}[op]
    (g,), (r,) = run(cuda_executor, [out], oracle_mod)
    bitexact(g, r)  # IEEE +,-,*,/ are correctly rounded on both sides


def test_div_by_zero_semantics(cuda_executor, oracle_mod):
    # executor.cpp:322-340: 0/0 -> NaN, x/0 -> +-inf by the dividend's sign (also for -0 divisors)
    a = pf.tensor([0.0, 1.0, -1.0, 2.0, -2.0, 0.0, 3.0])
    b = pf.tensor([0.0, 0.0, 0.0, -0.0, -0.0, 5.0, 2.0])
    (g,), (r,) = run(cuda_executor, [a / b], oracle_mod)
    bitexact(g, r)
    assert np.isnan(g[0]) and g[1] == np.inf and g[2] == -np.inf and g[3] == np.inf and g[4] == -np.inf


def test_comparisons_bitexact(cuda_executor, oracle_mod, rng):
    a = pf.tensor(np.round(rng.standard_normal((33, 65)) * 2).astype(np.float32))
    b = pf.tensor(np.round(rng.standard_normal((33, 65)) * 2).astype(np.float32))
    outs = [a == b, a != b, a < b, a <= b, a > b, a >= b, pf.maximum(a, b), pf.minimum(a, b),
            pf.clamp(a, -1.0, 1.5)]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    for g, r in zip(gpu, ref):
        bitexact(g, r)


def test_pow(cuda_executor, oracle_mod, rng):
    a = pf.tensor(np.abs(rng.standard_normal(500)).astype(np.float32) + 0.1)
    (g,), (r,) = run(cuda_executor, [pf.pow(a, 2.5)], oracle_mod)
    close(g, r, rtol=1e-5)


# ---- reductions, softmax, LayerNorm -----------------------------------------------

@pytest.mark.parametrize("shape,dim", [((8, 4096), 1), ((37, 1000), -1), ((5, 3), 1), ((7, 4097), 1),
                                       ((130, 77), 0), ((6, 33, 10), 1), ((4, 5, 6), 2), ((1, 1), 1),
                                       ((3000,), 0), ((64, 10), -1)])
@pytest.mark.parametrize("kind", ["sum", "mean", "max", "min"])
def test_reductions(cuda_executor, oracle_mod, rng, shape, dim, kind):
    data = rng.standard_normal(shape).astype(np.float32)
    x = pf.tensor(data)
    out = getattr(x, kind)(dim)
    (g,), (r,) = run(cuda_executor, [out], oracle_mod)
    if kind in ("max", "min"):
        bitexact(g, r)
    else:
        terms = np.abs(data).sum(axis=dim)
        if kind == "mean":
            terms = terms / data.shape[dim]
        close_sum(g, r, terms, what=f"{kind}{shape}")


@pytest.mark.parametrize("kind", ["sum", "mean", "max", "min", "prod"])
def test_full_reduction(cuda_executor, oracle_mod, rng, kind):
    data = rng.standard_normal((1000, 777)).astype(np.float32)
    if kind == "prod":
        data = (1.0 + data[:3, :7] * 1e-2).astype(np.float32)
    x = pf.tensor(data)
    (g,), (r,) = run(cuda_executor, [getattr(x, kind)()], oracle_mod)
    assert g.shape == ()
    if kind in ("max", "min"):
        bitexact(g, r)
    else:
        close_sum(g, r, np.abs(data).sum() / (data.size if kind == "mean" else 1) if kind != "prod"
                  else np.abs(r) * 10, what=kind)


def test_keepdim(cuda_executor, oracle_mod, rng):
    data = rng.standard_normal((6, 40)).astype(np.float32)
    x = pf.tensor(data)
    outs = [x.sum(1, keepdim=True), x.max(0, keepdim=True), x.mean(keepdim=True)]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    assert gpu[0].shape == (6, 1) and gpu[1].shape == (1, 40) and gpu[2].shape == (1, 1)
    close_sum(gpu[0], ref[0], np.abs(data).sum(1, keepdims=True))
    bitexact(gpu[1], ref[1])


@pytest.mark.parametrize("shape,dim", [((64, 10), -1), ((8, 512), -1), ((3, 7, 5), 1), ((4, 2, 33), 2),
                                       ((2, 4097), 1)])
@pytest.mark.parametrize("log", [False, True])
def test_softmax(cuda_executor, oracle_mod, rng, shape, dim, log):
    x = pf.tensor((rng.standard_normal(shape) * 3).astype(np.float32))
    out = (pf.log_softmax if log else pf.softmax)(x, dim)
    (g,), (r,) = run(cuda_executor, [out], oracle_mod)
    close(g, r, rtol=1e-5, atol=1e-6 * (10 if log else 1), what="softmax")


@pytest.mark.parametrize("shape,ns,affine", [((16, 768), [768], True), ((37, 100), [100], False),
                                             ((4, 6, 10), [6, 10], True), ((3, 4096), [4096], True)])
def test_layer_norm(cuda_executor, oracle_mod, rng, shape, ns, affine):
    x = pf.tensor(rng.standard_normal(shape).astype(np.float32) * 2 + 0.5)
    ln = nn.LayerNorm(ns, eps=1e-5, elementwise_affine=affine)
    if affine:
        ln.set_parameter("weight", rng.standard_normal(ns).astype(np.float32))
        ln.set_parameter("bias", rng.standard_normal(ns).astype(np.float32))
    (g,), (r,) = run(cuda_executor, [ln(x)], oracle_mod)
    close_rows(g, r, 1e-5, what="layernorm")


@pytest.mark.parametrize("rows,cols", [(256, 4096), (37, 1000), (5, 3)])
def test_fused_graph(cuda_executor, oracle_mod, rows, cols):
    from pyflame_b200 import workloads
    w = workloads.fused(rows, cols)
    gpu, ref = run(cuda_executor, w.outputs, oracle_mod)
    plan = cuda_executor.describe_plan(w.outputs[0].graph(), [t.node().id() for t in w.outputs])
    assert plan.count("row kernel") == 1 and "fused elementwise" not in plan, plan
    x = w.inputs["x"].node().constant_data()
    y = w.inputs["y"].node().constant_data()
    z = ref[3]  # unused except for shape
    zz = oracle_mod.run(w.outputs[0].graph(), [w.outputs[0].node().inputs()[0].id()])
    zabs = np.abs(list(zz.values())[0]).sum(1)
    close_sum(gpu[0], ref[0], zabs, what="sum")
    close_sum(gpu[1], ref[1], zabs / cols, what="mean")
    close(gpu[2], ref[2], rtol=1e-5, atol=1e-6, what="max")  # selection of z, which carries ulp-level exp differences
    close_rows(gpu[3], ref[3], 1e-5, what="layernorm")
    assert z.shape == (rows, cols) and x.shape == y.shape


# ---- shape ops -------------------------------------------------------------------------

def test_views_bitexact(cuda_executor, oracle_mod, rng):
    a = pf.tensor(rng.standard_normal((4, 6, 8)).astype(np.float32))
    b = pf.tensor(rng.standard_normal((4, 6, 8)).astype(np.float32))
    outs = [a.transpose(0, 2), a.reshape([24, 8]).t(), a.slice(1, 2, 5), a.transpose(1, 2).reshape([4, 48]),
            a.unsqueeze(1).squeeze(1), a[2], pf.cat([a, b], 1), pf.stack([a, b], 0), (a + b).transpose(-1, -2),
            a.slice(2, -3, 100)]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    for g, r in zip(gpu, ref):
        bitexact(g, r)


# ---- contractions ------------------------------------------------------------------------

@pytest.mark.parametrize("m,k,n", [(64, 784, 256), (5, 7, 3), (130, 200, 70), (256, 512, 384), (1, 1, 1),
                                   (128, 4096, 128), (300, 33, 257)])
def test_matmul_2d(cuda_executor, oracle_mod, rng, m, k, n):
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    (g,), (r,) = run(cuda_executor, [pf.matmul(pf.tensor(a), pf.tensor(b))], oracle_mod)
    r64 = a.astype(np.float64) @ b.astype(np.float64)
    close_rows(g, r64, RTOL_GEMM_TF32X3, what="matmul vs fp64")
    close_rows(r, r64, RTOL_GEMM_TF32X3, what="oracle vs fp64")


@pytest.mark.parametrize("a_shape,b_shape", [((2, 3, 17, 40), (2, 3, 40, 9)), ((4, 33, 64), (64, 48)),
                                             ((3, 16, 8), (1, 8, 5)), ((40,), (40, 7)), ((7, 40), (40,)),
                                             ((40,), (40,)), ((2, 1, 8, 16), (3, 16, 4))])
def test_matmul_batched_and_1d(cuda_executor, oracle_mod, rng, a_shape, b_shape):
    a = rng.standard_normal(a_shape).astype(np.float32)
    b = rng.standard_normal(b_shape).astype(np.float32)
    (g,), (r,) = run(cuda_executor, [pf.matmul(pf.tensor(a), pf.tensor(b))], oracle_mod)
    r64 = np.matmul(a.astype(np.float64), b.astype(np.float64))
    assert g.shape == r64.shape
    close_rows(g, r64.reshape(g.shape) if g.ndim else r64, RTOL_GEMM_TF32X3) if g.ndim else \
        close(g, r64, rtol=RTOL_GEMM_TF32X3, atol=1e-4 * np.abs(a).sum())


def test_linear_relu_softmax_mlp(cuda_executor, oracle_mod):
    from pyflame_b200 import workloads
    w = workloads.mlp(64)
    (g,), (r,) = run(cuda_executor, w.outputs, oracle_mod)
    close(g, r, rtol=1e-4, atol=1e-6, what="mlp softmax")
    plan = cuda_executor.describe_plan(w.outputs[0].graph(), [w.outputs[0].node().id()])
    # Linear, ReLU, Linear and softmax in one launch on clusters of 8 CTAs
    assert "small mlp [64x256x784 -> 10] +softmax (clusters)" in plan and "row kernel" not in plan, plan
    assert "arrival counter" not in plan, plan


@pytest.mark.parametrize("m,k,n1,n2,act,soft", [(64, 784, 256, 10, "relu", "softmax"), (1, 7, 5, 3, "tanh", "log"),
                                                (256, 130, 96, 70, "gelu", "softmax"), (33, 64, 48, 17, "sigmoid", ""),
                                                (200, 64, 1000, 0, "", ""), (5, 12, 9, 0, "silu", ""),
                                                (17, 301, 40, 9, "relu", "softmax"),
                                                (256, 300, 200, 20, "gelu", "log"),
                                                (48, 128, 300, 130, "relu", "softmax")])
def test_small_batch_linear_layers(cuda_executor, oracle_mod, rng, m, k, n1, n2, act, soft):
    """Small batches of Linear layers run on the CUDA cores: one layer alone,
    or Linear -> activation -> Linear (-> softmax / log-softmax) as one
    launch; short rows (lane per column) and long rows (lanes split K), float4
    and scalar loads (K not a multiple of 4), layer 2 from shared memory or,
    when h and the weight do not fit there, from L2; softmax rows past 32;
    single rows.  Two layers with K a multiple of 4 run on clusters of 8 CTAs
    (a partial last row block, hidden units not a multiple of 32, rows of
    130 outputs); the others on the single-launch kernel with its last-CTA
    layer 2."""
    x = pf.tensor(rng.standard_normal((m, k)).astype(np.float32))
    with nn.deferred_init():
        l1 = nn.Linear(k, n1)
        l2 = nn.Linear(n1, max(n2, 1))
    l1.set_parameter("weight", (rng.standard_normal((n1, k)) / np.sqrt(k)).astype(np.float32))
    l1.set_parameter("bias", rng.standard_normal(n1).astype(np.float32))
    l2.set_parameter("weight", (rng.standard_normal((max(n2, 1), n1)) / np.sqrt(n1)).astype(np.float32))
    fn = {"relu": pf.relu, "tanh": pf.tanh, "gelu": pf.gelu, "sigmoid": pf.sigmoid, "silu": pf.silu,
          "": lambda t: t}[act]
    y = fn(l1(x))
    if n2:
        y = l2(y)
        if soft:
            y = (pf.softmax if soft == "softmax" else pf.log_softmax)(y, -1)
    plan = cuda_executor.describe_plan(y.graph(), [y.node().id()])
    assert ("small mlp" if n2 else "small gemm") in plan and "row kernel" not in plan, plan
    assert ("(clusters)" in plan) == (n2 > 0 and k % 4 == 0), plan
    (g,), (r,) = run(cuda_executor, [y], oracle_mod)
    close_rows(g, r, RTOL_GEMM_TF32X3, what="small batch layers")
    # scaled product without a bias
    z = pf.matmul(x, l1.p("weight").transpose(0, 1)) * 0.125
    (g,), (r,) = run(cuda_executor, [z], oracle_mod)
    close_rows(g, r, RTOL_GEMM_TF32X3, what="scaled small gemm")


def test_gemm_epilogues(cuda_executor, oracle_mod, rng):
    x = pf.tensor(rng.standard_normal((96, 160)).astype(np.float32))
    res = pf.tensor(rng.standard_normal((96, 72)).astype(np.float32))
    lin = nn.Linear(160, 72)
    lin.set_parameter("bias", rng.standard_normal(72).astype(np.float32))
    outs = [pf.gelu(lin(x)) + res, pf.matmul(x, lin.p("weight").transpose(0, 1)) * 0.125, pf.sigmoid(lin(x)),
            pf.tanh(lin(x)), pf.silu(lin(x))]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    for g, r in zip(gpu, ref):
        close_rows(g, r, RTOL_GEMM_TF32X3)


@pytest.mark.parametrize("m,n,k", [(1664, 1536, 2048), (1000, 1408, 1024)])
def test_gemm_split_last_wave(cuda_executor, oracle_mod, rng, m, n, k):
    """A partial last wave of long-K tiles is split along K over the idle
    CTAs (13 x 12 = 156 tiles on 148 SMs: 8 tiles in 4 parts; 8 x 11 = 88
    tiles fill one wave and stay whole), with a bias and GELU epilogue.  Two
    calls in a row: the parts' arrival counters must be back at zero."""
    x = rng.standard_normal((m, k)).astype(np.float32)
    lin = nn.Linear(k, n)
    lin.set_parameter("weight", (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float32))
    lin.set_parameter("bias", rng.standard_normal(n).astype(np.float32))
    out = pf.gelu(lin(pf.tensor(x)))
    for _ in range(2):
        (g,), (r,) = run(cuda_executor, [out], oracle_mod)
        close_rows(g, r, RTOL_GEMM_TF32X3, what="split last wave")


def test_gemm_bf16_mode(oracle_mod, rng, native):
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision="bf16"))
    a = rng.standard_normal((200, 300)).astype(np.float32)
    b = rng.standard_normal((300, 150)).astype(np.float32)
    out = pf.matmul(pf.tensor(a), pf.tensor(b))
    (g,), _ = run(ex, [out], oracle_mod)
    r64 = a.astype(np.float64) @ b.astype(np.float64)
    close_rows(g, r64, RTOL_GEMM_BF16, what="bf16 matmul")
    ex.close()


def test_conv2d_bf16_mode(oracle_mod, rng, native):
    """bf16 operands through the halo-staged 3x3 (64-channel blocks), the
    TMA-window 7x7 / 2 (few channels) and TMA boxes (64 channels per k-block)
    with 128- and 64-column tiles."""
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision="bf16"))
    outs = []
    for c, o, k, s, p, hw in [(64, 64, 3, 1, 1, (14, 18)), (3, 16, 7, 2, 3, (40, 40)), (64, 128, 3, 1, 1, (16, 40)),
                              (64, 64, 3, 1, 1, (12, 36)), (64, 192, 3, 1, 1, (10, 33))]:
        x = rng.random((2, c) + hw).astype(np.float32)
        conv = nn.Conv2d(c, o, k, s, p)
        conv.set_parameter("weight", (rng.standard_normal((o, c, k, k)) / np.sqrt(c * k * k)).astype(np.float32))
        conv.set_parameter("bias", np.zeros(o, np.float32))
        outs.append(conv(pf.tensor(x)))
    gpu, ref = run(ex, outs, oracle_mod)
    for g, r in zip(gpu, ref):
        close_rows(g.reshape(g.shape[0] * g.shape[1], -1), r.reshape(r.shape[0] * r.shape[1], -1), RTOL_GEMM_BF16,
                   what="bf16 conv")
    ex.close()


# ---- convolution and pooling ---------------------------------------------------------------

@pytest.mark.parametrize("cfg", [dict(n=2, c=3, h=17, w=15, o=8, k=3, s=1, p=1),
                                 dict(n=2, c=3, h=32, w=32, o=16, k=7, s=2, p=3),
                                 dict(n=1, c=5, h=9, w=11, o=4, k=2, s=3, p=0),
                                 # TMA-fed A (output width >= 32): 32-channel boxes, partial tiles, dilation
                                 dict(n=2, c=32, h=37, w=45, o=64, k=3, s=1, p=2, d=2),
                                 dict(n=1, c=64, h=33, w=70, o=96, k=3, s=1, p=1),
                                 # TMA-fed windows of a padded input: few channels, stride 2, row dilation
                                 dict(n=2, c=3, h=70, w=83, o=16, k=5, s=2, p=2),
                                 dict(n=2, c=4, h=40, w=36, o=8, k=3, s=1, p=1, d=(2, 1)),
                                 # halo-staged (stride 1, whole 32-channel blocks, halo <= 256 rows):
                                 # 3x3; dilation with a partial column tile; 1x1 over three channel
                                 # blocks and two column tiles; 5x5
                                 dict(n=3, c=64, h=20, w=30, o=64, k=3, s=1, p=1),
                                 dict(n=2, c=32, h=25, w=21, o=48, k=3, s=1, p=2, d=2),
                                 dict(n=2, c=96, h=9, w=13, o=80, k=1, s=1, p=0),
                                 dict(n=2, c=32, h=12, w=14, o=64, k=5, s=1, p=2),
                                 # TMA boxes with 128-column tiles: 128 channels; 192 (a partial tile)
                                 dict(n=2, c=64, h=20, w=40, o=128, k=3, s=1, p=1),
                                 dict(n=1, c=32, h=18, w=37, o=192, k=3, s=1, p=1)])
def test_conv2d(cuda_executor, oracle_mod, rng, cfg):
    x = rng.random((cfg["n"], cfg["c"], cfg["h"], cfg["w"])).astype(np.float32)
    conv = nn.Conv2d(cfg["c"], cfg["o"], cfg["k"], cfg["s"], cfg["p"], cfg.get("d", 1))
    conv.set_parameter("weight", rng.standard_normal((cfg["o"], cfg["c"], cfg["k"], cfg["k"])).astype(np.float32))
    conv.set_parameter("bias", rng.standard_normal(cfg["o"]).astype(np.float32))
    (g,), (r,) = run(cuda_executor, [conv(pf.tensor(x))], oracle_mod)
    close_rows(g.reshape(g.shape[0] * g.shape[1], -1), r.reshape(r.shape[0] * r.shape[1], -1), RTOL_GEMM_TF32X3)


def test_conv_bn_relu_pool_stack(cuda_executor, oracle_mod, rng):
    x = pf.tensor(rng.random((2, 3, 40, 40)).astype(np.float32))
    conv = nn.Conv2d(3, 16, 7, 2, 3)
    bn = nn.BatchNorm2d(16)
    bn.eval()
    params = {}
    for name, lo, hi in [("weight", 0.5, 1.5), ("bias", -0.5, 0.5), ("running_mean", -0.5, 0.5),
                         ("running_var", 0.5, 2.0)]:
        params[name] = rng.uniform(lo, hi, 16).astype(np.float32)
        bn.set_parameter(name, params[name])
    pool = nn.MaxPool2d(3, 2)
    c = conv(x)
    out = pool(pf.relu(bn(c)))
    gap = nn.AdaptiveAvgPool2d(1)(out)
    avg = nn.AvgPool2d(2)(out)
    gpu, ref = run(cuda_executor, [out, gap, avg, c], oracle_mod)
    # The folded BatchNorm can cancel most of a channel's conv value, so the
    # error bound follows the conv output's scale times the channel's BN scale
    # (the size of the terms accumulated), not the small value left after it.
    bn_scale = np.abs(params["weight"] / np.sqrt(params["running_var"].astype(np.float64) + 1e-5))
    conv_rms = np.sqrt(np.mean(ref[3].astype(np.float64) ** 2, axis=(2, 3)))  # [N, C]
    term_scale = (conv_rms * bn_scale[None, :]).reshape(-1, 1)
    for g, r in zip(gpu[:3], ref[:3]):
        g2, r2 = g.reshape(-1, g.shape[-1] * g.shape[-2]), r.reshape(-1, r.shape[-1] * r.shape[-2])
        close(g2, r2, rtol=RTOL_GEMM_TF32X3, atol=RTOL_GEMM_TF32X3 * term_scale)
    close_rows(gpu[3].reshape(-1, gpu[3].shape[-1] * gpu[3].shape[-2]),
               ref[3].reshape(-1, ref[3].shape[-1] * ref[3].shape[-2]), RTOL_GEMM_TF32X3)


@pytest.mark.parametrize("precision", ["tf32x3", "bf16"])
@pytest.mark.parametrize("n,h,w,pad", [(2, 64, 70, 0), (2, 64, 70, 1), (1, 224, 224, 0), (1, 224, 224, 1),
                                       (3, 150, 290, 0), (2, 151, 131, 1)])
def test_conv_bn_relu_maxpool_fused(oracle_mod, rng, native, precision, n, h, w, pad):
    """Conv2d(3 -> 64, 7x7 / 2) -> BatchNorm -> ReLU -> MaxPool2d(3, 2, pad)
    with the pool in the convolution's epilogue: strips of 1-3 column tiles,
    odd and even conv heights, runs of tiles that start inside a strip (the
    carried row recomputed), and the pooled map read both as an output and as
    the next convolution's operand.  Checked against the oracle and against
    the same graph evaluated without the fusion (the conv output also an
    output), which may differ only by the epilogue's rounding."""
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision=precision))
    x = pf.tensor(rng.random((n, 3, h, w)).astype(np.float32))
    conv = nn.Conv2d(3, 64, 7, 2, 3)
    conv.set_parameter("weight", (rng.standard_normal((64, 3, 7, 7)) * np.sqrt(2 / 147)).astype(np.float32))
    bn = nn.BatchNorm2d(64)
    bn.eval()
    params = {}
    for name, lo, hi in [("weight", 0.5, 1.5), ("bias", -0.3, 0.3), ("running_mean", -0.3, 0.3),
                         ("running_var", 0.5, 2.0)]:
        params[name] = rng.uniform(lo, hi, 64).astype(np.float32)
        bn.set_parameter(name, params[name])
    c = conv(x)
    r = pf.relu(bn(c))
    pooled = nn.MaxPool2d(3, 2, pad)(r)
    conv2 = nn.Conv2d(64, 64, 3, 1, 1)
    conv2.set_parameter("weight", (rng.standard_normal((64, 64, 3, 3)) * np.sqrt(2 / 576)).astype(np.float32))
    nxt = conv2(pooled)
    g = pooled.graph()
    plan = ex.describe_plan(g, [pooled.node().id(), nxt.node().id()])
    assert "+max_pool2d" in plan and "] max_pool2d" not in plan, plan
    assert "(row runs)" in plan and "(de-interleaved rows)" in plan, plan
    gpu, ref = run(ex, [pooled, nxt], oracle_mod)
    # unfused: the ReLU output is an output too, so the pool runs on its own
    plan2 = ex.describe_plan(g, [pooled.node().id(), r.node().id()])
    assert "+max_pool2d" not in plan2, plan2
    res2 = ex.execute(g, [pooled.node().id(), r.node().id()])
    assert res2.success, res2.error_message
    unfused, conv_ref = res2.outputs[pooled.node().id()], oracle_mod.run(g, [c.node().id()])[c.node().id()]
    tol = RTOL_GEMM_TF32X3 if precision == "tf32x3" else RTOL_GEMM_BF16
    bn_scale = np.abs(params["weight"] / np.sqrt(params["running_var"].astype(np.float64) + 1e-5))
    conv_rms = np.sqrt(np.mean(conv_ref.astype(np.float64) ** 2, axis=(2, 3)))
    term = (conv_rms * bn_scale[None, :]).reshape(-1, 1)
    flat = lambda a: a.reshape(-1, a.shape[-1] * a.shape[-2])
    close(flat(gpu[0]), flat(ref[0]), rtol=tol, atol=tol * term, what="fused pool vs oracle")
    np.testing.assert_allclose(flat(gpu[0]), flat(unfused), rtol=1e-6, atol=1e-6 * term.max(),
                               err_msg="fused pool vs unfused")
    close_rows(flat(gpu[1]), flat(ref[1]), tol if precision == "tf32x3" else 4 * tol, what="conv after the pool")
    ex.close()


@pytest.mark.parametrize("precision", ["tf32x3", "bf16"])
@pytest.mark.parametrize("pad", [0, 1])
def test_conv_relu_maxpool_fused_windows(oracle_mod, rng, native, precision, pad):
    """A stride-1 5x5 convolution of 3 channels with ReLU and MaxPool2d(3, 2):
    the pool runs in the epilogue of the overlapping-window feed (64-column
    tiles, 31 pooled columns each), not the row-run feed of the stride-2
    stem."""
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision=precision))
    x = pf.tensor(rng.random((2, 3, 41, 75)).astype(np.float32))
    conv = nn.Conv2d(3, 64, 5, 1, 2)
    conv.set_parameter("weight", (rng.standard_normal((64, 3, 5, 5)) * np.sqrt(2 / 75)).astype(np.float32))
    conv.set_parameter("bias", rng.uniform(-0.2, 0.2, 64).astype(np.float32))
    c = conv(x)
    pooled = nn.MaxPool2d(3, 2, pad)(pf.relu(c))
    g = pooled.graph()
    plan = ex.describe_plan(g, [pooled.node().id()])
    assert "+max_pool2d" in plan and "(row runs)" not in plan, plan
    (gpu,), (ref,) = run(ex, [pooled], oracle_mod)
    conv_ref = oracle_mod.run(g, [c.node().id()])[c.node().id()].astype(np.float64)
    term = np.sqrt(np.mean(conv_ref ** 2, axis=(2, 3))).reshape(-1, 1) + 0.2
    tol = RTOL_GEMM_TF32X3 if precision == "tf32x3" else RTOL_GEMM_BF16
    flat = lambda a: a.reshape(-1, a.shape[-1] * a.shape[-2])
    close(flat(gpu), flat(ref), rtol=tol, atol=tol * term, what="windowed fused pool vs oracle")
    ex.close()


@pytest.mark.parametrize("precision", ["tf32x3", "bf16"])
@pytest.mark.parametrize("cin,cout,k,st,pd,n,h,w,act", [
    (64, 64, 3, 1, 1, 3, 55, 55, "relu"),    # the conv stack's last convolution: 64 x 2 boxes, 9 columns dropped
    (64, 128, 3, 1, 1, 2, 33, 40, "none"),   # 128-column tiles, an odd height, 24 columns dropped per tile
    (128, 64, 1, 1, 0, 2, 20, 32, "bnrelu"),  # 32 x 4 boxes
    (3, 64, 7, 2, 3, 2, 96, 100, "bnrelu"),  # windows over the padded input (the stem's feed)
])
def test_conv_global_avg_pool_fused(oracle_mod, rng, native, precision, cin, cout, k, st, pd, n, h, w, act):
    """Conv2d (+ bias or BatchNorm) (+ ReLU) -> AdaptiveAvgPool2d(1) with the
    pool's sums in the convolution's epilogue (one row of column sums per
    tile and TMEM lane quarter, added per image in slot order by the pool
    step): tiles with columns or rows outside the image, 64- and 128-column
    tiles, boxes and windows.  Checked against the oracle and against the
    unfused graph (the conv output also an output)."""
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision=precision))
    x = pf.tensor(rng.standard_normal((n, cin, h, w)).astype(np.float32))
    conv = nn.Conv2d(cin, cout, k, st, pd)
    conv.set_parameter("weight", (rng.standard_normal((cout, cin, k, k)) * np.sqrt(2 / (cin * k * k))).astype(np.float32))
    conv.set_parameter("bias", rng.uniform(-0.2, 0.2, cout).astype(np.float32))
    c = conv(x)
    scale = np.ones(cout)
    if act == "bnrelu":
        bn = nn.BatchNorm2d(cout)
        bn.eval()
        params = {}
        for name, lo, hi in [("weight", 0.5, 1.5), ("bias", -0.3, 0.3), ("running_mean", -0.3, 0.3),
                             ("running_var", 0.5, 2.0)]:
            params[name] = rng.uniform(lo, hi, cout).astype(np.float32)
            bn.set_parameter(name, params[name])
        r = pf.relu(bn(c))
        scale = np.abs(params["weight"] / np.sqrt(params["running_var"].astype(np.float64) + 1e-5))
    else:
        r = pf.relu(c) if act == "relu" else c
    gap = nn.AdaptiveAvgPool2d(1)(r)
    g = gap.graph()
    plan = ex.describe_plan(g, [gap.node().id()])
    assert "+average sums" in plan and "from the convolution's sums" in plan, plan
    (fused,), (ref,) = run(ex, [gap], oracle_mod)
    plan2 = ex.describe_plan(g, [gap.node().id(), r.node().id()])
    assert "+average sums" not in plan2, plan2
    res2 = ex.execute(g, [gap.node().id(), r.node().id()])
    assert res2.success, res2.error_message
    unfused = res2.outputs[gap.node().id()]
    conv_ref = oracle_mod.run(g, [c.node().id()])[c.node().id()].astype(np.float64)
    term = np.sqrt(np.mean(conv_ref ** 2, axis=(2, 3))) * scale[None, :] + 0.2
    tol = RTOL_GEMM_TF32X3 if precision == "tf32x3" else RTOL_GEMM_BF16
    assert fused.shape == (n, cout, 1, 1)
    close(fused.reshape(n, cout), ref.reshape(n, cout), rtol=tol, atol=tol * term, what="fused average vs oracle")
    close(unfused.reshape(n, cout), ref.reshape(n, cout), rtol=tol, atol=tol * term, what="unfused average vs oracle")
    close(fused.reshape(n, cout), unfused.reshape(n, cout), rtol=1e-5, atol=1e-5 * term, what="fused average vs unfused")
    ex.close()


def test_batchnorm_alone_and_pools(cuda_executor, oracle_mod, rng):
    x = pf.tensor(rng.standard_normal((3, 4, 9, 7)).astype(np.float32))
    bn = nn.BatchNorm2d(4)
    bn.set_parameter("running_var", rng.uniform(0.5, 2, 4).astype(np.float32))
    outs = [bn(x), nn.MaxPool2d(2, 2, 1)(x), nn.AvgPool2d(3, 2, 1)(x), nn.AdaptiveAvgPool2d((2, 3))(x)]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    close(gpu[0], ref[0], rtol=1e-5, atol=1e-6)
    bitexact(gpu[1], ref[1])
    close(gpu[2], ref[2], rtol=1e-6, atol=1e-7)
    close(gpu[3], ref[3], rtol=1e-6, atol=1e-7)


def test_pools_channels_last(cuda_executor, oracle_mod, rng):
    """Pools over a channels-last view (the layout conv outputs have), which
    takes the float4 channels-last kernel; adaptive 1x1 takes the global one."""
    data = rng.standard_normal((3, 11, 13, 8)).astype(np.float32)  # N, H, W, C
    data[0, 2, 3, 1] = np.nan
    x = pf.tensor(data).transpose(1, 3).transpose(2, 3)  # [N, C, H, W] view, channel stride 1
    outs = [nn.MaxPool2d(3, 2)(x), nn.MaxPool2d(2, 2, 1)(x), nn.AvgPool2d(3, 2, 1)(x), nn.AdaptiveAvgPool2d(1)(x)]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    bitexact(gpu[0], ref[0])
    bitexact(gpu[1], ref[1])
    close(gpu[2], ref[2], rtol=1e-6, atol=1e-7)
    close(gpu[3], ref[3], rtol=1e-5, atol=1e-6)


# ---- attention / encoder block ---------------------------------------------------------

def test_multihead_attention(cuda_executor, oracle_mod, rng):
    x = pf.tensor(rng.standard_normal((2, 9, 16)).astype(np.float32))
    mha = nn.MultiheadAttention(16, 2, batch_first=True)
    for name, p in list(mha.named_parameters()):
        mha.set_parameter(name, (rng.standard_normal(p.shape) * 0.3).astype(np.float32))
    (g,), (r,) = run(cuda_executor, [mha(x)], oracle_mod)
    close_rows(g, r, RTOL_GEMM_TF32X3, what="mha")


@pytest.mark.parametrize("b,h,m,l,d,scale", [(2, 3, 300, 200, 64, 0.125), (1, 2, 128, 512, 32, 1.0),
                                             (3, 1, 50, 70, 40, 4.0)])
def test_fused_attention(cuda_executor, oracle_mod, rng, b, h, m, l, d, scale):
    """softmax(scale * Q K^T) V as one fused step: partial query tiles and key
    blocks, a 32-wide head, and a peaked softmax (logits around +-75)."""
    q = pf.tensor(rng.standard_normal((b, h, m, d)).astype(np.float32))
    k = pf.tensor(rng.standard_normal((b, h, l, d)).astype(np.float32))
    v = pf.tensor(rng.standard_normal((b, h, l, d)).astype(np.float32))
    out = pf.matmul(pf.softmax(pf.matmul(q, k.transpose(-2, -1)) * scale, -1), v)
    assert "attention " in cuda_executor.describe_plan(out.graph(), [out.node().id()])
    (g,), (r,) = run(cuda_executor, [out], oracle_mod)
    close_rows(g.reshape(-1, d), r.reshape(-1, d), RTOL_GEMM_TF32X3, what="attention")


@pytest.mark.parametrize("b,h,m,l,d,scale", [(2, 3, 300, 200, 64, 0.125), (1, 2, 128, 512, 32, 1.0),
                                             (3, 1, 50, 70, 40, 4.0)])
def test_fused_attention_bf16(native, rng, b, h, m, l, d, scale):
    """The bf16 mode's fused attention (bf16 Q, K, V and P, fp32 softmax and
    accumulation), the same shapes as the tf32 test.  The reference is the
    attention of the bf16-rounded Q, K and V in float64: rounding the inputs
    alone moves a peaked softmax (scaled logits of spread 5-25 here) by a few
    per cent, which is the mode's contract, not the kernel's error; against
    it the kernel's own arithmetic (bf16 P, fp32 sums) is held to 1e-2."""
    def bf16(x):
        u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
        u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        return u.astype(np.uint32).view(np.float32)
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision="bf16"))
    qa, ka, va = (rng.standard_normal((b, h, n, d)).astype(np.float32) for n in (m, l, l))
    q, k, v = pf.tensor(qa), pf.tensor(ka), pf.tensor(va)
    out = pf.matmul(pf.softmax(pf.matmul(q, k.transpose(-2, -1)) * scale, -1), v)
    assert "attention " in ex.describe_plan(out.graph(), [out.node().id()])
    res = ex.execute(out.graph(), [out.node().id()])
    assert res.success, res.error_message
    g = res.outputs[out.node().id()]
    qb, kb, vb = (bf16(a).astype(np.float64) for a in (qa, ka, va))
    s64 = np.float64(np.float32(scale)) * (qb @ kb.swapaxes(-1, -2))
    p64 = np.exp(s64 - s64.max(-1, keepdims=True))
    r = (p64 / p64.sum(-1, keepdims=True)) @ vb
    close_rows(g.reshape(-1, d), r.reshape(-1, d), 1e-2, what="bf16 attention")
    ex.close()


def test_encoder_block_bf16(oracle_mod, native):
    """A whole encoder block in the bf16 mode: head-split bf16 projections,
    the fused attention writing the out-projection's bf16 operand."""
    from pyflame_b200 import workloads
    ex = pf.CudaExecutor(pf.CudaExecutor.Config(precision="bf16"))
    w = workloads.encoder(batch=2, seq=64, d=128, heads=2, ff=256)
    plan = ex.describe_plan(w.outputs[0].graph(), w.output_ids())
    assert "attention " in plan and "+operand" in plan, plan
    (g,), (r,) = run(ex, w.outputs, oracle_mod)
    close_rows(g, r, 2 * RTOL_GEMM_BF16, what="bf16 encoder")
    ex.close()


def test_encoder_block_small(cuda_executor, oracle_mod):
    from pyflame_b200 import workloads
    w = workloads.encoder(batch=2, seq=16, d=64, heads=4, ff=256)
    (g,), (r,) = run(cuda_executor, w.outputs, oracle_mod)
    close_rows(g, r, RTOL_GEMM_TF32X3, what="encoder")


def test_gemm_chain_small(cuda_executor, oracle_mod):
    from pyflame_b200 import workloads
    w = workloads.gemm_chain(rows=64, d=512, h=1024)
    (g,), (r,) = run(cuda_executor, w.outputs, oracle_mod)
    close_rows(g, r, RTOL_GEMM_TF32X3, what="gemm chain")


def test_convstack_small(cuda_executor, oracle_mod):
    from pyflame_b200 import workloads
    w = workloads.convstack(batch=2, hw=64)
    (g,), (r,) = run(cuda_executor, w.outputs, oracle_mod)
    close_rows(g, r, RTOL_GEMM_TF32X3, what="convstack")


# ---- executor behaviour --------------------------------------------------------------------

def test_repeat_execution_uses_cached_plan(cuda_executor, oracle_mod, rng):
    x = pf.tensor(rng.standard_normal((64, 128)).astype(np.float32))
    out = pf.softmax(pf.relu(x) * 2.0, -1)
    g = out.graph()
    r1 = cuda_executor.execute(g, [out.node().id()])
    r2 = cuda_executor.execute(g, [out.node().id()])
    r3 = cuda_executor.execute(g, [out.node().id()])
    assert r1.success and r2.success and r3.success
    bitexact(r1.outputs[out.node().id()], r2.outputs[out.node().id()])
    bitexact(r1.outputs[out.node().id()], r3.outputs[out.node().id()])
    assert r3.compile_time_ms < 1000.0


def test_errors_do_not_raise(cuda_executor):
    a = pf.tensor(np.ones((4, 4), np.float32))
    g = a.graph()
    bad = g.create_op(pf.OpType.CONV3D, [a.node()], pf.TensorSpec([4, 4]))
    res = cuda_executor.execute(g, [bad.id()])
    assert not res.success and "Unsupported" in res.error_message
    res = cuda_executor.execute(g, [123456])
    assert not res.success
    # the executor stays usable
    ok = cuda_executor.execute(g, [pf.relu(a).node().id()])
    assert ok.success


def test_executor_boundary_dispatch():
    ex = pf.Executor(pf.ExecutorConfig(backend=pf.Backend.CUDA))
    a = pf.tensor([1.0, -2.0, 3.0])
    r = ex.execute(a.graph(), [pf.relu(a).node().id()])
    assert r.success
    np.testing.assert_array_equal(list(r.outputs.values())[0], [1, 0, 3])
    assert not pf.Executor(pf.ExecutorConfig(backend=pf.Backend.SIMULATOR)).execute(a.graph(), []).success


def test_tensor_api_eval_numpy():
    pf.set_device("cuda")
    a = pf.tensor([[1.0, 2.0], [3.0, 4.0]])
    b = pf.tensor([[5.0, 6.0], [7.0, 8.0]])
    np.testing.assert_allclose(pf.matmul(a, b).numpy(), [[19, 22], [43, 50]], rtol=1e-6)
    np.testing.assert_allclose((a * 2.0 + 1.0).numpy(), [[3, 5], [7, 9]])
    info = pf.device_info()
    assert info["type"] == "cuda" and info["compute_units"] > 0


def test_device_resident_execution(cuda_executor, oracle_mod):
    import torch
    from pyflame_b200 import workloads
    w = workloads.fused(64, 512)
    g = w.outputs[0].graph()
    ids = [t.node().id() for t in w.outputs]
    xd = torch.from_numpy(w.inputs["x"].node().constant_data().copy()).cuda()
    yd = torch.from_numpy(w.inputs["y"].node().constant_data().copy()).cuda()
    outs = [torch.empty(t.shape, device="cuda") for t in w.outputs]
    for _ in range(3):
        cuda_executor.execute_device(g, {w.inputs["x"].node().id(): xd.data_ptr(),
                                         w.inputs["y"].node().id(): yd.data_ptr()}, ids,
                                     [o.data_ptr() for o in outs])
    torch.cuda.synchronize()
    ref = oracle_mod.run(g, ids)
    # the row max selects one value of z = sigmoid(x*y+0.5) - relu(x), which
    # carries the device exp's last-bit difference from the host libm
    close(outs[2].cpu().numpy(), ref[ids[2]], rtol=1e-5, atol=1e-6)
    close_rows(outs[3].cpu().numpy(), ref[ids[3]], 1e-5)


@pytest.mark.parametrize("chunks", [1, 2, 5])
def test_streamed_execution(cuda_executor, oracle_mod, chunks):
    """execute_streamed over `chunks` chunks equals the oracle on the whole
    batch (rows are independent), for row kernels and a GEMM chain."""
    import torch
    from pyflame_b200 import workloads
    rows, cols = 48, 256
    full = workloads.fused(rows * chunks, cols)
    ids_full = [t.node().id() for t in full.outputs]
    ref = oracle_mod.run(full.outputs[0].graph(), ids_full)
    xs = torch.from_numpy(full.inputs["x"].node().constant_data().copy()).pin_memory()
    ys = torch.from_numpy(full.inputs["y"].node().constant_data().copy()).pin_memory()
    w = workloads.fused(rows, cols)
    g = w.outputs[0].graph()
    ids = [t.node().id() for t in w.outputs]
    outs = [torch.empty((rows * chunks,) + tuple(t.shape[1:])).pin_memory().numpy() for t in w.outputs]
    for _ in range(2):  # the second call replays captured graphs
        cuda_executor.execute_streamed(g, {w.inputs["x"].node().id(): xs.numpy(), w.inputs["y"].node().id(): ys.numpy()},
                                       ids, outs)
    z = full.outputs[0].node().inputs()[0]
    zabs = np.abs(oracle_mod.run(full.outputs[0].graph(), [z.id()])[z.id()]).sum(1)
    close_sum(outs[0], ref[ids_full[0]], zabs, what="sum")
    close_sum(outs[1], ref[ids_full[1]], zabs / cols, what="mean")
    close(outs[2], ref[ids_full[2]], rtol=1e-5, atol=1e-6, what="max")
    close_rows(outs[3], ref[ids_full[3]], 1e-5, what="layernorm")
    mc = workloads.mlp(batch=16)
    mfull = workloads.mlp(batch=16 * chunks)
    mids = [t.node().id() for t in mfull.outputs]
    mref = oracle_mod.run(mfull.outputs[0].graph(), mids)[mids[0]]
    xin = torch.from_numpy(mfull.inputs["x"].node().constant_data().copy()).pin_memory()
    mout = torch.empty(mref.shape).pin_memory().numpy()
    cuda_executor.execute_streamed(mc.outputs[0].graph(), {mc.inputs["x"].node().id(): xin.numpy()},
                                   [mc.outputs[0].node().id()], [mout])
    close_rows(mout, mref, RTOL_GEMM_TF32X3, what="mlp streamed")


@pytest.mark.parametrize("fail_at", [1, 2, 4])
def test_injected_allocation_failure(native, oracle_mod, fail_at):
    """An allocation that fails (injected on the host at the fail_at-th
    allocation) comes back as success=False naming the injection, never as an
    exception; releasing the executor's memory leaves nothing allocated; a
    fresh executor then runs the same graph correctly."""
    from pyflame_b200 import workloads
    from pyflame_b200.backend import CudaExecutor
    w = workloads.gemm_chain(rows=64, d=256, h=512)
    g, ids = w.graph(), w.output_ids()
    ex = CudaExecutor(CudaExecutor.Config(fail_after_n_allocations=fail_at))
    try:
        r = ex.execute(g, ids)
        assert not r.success and "injected allocation failure" in r.error_message, r.error_message
        assert ex.get_memory_stats().total_allocations == fail_at - 1
        ex.release_constants()
        s = ex.get_memory_stats()
        assert s.total_allocated == 0 and s.resident_constant_bytes == 0, s
    finally:
        ex.close()
    ok = CudaExecutor(CudaExecutor.Config())
    try:
        r = ok.execute(g, ids)
        assert r.success, r.error_message
        close_rows(r.outputs[ids[0]], oracle_mod.run(g, ids)[ids[0]], RTOL_GEMM_TF32X3, what="after injection")
    finally:
        ok.close()


def test_memory_stats_and_release(cuda_executor):
    s = cuda_executor.get_memory_stats()
    assert s.total_allocations >= 1
    info = cuda_executor.get_device_info()
    assert info.architecture.startswith("sm_10")


def test_empty_and_degenerate_shapes(cuda_executor, oracle_mod, rng):
    """Zero-row batches, a reduction over a length-1 dim, a 1x1 matmul and a
    single-element softmax row: the executor returns correctly shaped (and,
    where defined, exact) results instead of failing a launch."""
    e = pf.tensor(np.zeros((0, 8), np.float32))
    w = pf.tensor(rng.standard_normal((8, 4)).astype(np.float32))
    one = pf.tensor(rng.standard_normal((5, 1)).astype(np.float32))
    outs = [pf.relu(e) * 2.0, pf.matmul(e, w), one.sum(1), one.max(1), pf.softmax(one, -1),
            pf.matmul(pf.tensor([[3.0]]), pf.tensor([[-2.0]]))]
    gpu, ref = run(cuda_executor, outs, oracle_mod)
    assert gpu[0].shape == (0, 8) and gpu[1].shape == (0, 4)
    for g_, r_ in zip(gpu[2:], ref[2:]):
        bitexact(g_, r_)


def test_repeated_call_sees_changed_input_values(cuda_executor, oracle_mod, rng):
    """A repeated call on an unchanged graph skips re-analysis, but an INPUT
    whose values were all equal (a scalar in the plan) and then change in
    place must be read again, not served from the old plan."""
    g = pf.get_current_graph()
    data = np.full((16, 64), 2.0, np.float32)
    x = pf.Tensor(g, g.create_input(pf.TensorSpec([16, 64])))
    x.node().set_constant_data(data, copy=False)
    y = pf.relu(x) * 3.0 + 1.0
    r1 = cuda_executor.execute(g, [y.node().id()])
    assert r1.success and np.all(r1.outputs[y.node().id()] == 7.0)
    data[...] = rng.standard_normal((16, 64)).astype(np.float32)  # same array, same graph version
    r2 = cuda_executor.execute(g, [y.node().id()])
    assert r2.success
    np.testing.assert_array_equal(r2.outputs[y.node().id()], oracle_mod.run(g, [y.node().id()])[y.node().id()])
    r3 = cuda_executor.execute(g, [y.node().id()])
    np.testing.assert_array_equal(r3.outputs[y.node().id()], r2.outputs[y.node().id()])
