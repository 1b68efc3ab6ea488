"""An independent pin for the oracle's restated ops.

PyFlame has no CPU code for Conv2d, BatchNorm, LayerNorm, the pools,
softmax over a non-last dim, batched/broadcast matmul or the
MultiheadAttention composition, so the oracle restates them from the
producers' attribute contracts (conv.cpp:75-131, normalization.cpp:53-93,224-255,
pooling.cpp:33-168, attention.cpp:16-164, shape_inference.hpp:146-217).
These CPU tests hold that restatement to a second, unrelated implementation
of the same PyTorch-compatible semantics: torch's CPU kernels, in float64.
The oracle's float64 shadow must agree to rounding (1e-10 relative to the
row scale), and its float32 evaluation within the parity tolerances.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import pyflame_b200 as pf
from pyflame_b200 import nn
from tests.helpers import close_rows

T64 = torch.float64


def _oracle(oracle_mod, t, precision):
    g = t.graph()
    return oracle_mod.run(g, [t.node().id()], precision)[t.node().id()]


def _check(oracle_mod, t, want, rows_last=True, f32_rtol=1e-5):
    want = np.asarray(want, np.float64)
    got64 = _oracle(oracle_mod, t, "f64")
    got32 = _oracle(oracle_mod, t, "f32")
    assert got64.shape == want.shape, (got64.shape, want.shape)
    shape2 = (-1, want.shape[-1]) if rows_last and want.ndim > 1 else (1, -1)
    close_rows(got64.reshape(shape2), want.reshape(shape2), 1e-10, what="oracle f64 vs torch f64")
    close_rows(got32.reshape(shape2), want.reshape(shape2), f32_rtol, what="oracle f32 vs torch f64")


CONV = [dict(n=2, c=3, h=17, w=15, o=8, k=3, s=1, p=1, d=1, g=1),
        dict(n=2, c=3, h=31, w=29, o=16, k=7, s=2, p=3, d=1, g=1),
        dict(n=1, c=8, h=12, w=13, o=6, k=3, s=2, p=0, d=1, g=1),
        dict(n=1, c=4, h=14, w=14, o=4, k=3, s=1, p=2, d=2, g=1),
        dict(n=2, c=6, h=10, w=9, o=4, k=3, s=1, p=1, d=1, g=2),
        dict(n=1, c=5, h=6, w=20, o=3, k=(1, 5), s=(1, 2), p=(0, 2), d=1, g=1)]


@pytest.mark.parametrize("cfg", CONV, ids=[f"conv{i}" for i in range(len(CONV))])
def test_conv2d_with_bias(oracle_mod, rng, cfg):
    k = cfg["k"] if isinstance(cfg["k"], tuple) else (cfg["k"], cfg["k"])
    x = rng.standard_normal((cfg["n"], cfg["c"], cfg["h"], cfg["w"])).astype(np.float32)
    w = rng.standard_normal((cfg["o"], cfg["c"] // cfg["g"], *k)).astype(np.float32)
    b = rng.standard_normal(cfg["o"]).astype(np.float32)
    with nn.deferred_init():
        conv = nn.Conv2d(cfg["c"], cfg["o"], k, cfg["s"], cfg["p"], cfg["d"], cfg["g"])
    conv.set_parameter("weight", w)
    conv.set_parameter("bias", b)
    out = conv(pf.tensor(x))
    want = F.conv2d(torch.from_numpy(x).to(T64), torch.from_numpy(w).to(T64), torch.from_numpy(b).to(T64),
                    stride=cfg["s"], padding=cfg["p"], dilation=cfg["d"], groups=cfg["g"])
    _check(oracle_mod, out, want.numpy(), rows_last=False)


def test_batchnorm_eval(oracle_mod, rng):
    c = 5
    x = rng.standard_normal((3, c, 7, 6)).astype(np.float32)
    gamma, beta = rng.standard_normal(c).astype(np.float32), rng.standard_normal(c).astype(np.float32)
    mean, var = rng.standard_normal(c).astype(np.float32), rng.uniform(0.1, 3.0, c).astype(np.float32)
    bn = nn.BatchNorm2d(c, eps=1e-3)
    bn.eval()
    for name, v in (("weight", gamma), ("bias", beta), ("running_mean", mean), ("running_var", var)):
        bn.set_parameter(name, v)
    out = bn(pf.tensor(x))
    t = lambda a: torch.from_numpy(a).to(T64)  # noqa: E731
    want = F.batch_norm(t(x), t(mean), t(var), t(gamma), t(beta), training=False, eps=1e-3)
    _check(oracle_mod, out, want.numpy(), rows_last=False)


@pytest.mark.parametrize("shape,ns,affine", [((4, 6, 10), [10], True), ((4, 6, 10), [6, 10], True),
                                            ((7, 33), [33], False)])
def test_layer_norm(oracle_mod, rng, shape, ns, affine):
    x = (rng.standard_normal(shape) * 3 + 1).astype(np.float32)
    ln = nn.LayerNorm(ns, eps=1e-5, elementwise_affine=affine)
    w = b = None
    if affine:
        w, b = rng.standard_normal(ns).astype(np.float32), rng.standard_normal(ns).astype(np.float32)
        ln.set_parameter("weight", w)
        ln.set_parameter("bias", b)
    out = ln(pf.tensor(x))
    want = F.layer_norm(torch.from_numpy(x).to(T64), ns, None if w is None else torch.from_numpy(w).to(T64),
                        None if b is None else torch.from_numpy(b).to(T64), eps=1e-5)
    _check(oracle_mod, out, want.numpy())


@pytest.mark.parametrize("kind,k,s,p", [("max", 3, 2, 0), ("max", 3, 2, 1), ("max", 2, 2, 0), ("avg", 3, 2, 1),
                                        ("avg", 2, 1, 0), ("avg", 3, 3, 1)])
def test_pools(oracle_mod, rng, kind, k, s, p):
    x = rng.standard_normal((2, 3, 11, 12)).astype(np.float32)
    mod = (nn.MaxPool2d if kind == "max" else nn.AvgPool2d)(k, s, p)
    out = mod(pf.tensor(x))
    xt = torch.from_numpy(x).to(T64)
    want = F.max_pool2d(xt, k, s, p) if kind == "max" else F.avg_pool2d(xt, k, s, p, count_include_pad=True)
    _check(oracle_mod, out, want.numpy(), rows_last=False)
    if kind == "max":  # selection: bit-exact in float32 too
        np.testing.assert_array_equal(_oracle(oracle_mod, out, "f32"),
                                      F.max_pool2d(torch.from_numpy(x), k, s, p).numpy())


@pytest.mark.parametrize("osz", [(1, 1), (2, 3), (4, 4)])
def test_adaptive_avg_pool(oracle_mod, rng, osz):
    x = rng.standard_normal((2, 3, 9, 10)).astype(np.float32)
    out = nn.AdaptiveAvgPool2d(osz)(pf.tensor(x))
    want = F.adaptive_avg_pool2d(torch.from_numpy(x).to(T64), osz)
    _check(oracle_mod, out, want.numpy(), rows_last=False)


@pytest.mark.parametrize("shape,dim", [((3, 7, 5), 1), ((4, 2, 33), 0), ((5, 6), -1)])
@pytest.mark.parametrize("log", [False, True])
def test_softmax_any_dim(oracle_mod, rng, shape, dim, log):
    x = (rng.standard_normal(shape) * 4).astype(np.float32)
    out = (pf.log_softmax if log else pf.softmax)(pf.tensor(x), dim)
    xt = torch.from_numpy(x).to(T64)
    want = (F.log_softmax if log else F.softmax)(xt, dim=dim)
    _check(oracle_mod, out, want.numpy(), rows_last=False)


@pytest.mark.parametrize("a_shape,b_shape", [((2, 1, 5, 7), (3, 7, 4)), ((4, 9, 6), (6, 5)), ((2, 3, 4, 8), (2, 3, 8, 2))])
def test_batched_broadcast_matmul(oracle_mod, rng, a_shape, b_shape):
    a = rng.standard_normal(a_shape).astype(np.float32)
    b = rng.standard_normal(b_shape).astype(np.float32)
    out = pf.matmul(pf.tensor(a), pf.tensor(b))
    want = torch.matmul(torch.from_numpy(a).to(T64), torch.from_numpy(b).to(T64))
    _check(oracle_mod, out, want.numpy())


@pytest.mark.parametrize("batch_first", [True, False])
def test_multihead_attention_composition(oracle_mod, rng, batch_first):
    """PyFlame's MHA graph (four projections, head split, scaled scores,
    softmax, AV, head merge, out projection) against torch's fused module."""
    e, h, b, s = 16, 4, 2, 7
    x = rng.standard_normal((b, s, e) if batch_first else (s, b, e)).astype(np.float32)
    ws = {n: (rng.standard_normal((e, e)) * 0.3).astype(np.float32) for n in ("q", "k", "v", "out")}
    bs = {n: (rng.standard_normal(e) * 0.1).astype(np.float32) for n in ("q", "k", "v", "out")}
    with nn.deferred_init():
        mha = nn.MultiheadAttention(e, h, batch_first=batch_first)
    for n in ws:
        mha.set_parameter(f"{n}_proj.weight", ws[n])
        mha.set_parameter(f"{n}_proj.bias", bs[n])
    out = mha(pf.tensor(x))
    ref = torch.nn.MultiheadAttention(e, h, bias=True, batch_first=batch_first, dtype=T64)
    with torch.no_grad():
        ref.in_proj_weight.copy_(torch.from_numpy(np.concatenate([ws["q"], ws["k"], ws["v"]])))
        ref.in_proj_bias.copy_(torch.from_numpy(np.concatenate([bs["q"], bs["k"], bs["v"]])))
        ref.out_proj.weight.copy_(torch.from_numpy(ws["out"]))
        ref.out_proj.bias.copy_(torch.from_numpy(bs["out"]))
        xt = torch.from_numpy(x).to(T64)
        want, _ = ref(xt, xt, xt, need_weights=False)
    _check(oracle_mod, out, want.numpy())


def test_encoder_block_composition(oracle_mod, rng):
    """Post-LN encoder block (transformer.cpp:222-240) with GELU (tanh form)
    against torch's TransformerEncoderLayer in float64.  Head dim 4, so the
    graph's float32 score scale 1/sqrt(4) is exact."""
    d, h, ff, b, s = 16, 4, 32, 2, 5
    x = rng.standard_normal((b, s, d)).astype(np.float32)
    with nn.deferred_init():
        blk = nn.TransformerEncoderLayer(d, h, ff, dropout=0.0, activation="gelu", batch_first=True)
    blk.eval()
    params = {}
    for name, p in list(blk.named_parameters()):
        v = (rng.standard_normal(p.shape) * (0.3 if len(p.shape) == 2 else 0.1)).astype(np.float32)
        if name.startswith("norm"):
            v = (1.0 + v) if name.endswith("weight") else v
        blk.set_parameter(name, v)
        params[name] = v
    out = blk(pf.tensor(x))
    # GELU's tanh form with PyFlame's float literals (executor.cpp:404-409)
    c1, c2 = float(np.float32(0.7978845608)), float(np.float32(0.044715))

    def gelu(t):
        return 0.5 * t * (1.0 + torch.tanh(c1 * (t + c2 * t * t * t)))

    ref = torch.nn.TransformerEncoderLayer(d, h, ff, dropout=0.0, activation=gelu, batch_first=True,
                                           norm_first=False, dtype=T64)
    ref.eval()
    t = lambda a: torch.from_numpy(a).to(T64)  # noqa: E731
    with torch.no_grad():
        sa = ref.self_attn
        sa.in_proj_weight.copy_(torch.cat([t(params[f"self_attn.{n}_proj.weight"]) for n in "qkv"]))
        sa.in_proj_bias.copy_(torch.cat([t(params[f"self_attn.{n}_proj.bias"]) for n in "qkv"]))
        sa.out_proj.weight.copy_(t(params["self_attn.out_proj.weight"]))
        sa.out_proj.bias.copy_(t(params["self_attn.out_proj.bias"]))
        for n in ("linear1", "linear2", "norm1", "norm2"):
            getattr(ref, n).weight.copy_(t(params[f"{n}.weight"]))
            getattr(ref, n).bias.copy_(t(params[f"{n}.bias"]))
        want = ref(t(x))
    _check(oracle_mod, out, want.numpy())
