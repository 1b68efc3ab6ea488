"""Neural-network modules that emit the same IR as PyFlame's C++ producers
(src/nn/*.cpp): node types, input order, attribute names and C++ attribute
types.  Only the forward (inference) graph builders are provided; training
(autograd, optimisers, losses) is outside the CUDA executor's scope.
"""
from __future__ import annotations

import math
from collections import OrderedDict
from typing import Optional, Sequence, Tuple

import numpy as np

from . import ir
from .ir import OpType, TensorSpec
from .tensor import Tensor, gelu, matmul, relu, sigmoid, silu, softmax, tanh


def _pair(v) -> Tuple[int, int]:
    return (int(v[0]), int(v[1])) if isinstance(v, (tuple, list)) else (int(v), int(v))


_deferred = [False]


class deferred_init:
    """Inside this context, modules create their parameters as data-less
    leaves of the right shape instead of random/constant tensors (for models
    whose weights are loaded right after construction)."""

    def __enter__(self):
        self._prev = _deferred[0]
        _deferred[0] = True
        return self

    def __exit__(self, *exc):
        _deferred[0] = self._prev


def _param(shape, make):
    if _deferred[0]:
        from .tensor import get_current_graph
        g = get_current_graph()
        return Tensor(g, g.create_constant(TensorSpec(shape)))
    return make()


class Module:
    """module.hpp:15-135 (parameters, submodules, train/eval)."""

    def __init__(self):
        self._params: "OrderedDict[str, Tensor]" = OrderedDict()
        self._modules: "OrderedDict[str, Module]" = OrderedDict()
        self._training = False

    def register_parameter(self, name: str, t: Tensor) -> Tensor:
        self._params[name] = t
        return t

    def register_module(self, name: str, m: "Module") -> "Module":
        self._modules[name] = m
        return m

    def parameters(self):
        out = list(self._params.values())
        for m in self._modules.values():
            out += m.parameters()
        return out

    def named_parameters(self, prefix: str = ""):
        for k, v in self._params.items():
            yield prefix + k, v
        for mk, m in self._modules.items():
            yield from m.named_parameters(prefix + mk + ".")

    def set_parameter(self, name: str, value: np.ndarray) -> None:
        """Replace a parameter by a constant holding `value` (weight loading)."""
        mod, _, leaf = name.rpartition(".")
        target = self
        for part in [p for p in mod.split(".") if p]:
            target = target._modules[part]
        old = target._params[leaf]
        arr = np.asarray(value, dtype=np.float32)
        if list(arr.shape) != old.shape:
            raise ValueError(f"{name}: shape {list(arr.shape)} != {old.shape}")
        t = Tensor.from_data(arr)
        target._params[leaf] = t
        setattr(target, "_p_" + leaf, t)

    def load_state_dict(self, state: dict) -> None:
        for k, v in state.items():
            self.set_parameter(k, v)

    def train(self, mode: bool = True) -> "Module":
        self._training = mode
        for m in self._modules.values():
            m.train(mode)
        return self

    def eval(self) -> "Module":
        return self.train(False)

    def is_training(self) -> bool:
        return self._training

    def __call__(self, *a, **k):
        return self.forward(*a, **k)

    def forward(self, x):  # pragma: no cover - abstract
        raise NotImplementedError

    def p(self, name: str) -> Tensor:
        return self._params[name]


class Linear(Module):
    """linear.cpp:8-44: weight [out, in] ~ N(0, 2/in), bias zeros;
    forward = matmul(x, transpose(weight, 0, 1)) + bias."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features, self.out_features, self.use_bias = in_features, out_features, bias
        std = math.sqrt(2.0 / in_features)
        self.register_parameter("weight", _param([out_features, in_features],
                                                 lambda: Tensor.randn([out_features, in_features]) * std))
        if bias:
            self.register_parameter("bias", _param([out_features], lambda: Tensor.zeros([out_features])))

    def forward(self, x: Tensor) -> Tensor:
        out = matmul(x, self.p("weight").transpose(0, 1))
        if self.use_bias:
            out = out + self.p("bias")
        return out


class Conv2d(Module):
    """conv.cpp:20-131: CONV2D(x, w) with attrs stride/padding/dilation
    (vector<int64_t>) and groups (int64_t); bias added as [1, C, 1, 1]."""

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, groups=1,
                 bias=True):
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.kernel_size, self.stride = _pair(kernel_size), _pair(stride)
        self.padding, self.dilation, self.groups, self.use_bias = _pair(padding), _pair(dilation), groups, bias
        fan_in = (in_channels // groups) * self.kernel_size[0] * self.kernel_size[1]
        std = math.sqrt(2.0 / fan_in)
        wshape = [out_channels, in_channels // groups, *self.kernel_size]
        self.register_parameter("weight", _param(wshape, lambda: Tensor.randn(wshape) * std))
        if bias:
            self.register_parameter("bias", _param([out_channels], lambda: Tensor.zeros([out_channels])))

    @staticmethod
    def calc_output_size(size, k, s, p, d):
        return (size + 2 * p - d * (k - 1) - 1) // s + 1  # conv.cpp:75-78

    def forward(self, x: Tensor) -> Tensor:
        n, c, h, w = x.shape
        if c != self.in_channels:
            raise ValueError("Input channels mismatch")
        oh = self.calc_output_size(h, self.kernel_size[0], self.stride[0], self.padding[0], self.dilation[0])
        ow = self.calc_output_size(w, self.kernel_size[1], self.stride[1], self.padding[1], self.dilation[1])
        g = x.graph()
        node = g.create_op(OpType.CONV2D, [x.node(), self.p("weight").node()],
                           TensorSpec([n, self.out_channels, oh, ow], x.dtype))
        node.set_attr("stride", list(self.stride), ir.A_INT64_VEC)
        node.set_attr("padding", list(self.padding), ir.A_INT64_VEC)
        node.set_attr("dilation", list(self.dilation), ir.A_INT64_VEC)
        node.set_attr("groups", int(self.groups), ir.A_INT64)
        out = Tensor(g, node)
        if self.use_bias:
            out = out + self.p("bias").reshape([1, self.out_channels, 1, 1])
        return out


class BatchNorm2d(Module):
    """normalization.cpp:53-93: BATCH_NORM(x, weight, bias, running_mean,
    running_var) with attrs eps/momentum (float) and training/affine/
    track_running_stats (bool)."""

    def __init__(self, num_features, eps=1e-5, momentum=0.1, affine=True, track_running_stats=True):
        super().__init__()
        self.num_features, self.eps, self.momentum = num_features, eps, momentum
        self.affine, self.track_running_stats = affine, track_running_stats
        if affine:
            self.register_parameter("weight", Tensor.ones([num_features]))
            self.register_parameter("bias", Tensor.zeros([num_features]))
        if track_running_stats:
            self.register_parameter("running_mean", Tensor.zeros([num_features]))
            self.register_parameter("running_var", Tensor.ones([num_features]))

    def forward(self, x: Tensor) -> Tensor:
        if x.ndim != 4:
            raise ValueError("BatchNorm2d expects 4D input [N, C, H, W]")
        ins = [x.node()]
        if self.affine:
            ins += [self.p("weight").node(), self.p("bias").node()]
        if self.track_running_stats:
            ins += [self.p("running_mean").node(), self.p("running_var").node()]
        g = x.graph()
        node = g.create_op(OpType.BATCH_NORM, ins, TensorSpec(x.shape, x.dtype))
        node.set_attr("eps", float(self.eps), ir.A_FLOAT)
        node.set_attr("momentum", float(self.momentum), ir.A_FLOAT)
        node.set_attr("training", bool(self.is_training()), ir.A_BOOL)
        node.set_attr("affine", bool(self.affine), ir.A_BOOL)
        node.set_attr("track_running_stats", bool(self.track_running_stats), ir.A_BOOL)
        return Tensor(g, node)


class LayerNorm(Module):
    """normalization.cpp:224-255: LAYER_NORM(x, weight, bias) with attrs
    normalized_shape (vector<int64_t>), eps (float), elementwise_affine (bool)."""

    def __init__(self, normalized_shape, eps=1e-5, elementwise_affine=True):
        super().__init__()
        self.normalized_shape = [int(normalized_shape)] if isinstance(normalized_shape, int) else \
            [int(s) for s in normalized_shape]
        self.eps, self.elementwise_affine = eps, elementwise_affine
        if elementwise_affine:
            self.register_parameter("weight", Tensor.ones(self.normalized_shape))
            self.register_parameter("bias", Tensor.zeros(self.normalized_shape))

    def forward(self, x: Tensor) -> Tensor:
        k = len(self.normalized_shape)
        if x.shape[-k:] != self.normalized_shape:
            raise ValueError("Input shape doesn't match normalized_shape")
        ins = [x.node()]
        if self.elementwise_affine:
            ins += [self.p("weight").node(), self.p("bias").node()]
        g = x.graph()
        node = g.create_op(OpType.LAYER_NORM, ins, TensorSpec(x.shape, x.dtype))
        node.set_attr("normalized_shape", list(self.normalized_shape), ir.A_INT64_VEC)
        node.set_attr("eps", float(self.eps), ir.A_FLOAT)
        node.set_attr("elementwise_affine", bool(self.elementwise_affine), ir.A_BOOL)
        return Tensor(g, node)


class _Pool2d(Module):
    OP = OpType.MAX_POOL2D

    def __init__(self, kernel_size, stride=0, padding=0):
        super().__init__()
        self.kernel_size = _pair(kernel_size)
        s = _pair(stride)
        self.stride = self.kernel_size if s[0] == 0 else s
        self.padding = _pair(padding)

    def forward(self, x: Tensor) -> Tensor:
        n, c, h, w = x.shape
        oh = (h + 2 * self.padding[0] - self.kernel_size[0]) // self.stride[0] + 1  # pooling.cpp:33-36
        ow = (w + 2 * self.padding[1] - self.kernel_size[1]) // self.stride[1] + 1
        g = x.graph()
        node = g.create_op(self.OP, [x.node()], TensorSpec([n, c, oh, ow], x.dtype))
        node.set_attr("kernel_size", list(self.kernel_size), ir.A_INT64_VEC)
        node.set_attr("stride", list(self.stride), ir.A_INT64_VEC)
        node.set_attr("padding", list(self.padding), ir.A_INT64_VEC)
        return Tensor(g, node)


class MaxPool2d(_Pool2d):
    """pooling.cpp:38-63."""
    OP = OpType.MAX_POOL2D


class AvgPool2d(_Pool2d):
    """pooling.cpp:97-122."""
    OP = OpType.AVG_POOL2D


class AdaptiveAvgPool2d(Module):
    """pooling.cpp:150-168: attr output_size (vector<int64_t>)."""

    def __init__(self, output_size):
        super().__init__()
        self.output_size = _pair(output_size)

    def forward(self, x: Tensor) -> Tensor:
        n, c = x.shape[0], x.shape[1]
        g = x.graph()
        node = g.create_op(OpType.ADAPTIVE_AVG_POOL2D, [x.node()], TensorSpec([n, c, *self.output_size], x.dtype))
        node.set_attr("output_size", list(self.output_size), ir.A_INT64_VEC)
        return Tensor(g, node)


class ReLU(Module):
    def forward(self, x):
        return relu(x)


class GELU(Module):
    def forward(self, x):
        return gelu(x)


class Sigmoid(Module):
    def forward(self, x):
        return sigmoid(x)


class Tanh(Module):
    def forward(self, x):
        return tanh(x)


class SiLU(Module):
    def forward(self, x):
        return silu(x)


class Softmax(Module):
    def __init__(self, dim: int = -1):
        super().__init__()
        self.dim = dim

    def forward(self, x):
        return softmax(x, self.dim)


class Dropout(Module):
    """dropout.cpp:26-30: identity outside training."""

    def __init__(self, p: float = 0.5):
        super().__init__()
        self.p_drop = p

    def forward(self, x):
        if self.is_training():
            raise NotImplementedError("dropout in training mode is not part of the inference executor")
        return x


class Flatten(Module):
    def __init__(self, start_dim: int = 1):
        super().__init__()
        self.start_dim = start_dim

    def forward(self, x):
        s = x.shape
        return x.reshape(s[:self.start_dim] + [int(np.prod(s[self.start_dim:]))])


class Sequential(Module):
    """module.cpp:252-258."""

    def __init__(self, *mods: Module):
        super().__init__()
        for i, m in enumerate(mods):
            self.register_module(str(i), m)

    def forward(self, x):
        for m in self._modules.values():
            x = m(x)
        return x


class MultiheadAttention(Module):
    """attention.cpp:16-170: four Linear projections, heads split by
    reshape + transpose(1, 2), scores = matmul(q, k^T) * (1/sqrt(head_dim)),
    softmax(-1), matmul with v, heads merged, out_proj."""

    def __init__(self, embed_dim, num_heads, dropout=0.0, bias=True, add_bias_kv=False, add_zero_attn=False,
                 kdim=0, vdim=0, batch_first=False):
        super().__init__()
        if num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if embed_dim % num_heads:
            raise ValueError("embed_dim must be divisible by num_heads")
        self.embed_dim, self.num_heads, self.head_dim = embed_dim, num_heads, embed_dim // num_heads
        self.batch_first = batch_first
        self.kdim, self.vdim = kdim or embed_dim, vdim or embed_dim
        self.q_proj = self.register_module("q_proj", Linear(embed_dim, embed_dim, bias))
        self.k_proj = self.register_module("k_proj", Linear(self.kdim, embed_dim, bias))
        self.v_proj = self.register_module("v_proj", Linear(self.vdim, embed_dim, bias))
        self.out_proj = self.register_module("out_proj", Linear(embed_dim, embed_dim, bias))

    def scaled_dot_product_attention(self, q, k, v, attn_mask=None):
        scale = 1.0 / math.sqrt(float(self.head_dim))
        scores = matmul(q, k.transpose(-2, -1)) * scale
        if attn_mask is not None:
            scores = scores + attn_mask
        w = softmax(scores, -1)
        return matmul(w, v), w

    def forward(self, query, key=None, value=None, attn_mask=None, need_weights=False):
        key = query if key is None else key
        value = query if value is None else value
        qs = query.shape
        if self.batch_first:
            b, tl = qs[0], qs[1]
            sl = key.shape[1]
        else:
            tl, b = qs[0], qs[1]
            sl = key.shape[0]
        q, k, v = self.q_proj(query), self.k_proj(key), self.v_proj(value)
        H, D = self.num_heads, self.head_dim
        if self.batch_first:
            q = q.reshape([b, tl, H, D]).transpose(1, 2)
            k = k.reshape([b, sl, H, D]).transpose(1, 2)
            v = v.reshape([b, sl, H, D]).transpose(1, 2)
        else:
            q = q.transpose(0, 1).reshape([b, tl, H, D]).transpose(1, 2)
            k = k.transpose(0, 1).reshape([b, sl, H, D]).transpose(1, 2)
            v = v.transpose(0, 1).reshape([b, sl, H, D]).transpose(1, 2)
        out, w = self.scaled_dot_product_attention(q, k, v, attn_mask)
        out = out.transpose(1, 2).reshape([b, tl, self.embed_dim])
        if not self.batch_first:
            out = out.transpose(0, 1)
        out = self.out_proj(out)
        if need_weights:
            return out, w.mean(1)
        return out


class TransformerEncoderLayer(Module):
    """models/transformer.cpp:197-243, post-LN by default
    (transformer.hpp:99): x = norm1(x + attn(x)); x = norm2(x + ffn(x))."""

    def __init__(self, d_model, nhead, dim_feedforward=2048, dropout=0.1, activation="relu",
                 layer_norm_eps=1e-5, batch_first=True, norm_first=False):
        super().__init__()
        self.self_attn = self.register_module("self_attn", MultiheadAttention(d_model, nhead, dropout,
                                                                              batch_first=batch_first))
        self.linear1 = self.register_module("linear1", Linear(d_model, dim_feedforward))
        self.linear2 = self.register_module("linear2", Linear(dim_feedforward, d_model))
        self.norm1 = self.register_module("norm1", LayerNorm(d_model, layer_norm_eps))
        self.norm2 = self.register_module("norm2", LayerNorm(d_model, layer_norm_eps))
        self.activation, self.norm_first = activation, norm_first

    def _act(self, x):
        return relu(x) if self.activation == "relu" else gelu(x)

    def forward(self, src):
        x = src
        if self.norm_first:
            h = self.norm1(x)
            x = x + self.self_attn(h)
            x = x + self.linear2(self._act(self.linear1(self.norm2(x))))
            return x
        x = self.norm1(x + self.self_attn(x))
        x = self.norm2(x + self.linear2(self._act(self.linear1(x))))
        return x
