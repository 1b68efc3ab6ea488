"""pyflame_b200: a B200-native CUDA executor for PyFlame's lazy IR graphs.

The surface mirrors PyFlame's Python package (python/pyflame/__init__.py):
tensors, graph nodes, ops, nn modules, device selection and `eval`, with
'cuda[:N]' as the device.  Evaluation runs on sm_100a GPUs through
libpyflame_cuda.so (include/pyflame_cuda.h); there is no CPU evaluation path.
"""
from . import autograd, ir, nn, serving
from .backend import (Backend, CudaExecutor, DeviceInfo, ExecutionResult, Executor, ExecutorConfig, MemoryStats,
                      cuda_device_count, cuda_get_device, cuda_get_device_info, cuda_is_available, cuda_set_device,
                      cuda_synchronize)
from .device import device_info, eval, get_device, set_device, set_precision, synchronize
from .ir import DType, Graph, Node, NodeType, OpType, TensorSpec, dtype_name, dtype_size
from .tensor import (Tensor, abs, arange, broadcast_to, cat, clamp, cos, exp, from_numpy, full, gelu,
                     get_current_graph, log, log_softmax, manual_seed, matmul, maximum, minimum, ones, pow, rand,
                     randn, relu, reset_graph, sigmoid, silu, sin, softmax, sqrt, stack, tanh, tensor, zeros)

float32, float16, bfloat16 = DType.float32, DType.float16, DType.bfloat16
int32, int16, int8, int64, bool_ = DType.int32, DType.int16, DType.int8, DType.int64, DType.bool_

__version__ = "0.1.0"


def get_graph(t: Tensor) -> Graph:
    return t.graph()


def get_node(t: Tensor) -> Node:
    return t.node()
