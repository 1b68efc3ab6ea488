"""Generate the golden fixtures in this folder by running PyFlame's own CPU
code (oracle/_ref/libpyflame_ref.so, compiled from the PyFlame sources by
oracle/Makefile) on seeded inputs.

    python tests/golden/make_golden.py

Writes reference_outputs.npz: for every case, the inputs and the output of
PyFlame's CPU reference executor (src/backend/executor.cpp:205-524) or of its
scalar kernels ops::*_cpu (src/ops/*.cpp), keyed "<case>/<name>".  The
known-answer tests of PyFlame's tests/cpp/test_operations.cpp are recorded in
kats.json.  Both files are committed; the tests read them, never PyFlame's
sources.
"""
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

import pyflame_b200 as pf  # noqa: E402
from oracle import oracle as O  # noqa: E402

# Known answers of tests/cpp/test_operations.cpp (file:line of each case).
KATS = [
    {"case": "relu", "src": "tests/cpp/test_operations.cpp:16-29", "op": "relu", "x": [-2, -1, 0, 1, 2],
     "expect": [0, 0, 0, 1, 2]},
    {"case": "sigmoid0", "src": "tests/cpp/test_operations.cpp:31-40", "op": "sigmoid", "x": [0], "expect": [0.5]},
    {"case": "tanh0", "src": "tests/cpp/test_operations.cpp:42-51", "op": "tanh", "x": [0], "expect": [0]},
    {"case": "exp", "src": "tests/cpp/test_operations.cpp:53-63", "op": "exp", "x": [0, 1],
     "expect": [1, 2.718281828459045]},
    {"case": "log", "src": "tests/cpp/test_operations.cpp:65-75", "op": "log", "x": [1, 2.718281828459045],
     "expect": [0, 1]},
    {"case": "sqrt", "src": "tests/cpp/test_operations.cpp:77-89", "op": "sqrt", "x": [1, 4, 9], "expect": [1, 2, 3]},
    {"case": "abs", "src": "tests/cpp/test_operations.cpp:91-103", "op": "abs", "x": [-3, -1, 0, 1, 3],
     "expect": [3, 1, 0, 1, 3]},
    {"case": "sum", "src": "tests/cpp/test_operations.cpp:105-114", "op": "sum", "x": [1, 2, 3, 4], "expect": 10},
    {"case": "mean", "src": "tests/cpp/test_operations.cpp:116-125", "op": "mean", "x": [1, 2, 3, 4], "expect": 2.5},
    {"case": "max", "src": "tests/cpp/test_operations.cpp:127-136", "op": "max", "x": [1, 5, 3, 2], "expect": 5},
    {"case": "min", "src": "tests/cpp/test_operations.cpp:138-147", "op": "min", "x": [5, 1, 3, 2], "expect": 1},
    {"case": "chained", "src": "tests/cpp/test_operations.cpp:149-162", "op": "chained", "x": [],
     "expect": [8.0] * 10},
    {"case": "multiple_reductions", "src": "tests/cpp/test_operations.cpp:164-175", "op": "arange_sum_mean",
     "x": [], "expect": [55.0, 5.5]},
    {"case": "matmul2d", "src": "tests/cpp/test_operations.cpp:177-195", "op": "matmul", "a": [[1, 2], [3, 4]],
     "b": [[5, 6], [7, 8]], "expect": [[19, 22], [43, 50]]},
    {"case": "matmul_nonsquare", "src": "tests/cpp/test_operations.cpp:211-227", "op": "matmul",
     "a": [[1, 2, 3]], "b": [[1], [2], [3]], "expect": [[14]]},
    {"case": "tensor_add", "src": "tests/cpp/test_tensor.cpp:95-108", "op": "ones_plus_full2", "x": [],
     "expect": [[3.0] * 3] * 2},
    {"case": "tensor_mul", "src": "tests/cpp/test_tensor.cpp:110-120", "op": "full3_times_full4", "x": [],
     "expect": [[12.0] * 2] * 2},
    {"case": "scalar_ops", "src": "tests/cpp/test_tensor.cpp:122-137", "op": "ones_plus2_times3", "x": [],
     "expect": [[3.0] * 3, [3.0] * 3]},
    {"case": "negation", "src": "tests/cpp/test_tensor.cpp:139-147", "op": "neg_full5", "x": [],
     "expect": [[-5.0] * 2] * 2},
]


def executor_cases(ref, rng):
    """Graphs PyFlame's CPU executor supports end to end (same-shape binary
    ops, unary ops, activations, full reductions, 2-D matmul, reshape, 2-D
    transpose)."""
    out = {}
    specials = np.array([0.0, -0.0, 1.0, -1.0, 3.5, -2.25, 1e-20, 30.0, -30.0, 0.5], np.float32)

    def add_case(name, tensors, inputs):
        g = tensors[0].graph()
        ids = [t.node().id() for t in tensors]
        res = ref.execute_cpu(g, ids)
        for k, v in inputs.items():
            out[f"{name}/in_{k}"] = v
        for j, i in enumerate(ids):
            out[f"{name}/out{j}"] = res[i]

    for op in ["neg", "abs", "sqrt", "exp", "log", "sin", "cos", "tanh", "relu", "sigmoid", "gelu", "silu"]:
        pf.reset_graph()
        x = np.concatenate([rng.standard_normal(250).astype(np.float32) * 3, specials])
        if op in ("sqrt", "log"):
            x = np.abs(x) + np.float32(1e-3)
        t = pf.tensor(x)
        f = (lambda a: -a) if op == "neg" else getattr(pf, op)
        add_case(f"unary_{op}", [f(t)], {"x": x})
    for op in ["add", "sub", "mul", "div"]:
        pf.reset_graph()
        a = rng.standard_normal((17, 33)).astype(np.float32)
        b = rng.standard_normal((17, 33)).astype(np.float32)
        if op == "div":
            b[0, :4] = [0.0, 0.0, -0.0, 0.0]
            a[0, :4] = [0.0, 2.0, 2.0, -3.0]
        ta, tb = pf.tensor(a), pf.tensor(b)
        add_case(f"binary_{op}", [{"add": ta + tb, "sub": ta - tb, "mul": ta * tb, "div": ta / tb}[op]],
                 {"a": a, "b": b})
    for op in ["sum", "mean", "max", "min"]:
        pf.reset_graph()
        x = rng.standard_normal(999).astype(np.float32)
        add_case(f"full_{op}", [getattr(pf.tensor(x), op)()], {"x": x})
    pf.reset_graph()
    a = rng.standard_normal((13, 29)).astype(np.float32)
    b = rng.standard_normal((29, 7)).astype(np.float32)
    add_case("matmul_2d", [pf.matmul(pf.tensor(a), pf.tensor(b))], {"a": a, "b": b})
    pf.reset_graph()
    x = rng.standard_normal((6, 10)).astype(np.float32)
    t = pf.tensor(x)
    add_case("reshape", [t.reshape([3, 20])], {"x": x})
    pf.reset_graph()
    t = pf.tensor(x)
    add_case("transpose_2d", [t.transpose(0, 1)], {"x": x})
    # the elementwise part of the fused benchmark graph
    pf.reset_graph()
    x = rng.standard_normal((16, 64)).astype(np.float32)
    y = rng.standard_normal((16, 64)).astype(np.float32)
    tx, ty = pf.tensor(x), pf.tensor(y)
    add_case("fused_z", [pf.sigmoid(tx * ty + 0.5) - pf.relu(tx)], {"x": x, "y": y})
    return out


def kernel_cases(ref, rng):
    """PyFlame's scalar kernels ops::*_cpu (not reachable from its executors)."""
    out = {}
    x = (rng.standard_normal((12, 37)) * 3).astype(np.float32)
    out["ops_softmax/in_x"] = x
    out["ops_softmax/out0"] = ref.softmax(x)
    out["ops_log_softmax/in_x"] = x
    out["ops_log_softmax/out0"] = ref.softmax(x, log=True)
    for name in ["sum", "mean", "max", "min"]:
        for dim in (0, 1):
            out[f"ops_{name}_dim{dim}/in_x"] = x
            out[f"ops_{name}_dim{dim}/out0"] = ref.reduce_dim(name, x, dim)
    a = rng.standard_normal((3, 9, 11)).astype(np.float32)
    b = rng.standard_normal((3, 11, 5)).astype(np.float32)
    out["ops_batch_matmul/in_a"] = a
    out["ops_batch_matmul/in_b"] = b
    out["ops_batch_matmul/out0"] = ref.batch_matmul(a, b)
    bt = rng.standard_normal((6, 11)).astype(np.float32)
    out["ops_matmul_a_bt/in_a"] = a[0]
    out["ops_matmul_a_bt/in_bt"] = bt
    out["ops_matmul_a_bt/out0"] = ref.matmul_a_bt(a[0], bt)
    for name in ["relu", "sigmoid", "tanh", "gelu", "silu"]:
        v = (rng.standard_normal(300) * 4).astype(np.float32)
        out[f"ops_{name}/in_x"] = v
        out[f"ops_{name}/out0"] = ref.unary(name, v)
    return out


def main():
    ref = O.Reference()
    rng = np.random.default_rng(42)
    data = executor_cases(ref, rng)
    data.update(kernel_cases(ref, rng))
    np.savez_compressed(HERE / "reference_outputs.npz", **data)
    (HERE / "kats.json").write_text(json.dumps(KATS, indent=1))
    print(f"wrote {len(data)} arrays and {len(KATS)} known-answer tests")


if __name__ == "__main__":
    main()
