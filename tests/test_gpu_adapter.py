"""Graphs built by PyFlame's own C++ front end (Tensor API, nn::Linear,
Conv2d, BatchNorm2d, MaxPool2d, LayerNorm, MultiheadAttention) run through
the PyFlame-side bridge (pyflame_b200/integration/pyflame_graph_bridge.hpp)
into libpyflame_cuda.so, compared with the oracle and with PyFlame's CPU
executor (executor.cpp:236-520) in one process: the drop-in boundary as a
PyFlame maintainer would wire it."""
import subprocess

import pytest

from oracle import oracle as O

CHECK = O.HERE / "_ref" / "adapter_check"


@pytest.mark.gpu
@pytest.mark.skipif(not CHECK.exists(), reason="adapter check not built (oracle/_ref)")
def test_pyflame_front_end_through_bridge():
    r = subprocess.run([str(CHECK)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASSED" in r.stdout
