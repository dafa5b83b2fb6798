"""graph_compute over HOST tensors: the staging a ggml host relies on when its tensors live in host
buffers (ggml_backend_sched hands the backend CPU-buffer tensors through supports_buft, as the
reference's plugin does, ggml-rocket.cpp:7795-7827).

A chain of claimed ops (RMS_NORM -> MUL -> MUL_MAT -> ADD, and a view of an intermediate read by a
later op) runs in one graph with every tensor in host memory, some pageable (plain malloc) and some
pinned (the backend's host buffer type). The backend copies inputs in on one stream, runs the
kernels on another and copies outputs out on a third; an output that a later op of the same graph
reads is taken from its device copy. The test checks the result of the whole chain against the
oracle composed op by op, a second call with new input values (nothing stale is reused), and a
read that straddles an earlier output and untouched bytes (the backend must land the output first).
"""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

_CHILD = r"""
import ctypes, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/ggml-rocket_b200", sys.argv[1] + "/tests"]
import numpy as np
import ggml_b200 as g
import oracle
from ggml_b200 import quants
from conftest import rel_err

be = g.Backend()
L = g.lib()
pins = []

def pinned(shape):
    n = int(np.prod(shape)) * 4
    p = L.ggml_backend_b200_host_alloc(n)
    assert p
    pins.append(p)
    return np.frombuffer((ctypes.c_uint8 * n).from_address(p), dtype=np.float32).reshape(shape)

rng = np.random.default_rng(31)
E, N, T = 1024, 768, 96
w_norm = rng.standard_normal(E).astype(np.float32)
wq = quants.quantize(g.Q4_K, (rng.standard_normal((N, E)) * 0.02).astype(np.float32))
x = np.empty((T, E), np.float32)                  # pageable
h1 = np.empty((T, E), np.float32)                 # pageable
h2 = pinned((T, E))                               # pinned
y = np.empty((T, N), np.float32)                  # pageable
res = pinned((T, N))
z = pinned((T, N))                                # pinned

tx = g.make_tensor(g.F32, [E, T], x.ctypes.data, name="x")
tw = g.make_tensor(g.F32, [E], w_norm.ctypes.data, name="norm.weight")
tq = g.make_tensor(g.Q4_K, [E, N], wq.ctypes.data, name="proj.weight")
tres = g.make_tensor(g.F32, [N, T], res.ctypes.data, name="residual")
t1 = g.make_tensor(g.F32, [E, T], h1.ctypes.data, op=g.OP_RMS_NORM, srcs=[tx], op_params=[1e-5], name="norm")
t2 = g.make_tensor(g.F32, [E, T], h2.ctypes.data, op=g.OP_MUL, srcs=[t1, tw], name="norm_w")
t3 = g.make_tensor(g.F32, [N, T], y.ctypes.data, op=g.OP_MUL_MAT, srcs=[tq, t2], name="proj")
t4 = g.make_tensor(g.F32, [N, T], z.ctypes.data, op=g.OP_ADD, srcs=[t3, tres], name="out")
nodes = [t1, t2, t3, t4]
for nd in nodes:
    assert g.supports_op(nd), nd.op

worst = 0.0
for call in range(2):
    x[:] = rng.standard_normal((T, E)).astype(np.float32) * (1 + call)
    res[:] = rng.standard_normal((T, N)).astype(np.float32)
    assert be.graph_compute(nodes) == g.STATUS_SUCCESS
    r1 = oracle.rms_norm(x, 1e-5)
    r2 = r1 * w_norm[None, :]
    r3 = oracle.mul_mat(g.Q4_K, wq, N, E, r2)
    r4 = r3 + res
    # every intermediate landed in its host tensor too
    assert rel_err(h1, r1) <= 1e-5 and rel_err(h2, r2) <= 1e-5
    worst = max(worst, rel_err(y, r3), rel_err(z, r4))
print("CHAIN", worst)

# a read that straddles an earlier output of the graph and bytes no op wrote: ADD over a view that
# starts in the second half of h1 (written by RMS_NORM) and runs into the tensor placed after it
big = np.zeros((2 * T, E), np.float32)             # rows [0, T) written by the graph, [T, 2T) host data
big[T:] = rng.standard_normal((T, E)).astype(np.float32)
x[:] = rng.standard_normal((T, E)).astype(np.float32)
half = T // 2
tn = g.make_tensor(g.F32, [E, T], big.ctypes.data, op=g.OP_RMS_NORM, srcs=[tx], op_params=[1e-5], name="norm2")
tv = g.make_tensor(g.F32, [E, T], big.ctypes.data + half * E * 4, op=g.OP_VIEW, srcs=[tn], name="straddle")
out2 = np.empty((T, E), np.float32)
ta = g.make_tensor(g.F32, [E, T], out2.ctypes.data, op=g.OP_ADD, srcs=[tv, tw], name="straddle_add")
assert be.graph_compute([tn, tv, ta]) == g.STATUS_SUCCESS
rn = oracle.rms_norm(x, 1e-5)
want = np.concatenate([rn[half:], big[T:T + half]]) + w_norm[None, :]
print("STRADDLE", rel_err(out2, want))
assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
for p in pins:
    L.ggml_backend_b200_host_free(p)
be.close()
"""


def test_host_tensor_chain_through_graph_compute(cuda):
    env = dict(os.environ, B200_GLUE="1")
    p = subprocess.run([sys.executable, "-c", _CHILD, ROOT], env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    chain = float(p.stdout.split("CHAIN")[1].split()[0])
    straddle = float(p.stdout.split("STRADDLE")[1].split()[0])
    assert chain <= 1e-2, chain
    assert straddle <= 1e-5, straddle
