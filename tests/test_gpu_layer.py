"""A whole dense Llama prefill layer executed through graph_compute, against the oracle composed op
by op.

ggml_b200.graph.llama_layer builds the layer's nodes the way llama.cpp does (attention norm, Q/K/V,
normal-mode RoPE, the f16 K/V cache writes, FLASH_ATTN_EXT on the cache views, output projection,
residual, FFN norm, gate/up, SWIGLU, down, residual). With B200_GLUE=1 every node is claimed; the
tensors live in one device buffer, so the layer runs on the GPU from its input embedding to its
output with no host copy in between. The oracle composes the same layer from its CPU restatements:
rms_norm, rope, the fp64 MUL_MAT over the Q4_K-decoded weights and the fp64 attention over the f16
caches. The tolerance is the north star's end-to-end bar (cosine >= 0.999) and the op bar
(max |err| / max |ref| <= 1e-2) on the layer output. Dimensions are a reduced Llama (hidden 1024,
FFN 2816, 8 query / 2 KV heads of 128) so the fp64 oracle finishes in seconds; bench.py --workload
layer runs the Llama-3-8B dimensions.
"""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

_CHILD = r"""
import sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/ggml-rocket_b200", sys.argv[1] + "/tests"]
import numpy as np
import ggml_b200 as g
import oracle
from ggml_b200 import quants
from ggml_b200.graph import llama_layer
from conftest import rel_err, rk_compare

T, E, F, H, HK, D, n_kv = 512, 1024, 2816, 8, 2, 128, 1024
eps, base = 1e-5, 500000.0
be = g.Backend()
buf = g.DeviceBuffer(be, 256 << 20)
top = [0]
def alloc(n):
    off = top[0]
    top[0] += (n + 255) // 256 * 256
    assert top[0] <= buf.size
    return buf.base + off, True
L = llama_layer(T, E=E, F=F, H=H, HK=HK, D=D, n_kv=n_kv, wtype=g.Q4_K, eps=eps, rope_base=base, alloc=alloc)
for nd in L.nodes:
    assert g.supports_op(nd), nd.name
off = lambda t: t.data - buf.base
rng = np.random.default_rng(0x1A7E)
x = rng.standard_normal((T, E), dtype=np.float32)
pos = np.arange(T, dtype=np.int32)
Tp = L.inputs["mask"].ne[1]
mask = np.full((Tp, n_kv), -np.inf, np.float32)
for t in range(T):
    mask[t, :t + 1] = 0.0
m16 = mask.astype(np.float16)
assert buf.set(off(L.inputs["x"]), x) == 0
assert buf.set(off(L.inputs["pos"]), pos) == 0
assert buf.set(off(L.inputs["mask"]), m16.view(np.uint16)) == 0
for c in L.caches.values():
    assert buf.set(off(c), np.zeros(c.ne[0] * c.ne[1], np.uint16)) == 0
W = {}
for name, t in L.weights.items():
    if t.type == g.F32:
        W[name] = (1.0 + 0.1 * rng.standard_normal(t.ne[0])).astype(np.float32)
        assert buf.set(off(t), W[name]) == 0
    else:
        W[name] = quants.quantize(g.Q4_K, (rng.standard_normal((t.ne[1], t.ne[0])) * 0.02).astype(np.float32))
        assert buf.set(off(t), W[name]) == 0
assert be.graph_compute(L.nodes) == g.STATUS_SUCCESS
got = np.zeros((T, E), np.float32)
assert buf.get(off(L.out), got) == 0

# the oracle, op by op
def mm(name, a):
    t = L.weights[name]
    return oracle.mul_mat(g.Q4_K, W[name], t.ne[1], t.ne[0], a)
an = oracle.rms_norm(x, eps) * W["attn_norm"][None, :]
q = mm("attn_q", an).reshape(T, H, D)
k = mm("attn_k", an).reshape(T, HK, D)
v = mm("attn_v", an).reshape(T, HK, D)
qr = oracle.rope(q, pos, D, 0, base)
kr = oracle.rope(k, pos, D, 0, base)
k16 = np.zeros((HK, n_kv, D), np.float16)
v16 = np.zeros((HK, n_kv, D), np.float16)
k16[:, :T] = np.transpose(kr, (1, 0, 2)).astype(np.float16)
v16[:, :T] = np.transpose(v, (1, 0, 2)).astype(np.float16)
att = oracle.flash_attn(np.ascontiguousarray(np.transpose(qr, (1, 0, 2))), k16.view(np.uint16), v16.view(np.uint16),
                        m16[:T].view(np.uint16), 1.0 / np.sqrt(D), q_mode=1)
h = mm("attn_output", att.reshape(T, E)) + x
fn = oracle.rms_norm(h, eps) * W["ffn_norm"][None, :]
act = oracle.swiglu(mm("ffn_gate", fn), mm("ffn_up", fn))
want = mm("ffn_down", act) + h
cos, bad = rk_compare(want, got)
print("LAYER", rel_err(got, want), cos, bad)
assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
print("ROUTES", be.route_ops("fa"), be.route_ops("glue"), be.route_ops(None), be.route_ops("fused"),
      be.route_ops("swiglu_fused"), be.route_ops("norm_pack"), be.route_ops("rope_cpy"))
buf.free()
be.close()
"""


def test_llama_layer_through_graph_compute(cuda):
    env = {k: v for k, v in os.environ.items() if not k.startswith("B200_")}
    env["B200_GLUE"] = "1"
    p = subprocess.run([sys.executable, "-c", _CHILD, ROOT], env=env, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    rel, cos, bad = [float(v) for v in p.stdout.split("LAYER")[1].split()[:3]]
    assert rel <= 1e-2, rel
    assert cos >= 0.999, cos
    assert bad == 0
    fa, glue, total, groups, swiglu_fused, norm_pack, rope_cpy = [int(v) for v in
                                                                  p.stdout.split("ROUTES")[1].split()[:7]]
    assert fa == 1 and glue >= 11
    # Q/K/V and gate/up each ran as one combined-N GEMM whose activation pack the norm in front of it
    # made; SWIGLU ran inside the down projection's pack; K's ROPE wrote the fp16 cache rows directly
    assert groups == 2 and swiglu_fused == 1 and norm_pack == 2 and rope_cpy == 1
