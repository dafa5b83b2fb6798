"""The ggml adapter's converter (ggml_backend_b200_builder_*), on the CPU.

A ggml host's adapter declares each tensor of a split with its fields and ggml's op NAMES; the
builder maps them to descriptors. The tests drive it the way the adapter does -- a whole Llama
prefill layer (ggml_b200.graph.llama_layer) re-declared source-first with the names ggml_op_name /
ggml_unary_op_name / ggml_glu_op_name return -- and check that the converted nodes are claimed
exactly like the originals, that shared sources stay shared (the QKV and gate/up groups), the
sub-op translation, unknown ops, and the declaration-order rule. The claim rules read descriptors
only, so no GPU is needed; knobs are read once per process, so each case runs in a child.
"""
import json
import os
import subprocess
import sys

from conftest import ROOT

_CHILD = r"""
import ctypes, json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200")
import ggml_b200 as g
from ggml_b200.graph import llama_layer

NAMES = {g.OP_NONE: "NONE", g.OP_RESHAPE: "RESHAPE", g.OP_VIEW: "VIEW", g.OP_PERMUTE: "PERMUTE",
         g.OP_TRANSPOSE: "TRANSPOSE", g.OP_MUL_MAT: "MUL_MAT", g.OP_MUL_MAT_ID: "MUL_MAT_ID",
         g.OP_FLASH_ATTN_EXT: "FLASH_ATTN_EXT", g.OP_RMS_NORM: "RMS_NORM", g.OP_ADD: "ADD", g.OP_MUL: "MUL",
         g.OP_UNARY: "UNARY", g.OP_GLU: "GLU", g.OP_ROPE: "ROPE", g.OP_GET_ROWS: "GET_ROWS", g.OP_CPY: "CPY"}
out = {}
L = llama_layer(512, n_kv=1024)
b = g.GraphBuilder()
keys = {}            # address of an original descriptor -> a host "tensor pointer" (the key)

def key_of(t):
    return keys.setdefault(ctypes.addressof(t), 0x1000 + 64 * len(keys))

def declare(t):
    k = key_of(t)
    if b.find(k) is not None:
        return k
    srcs = []
    for i in range(10):
        if t.src[i]:
            srcs.append(declare(t.src[i].contents))
        else:
            srcs.append(None)
    subop = None
    opp = list(t.op_params)
    if t.op == g.OP_GLU:
        subop = "SWIGLU"
        opp[0] = 7          # the host's own GLU enum value: the builder must replace it
    d = b.add(k, NAMES[t.op], t.type, list(t.ne), list(t.nb), op_params=opp, src_keys=srcs, data=t.data,
              on_device=bool(t.on_device), readable=bool(t.readable), name=t.name.decode(), subop_name=subop)
    assert d is not None
    return k

for nd in L.nodes:
    b.push(declare(nd))
conv = b.nodes()
out["n"] = [len(L.nodes), len(conv)]
out["claims_equal"] = all(bool(g.supports_op(a)) == bool(g.supports_op(c)) and
                          bool(g.offload_op(a)) == bool(g.offload_op(c)) for a, c in zip(L.nodes, conv))
out["names"] = [c.name.decode() for c in conv] == [a.name.decode() for a in L.nodes]
by = {c.name.decode(): c for c in conv}
src1 = lambda n: ctypes.addressof(by[n].src[1].contents)
out["qkv_shared"] = src1("Qcur") == src1("Kcur") == src1("Vcur")
out["gate_up_shared"] = src1("ffn_gate") == src1("ffn_up")
out["glu_subop"] = [by["ffn_swiglu"].op, by["ffn_swiglu"].op_params[0], by["ffn_swiglu"].op_params[1]]
# unknown op, unknown UNARY sub-op, undeclared source, repeated key
u = b.add(0x99990, "CONV_2D", g.F32, [8, 8], [4, 32, 256, 256])
out["unknown_op"] = [u.op, bool(g.supports_op(u))]
s = b.add(0x99a00, "UNARY", g.F32, [8, 8], [4, 32, 256, 256], op_params=[3], src_keys=[0x99990], subop_name="SILU")
gl = b.add(0x99a40, "UNARY", g.F32, [8, 8], [4, 32, 256, 256], op_params=[3], src_keys=[0x99990], subop_name="GELU")
out["unary"] = [s.op_params[0], gl.op_params[0]]
out["undeclared_src"] = b.add(0x99b00, "ADD", g.F32, [8], [4, 32, 32, 32], src_keys=[0x12345]) is None
again = b.add(0x99990, "ADD", g.F32, [4], [4, 16, 16, 16])
out["same_key_same_desc"] = ctypes.addressof(again) == ctypes.addressof(u)
out["push_undeclared"] = b.push(0x77777)
b.close()
print(json.dumps(out))
"""


def run(env):
    e = {k: v for k, v in os.environ.items() if not k.startswith("B200_")}
    e.update(env)
    p = subprocess.run([sys.executable, "-c", _CHILD, ROOT], env=e, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr[-3000:]
    return json.loads(p.stdout.strip().splitlines()[-1])


def test_converted_layer_claims_like_the_original():
    for env in ({}, {"B200_GLUE": "1"}):
        r = run(env)
        assert r["n"][0] == r["n"][1]
        assert r["claims_equal"] and r["names"]


def test_shared_sources_and_subops():
    r = run({"B200_GLUE": "1"})
    assert r["qkv_shared"] and r["gate_up_shared"]
    import ggml_b200 as g
    assert r["glu_subop"] == [g.OP_GLU, g.GLU_SWIGLU, 0]     # the host's enum value replaced, not swapped
    assert r["unknown_op"] == [g.OP_OTHER, False]            # never claimed
    assert r["unary"] == [g.UNARY_SILU, -1]                  # SILU translated, GELU unknown
    assert r["undeclared_src"] and r["same_key_same_desc"]
    assert r["push_undeclared"] == -1
