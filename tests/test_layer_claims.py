"""Placement of a whole Llama prefill layer, node by node, as llama.cpp builds it
(ggml_b200.graph.llama_layer): which nodes the claim rules give the backend with the defaults
(the reference's three ops) and with B200_GLUE=1 (every node), and the reference's short-context
rule for FLASH_ATTN_EXT (n_kv >= 1024). No GPU needed: the claim rules read descriptors only;
the knobs are read once per process, so each case runs in a child."""
import json
import os
import subprocess
import sys

from conftest import ROOT

_CHILD = r"""
import json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200")
import ggml_b200 as g
from ggml_b200.graph import llama_layer
out = {}
for n_kv in (512, 1024):
    L = llama_layer(512, n_kv=n_kv)
    out[n_kv] = {x.name.decode(): [bool(g.supports_op(x)), bool(g.offload_op(x))] for x in L.nodes}
# the same layer with storage: a bump allocator of (fake) device addresses, 256-byte aligned
top = [1 << 40]
spans = []
def alloc(n):
    a = top[0]
    top[0] += (n + 255) // 256 * 256
    spans.append((a, a + n))
    return a, True
L = llama_layer(512, n_kv=1024, alloc=alloc)
out["alloc_claims"] = all(bool(g.supports_op(x)) for x in L.nodes)
out["spans"] = spans
out["views"] = [[x.name.decode(), x.data, x.src[0].contents.data] for x in L.nodes
                if x.op in (g.OP_VIEW, g.OP_RESHAPE, g.OP_PERMUTE)]
print(json.dumps(out))
"""

VIEWS = {"Qcur_3d", "Kcur_3d", "Vcur_3d", "k_cache_view", "v_cache_view", "q", "k", "v", "kqv_out_2d"}
MATMULS = {"Qcur", "Kcur", "Vcur", "attn_out", "ffn_gate", "ffn_up", "ffn_out"}
GLUE = {"attn_norm", "attn_norm_w", "Qcur_rope", "Kcur_rope", "k_cache_cpy", "v_cache_cpy", "ffn_inp", "ffn_norm",
        "ffn_norm_w", "ffn_swiglu", "l_out"}


def claims(env):
    e = {k: v for k, v in os.environ.items() if not k.startswith("B200_")}
    e.update(env)
    p = subprocess.run([sys.executable, "-c", _CHILD, ROOT], env=e, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr[-2000:]
    return {(int(k) if k.isdigit() else k): v for k, v in json.loads(p.stdout.strip().splitlines()[-1]).items()}


def test_layer_nodes_are_all_accounted_for():
    r = claims({})
    assert set(r[1024]) == VIEWS | MATMULS | GLUE | {"kqv_out"}


def test_default_claims_are_the_references_three_ops():
    r = claims({})
    for name, (sup, off) in r[1024].items():
        if name in VIEWS:
            assert sup and not off, name
        elif name in MATMULS:
            assert sup and off, name            # MUL_MAT at 512 tokens: claimed and offloaded
        elif name == "kqv_out":
            assert sup and not off              # FLASH_ATTN_EXT: claimed, not offloaded
        else:
            assert not sup, name                # glue stays on the host's CPU backend
    assert not r[512]["kqv_out"][0]             # the reference's n_kv >= 1024 rule


def test_glue_knob_claims_every_node():
    r = claims({"B200_GLUE": "1"})
    assert all(sup for sup, _ in r[1024].values()), [n for n, (s, _) in r[1024].items() if not s]
    assert [n for n, (s, _) in r[512].items() if not s] == ["kqv_out"]
    assert not any(off for n, (_, off) in r[1024].items() if n not in MATMULS)


def test_layer_with_storage():
    """With an allocator, every tensor gets its own 256-byte aligned range, views address their
    base tensor's bytes, and the claims hold for device-resident tensors too."""
    r = claims({"B200_GLUE": "1"})
    assert r["alloc_claims"]
    spans = sorted(r["spans"])
    assert all(a % 256 == 0 for a, _ in spans)
    assert all(spans[i][1] <= spans[i + 1][0] for i in range(len(spans) - 1))
    for name, data, base in r["views"]:
        assert data == base, name               # every view here starts at its source's first byte
