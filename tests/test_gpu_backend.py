"""The backend layer on the GPU: graph_compute over host tensors, as a ggml host drives it.

Mirrors the reference's gates: every op it claims runs on the device (route counters, zero CPU
fallbacks -- test-common.h:160-177), fused shared-src1 groups (test-rocket-matmul.cpp:261-314),
"same name, new bytes" cache identity (:223-259), batch broadcast, FLASH_ATTN_EXT and
MUL_MAT_ID through graph_compute, and a malformed MUL_MAT_ID failing the graph.
"""
import math

import numpy as np
import pytest

import ggml_b200 as g
import oracle
from conftest import rel_err
from ggml_b200 import quants

pytestmark = pytest.mark.gpu


def weight(rng, t, N, K, name, scale=0.02):
    raw = quants.quantize(t, (rng.standard_normal((N, K)) * scale).astype(np.float32))
    return raw, g.make_tensor(t, [K, N], raw, name=name)


def test_backend_mul_mat_routes_and_parity(cuda):
    be = g.Backend()
    rng = np.random.default_rng(1)
    K, N, M = 1024, 512, 96
    nodes, keep = [], []
    for t in (g.F16, g.Q8_0, g.Q4_K, g.Q6_K):
        raw, w = weight(rng, t, N, K, f"w.{t}")
        a = rng.standard_normal((M, K)).astype(np.float32)
        x = g.make_tensor(g.F32, [K, M], a, name="x")
        out = np.full((M, N), np.nan, np.float32)
        d = g.make_tensor(g.F32, [N, M], out, op=g.OP_MUL_MAT, srcs=[w, x], name="mm")
        keep.append((raw, a, out, w, x, d, t))
        nodes.append(d)
    assert be.graph_compute(nodes) == g.STATUS_SUCCESS
    for raw, a, out, w, x, d, t in keep:
        assert rel_err(out, oracle.mul_mat(t, raw, N, K, a)) <= 1e-2
    assert be.route_ops("f16") == 1 and be.route_ops("q8_0") == 1
    assert be.route_ops("q4_K") == 1 and be.route_ops("q6_K") == 1
    assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
    be.close()


def test_backend_fused_groups(cuda):
    """QKV (unequal N, GQA) and gate/up (equal N) share src1 -> one fused group each."""
    be = g.Backend()
    rng = np.random.default_rng(2)
    K, M = 3840, 128
    for Ns in ((4096, 1024, 1024), (2048, 2048)):
        a = rng.standard_normal((M, K)).astype(np.float32)
        x = g.make_tensor(g.F32, [K, M], a, name="attn_norm")
        ws, outs, nodes = [], [], []
        for i, N in enumerate(Ns):
            raw, w = weight(rng, g.F16, N, K, f"blk.0.w{i}.{len(Ns)}")
            out = np.full((M, N), np.nan, np.float32)
            nodes.append(g.make_tensor(g.F32, [N, M], out, op=g.OP_MUL_MAT, srcs=[w, x]))
            ws.append((raw, w))
            outs.append(out)
        before = be.route_ops("fused")
        assert be.graph_compute(nodes) == g.STATUS_SUCCESS
        assert be.route_ops("fused") == before + 1
        for (raw, _), out, N in zip(ws, outs, Ns):
            assert rel_err(out, oracle.mul_mat(g.F16, raw, N, K, a)) <= 1e-2
    be.close()


def test_backend_same_name_new_bytes(cuda):
    """A weight whose bytes change under the same name must not be served from the cache."""
    be = g.Backend()
    rng = np.random.default_rng(3)
    K, N, M = 512, 256, 64
    a = rng.standard_normal((M, K)).astype(np.float32)
    for rep in range(2):
        raw, w = weight(rng, g.Q4_K, N, K, "blk.7.ffn_up.weight")
        x = g.make_tensor(g.F32, [K, M], a)
        out = np.zeros((M, N), np.float32)
        d = g.make_tensor(g.F32, [N, M], out, op=g.OP_MUL_MAT, srcs=[w, x])
        assert be.graph_compute([d]) == g.STATUS_SUCCESS
        assert rel_err(out, oracle.mul_mat(g.Q4_K, raw, N, K, a)) <= 1e-2
    assert be.weight_cache()[1] == 2
    be.close()


def test_backend_batch_broadcast(cuda):
    """src1 [K, M, 3, 2] against a 2-D weight (r2 = 3, r3 = 2)."""
    be = g.Backend()
    rng = np.random.default_rng(4)
    K, N, M = 256, 128, 40
    raw, w = weight(rng, g.Q8_0, N, K, "w.bcast")
    a = rng.standard_normal((2, 3, M, K)).astype(np.float32)
    x = g.make_tensor(g.F32, [K, M, 3, 2], a)
    out = np.zeros((2, 3, M, N), np.float32)
    d = g.make_tensor(g.F32, [N, M, 3, 2], out, op=g.OP_MUL_MAT, srcs=[w, x])
    assert be.graph_compute([d]) == g.STATUS_SUCCESS
    for i3 in range(2):
        for i2 in range(3):
            assert rel_err(out[i3, i2], oracle.mul_mat(g.Q8_0, raw, N, K, a[i3, i2])) <= 1e-2
    be.close()


def test_backend_flash_attn(cuda):
    be = g.Backend()
    rng = np.random.default_rng(5)
    H, HK, D, T, KV = 8, 2, 128, 64, 1024
    Q = rng.standard_normal((H, T, D)).astype(np.float32)
    K16 = rng.standard_normal((HK, KV, D)).astype(np.float16).view(np.uint16)
    V16 = rng.standard_normal((HK, KV, D)).astype(np.float16).view(np.uint16)
    M = np.zeros((T, KV), np.float32)
    for t in range(T):
        M[t, KV - T + t + 1:] = -np.inf
    M16 = M.astype(np.float16).view(np.uint16)
    q = g.make_tensor(g.F32, [D, T, H], Q)
    k = g.make_tensor(g.F16, [D, KV, HK], K16)
    v = g.make_tensor(g.F16, [D, KV, HK], V16)
    m = g.make_tensor(g.F16, [KV, T], M16)
    out = np.full((T, H, D), np.nan, np.float32)
    scale = 1.0 / math.sqrt(D)
    d = g.make_tensor(g.F32, [D, H, T], out, op=g.OP_FLASH_ATTN_EXT, srcs=[q, k, v, m],
                      op_params=[scale, 0.0, 0.0])
    assert g.supports_op(d)
    assert be.graph_compute([d]) == g.STATUS_SUCCESS
    want = oracle.flash_attn(Q, K16, V16, M16, scale, q_mode=2)
    assert rel_err(out, want) <= 1e-2
    assert be.route_ops("fa") == 1 and be.cpu_fallbacks() == 0
    be.close()


def test_backend_mul_mat_id_and_bad_ids(cuda):
    be = g.Backend()
    rng = np.random.default_rng(6)
    K, N, n_expert, n_tokens, n_used = 512, 256, 16, 64, 4
    raw = quants.quantize(g.Q4_K, (rng.standard_normal((n_expert * N, K)) * 0.02).astype(np.float32))
    as_t = g.make_tensor(g.Q4_K, [K, N, n_expert], raw, name="blk.0.ffn_up_exps.weight")
    b = rng.standard_normal((n_tokens, 1, K)).astype(np.float32)
    bt = g.make_tensor(g.F32, [K, 1, n_tokens], b)
    ids = np.stack([rng.permutation(n_expert)[:n_used] for _ in range(n_tokens)]).astype(np.int32)
    it = g.make_tensor(g.I32, [n_used, n_tokens], ids)
    out = np.full((n_tokens, n_used, N), np.nan, np.float32)
    d = g.make_tensor(g.F32, [N, n_used, n_tokens], out, op=g.OP_MUL_MAT_ID, srcs=[as_t, bt, it])
    assert g.supports_op(d)
    assert be.graph_compute([d]) == g.STATUS_SUCCESS
    want = oracle.mul_mat_id(g.Q4_K, raw.reshape(n_expert, N, -1), K, N, n_expert, b, ids)
    assert rel_err(out, want) <= 1e-2
    assert be.route_ops("moe") == 1
    assert be.moe_stats() == (1, 0)
    orig = int(ids[3, 2])
    ids[3, 2] = -1
    assert be.graph_compute([d]) == g.STATUS_FAILED
    # the backend stays usable after the failed op
    ids[3, 2] = orig
    assert be.graph_compute([d]) == g.STATUS_SUCCESS
    assert rel_err(out, want) <= 1e-2
    be.close()


def test_backend_groups_mul_mat_ids_sharing_inputs(cuda):
    """A MoE layer's gate and up (two MUL_MAT_ID nodes on the same b and ids) run as one group:
    one route and gather-pack, one grouped GEMM per stack; each result matches the oracle."""
    be = g.Backend()
    rng = np.random.default_rng(8)
    K, N, n_expert, n_tokens, n_used = 512, 128, 16, 96, 4
    b = rng.standard_normal((n_tokens, 1, K)).astype(np.float32)
    bt = g.make_tensor(g.F32, [K, 1, n_tokens], b)
    ids = np.stack([rng.permutation(n_expert)[:n_used] for _ in range(n_tokens)]).astype(np.int32)
    it = g.make_tensor(g.I32, [n_used, n_tokens], ids)
    nodes, outs, raws = [], [], []
    for name in ("blk.0.ffn_gate_exps.weight", "blk.0.ffn_up_exps.weight"):
        raw = quants.quantize(g.Q4_K, (rng.standard_normal((n_expert * N, K)) * 0.02).astype(np.float32))
        as_t = g.make_tensor(g.Q4_K, [K, N, n_expert], raw, name=name)
        out = np.full((n_tokens, n_used, N), np.nan, np.float32)
        nodes.append(g.make_tensor(g.F32, [N, n_used, n_tokens], out, op=g.OP_MUL_MAT_ID, srcs=[as_t, bt, it]))
        outs.append(out)
        raws.append(raw)
    assert be.graph_compute(nodes) == g.STATUS_SUCCESS
    for out, raw in zip(outs, raws):
        want = oracle.mul_mat_id(g.Q4_K, raw.reshape(n_expert, N, -1), K, N, n_expert, b, ids)
        assert rel_err(out, want) <= 1e-2
    assert be.route_ops("moe") == 2 and be.route_ops("moe_grouped") == 2
    be.close()


_DECODE_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
import ggml_b200 as g
import oracle
from conftest import rel_err
from ggml_b200 import quants
be = g.Backend()
rng = np.random.default_rng(7)
K = 4096
worst, n = 0.0, 0
Q4, Q6, Q8 = g.Q4_K, g.Q6_K, g.Q8_0
for M, Ws in ((1, ((Q4, 4096),)), (4, ((Q4, 4096), (Q8, 1024), (Q6, 1024))), (8, ((Q4, 14336), (Q4, 14336))),
              (12, ((Q6, 4096), (Q8, 2048), (Q4, 1024)))):
    a = rng.standard_normal((M, K)).astype(np.float32)
    x = g.make_tensor(g.F32, [K, M], a, name="x")
    keep, nodes = [], []
    for i, (t, N) in enumerate(Ws):
        raw = quants.quantize(t, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        w = g.make_tensor(t, [K, N], raw, name=f"blk.{M}.w{i}")
        out = np.full((M, N), np.nan, np.float32)
        d = g.make_tensor(g.F32, [N, M], out, op=g.OP_MUL_MAT, srcs=[w, x])
        assert g.supports_op(d)
        keep.append((t, raw, w, out, d, N))
        nodes.append(d)
    assert be.graph_compute(nodes) == g.STATUS_SUCCESS
    for t, raw, w, out, d, N in keep:
        e = rel_err(out, oracle.mul_mat(t, raw, N, K, a))
        print("CASE", t, M, N, e)
        worst = max(worst, e)
    n += len(Ws)
assert be.route_ops("decode") == n, be.route_ops("decode")
assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
be.close()
print("DECODE_WORST", worst)
"""


def test_backend_decode_route(cuda):
    """B200_DECODE=1 (read once per process, so in a child): Q4_K / Q6_K / Q8_0 MUL_MATs below the
    floor (M = 1, 4, 8, 12) -- one op, and shared-src1 groups mixing the types -- run on the
    weight-streaming kernels through graph_compute,
    within the decode kernel's bound against the oracle (fp16 activations, exact weights)."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, B200_DECODE="1")
    p = subprocess.run([sys.executable, "-c", _DECODE_CHILD, ROOT], env=env, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert float(p.stdout.split("DECODE_WORST")[1].split()[0]) <= 2e-3, p.stdout   # the decode kernel's bound
