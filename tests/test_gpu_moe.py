"""MUL_MAT_ID parity on the GPU through b200_mul_mat_id, against the CPU oracle.

Mirrors test-rocket-moe.cpp: ne11 = 1 and ne11 = n_used forms, 16/4-style routing, skewed ids
that leave experts empty (:160-166), several weight formats (:200-219), and a malformed id
(the reference returns 1 -> GGML_STATUS_FAILED, ggml-rocket.cpp:6719). The route arrays the
kernels leave in the workspace must equal the CPU counting sort exactly.
"""
import numpy as np
import pytest

import oracle
from conftest import rel_err
from ggml_b200 import quants

pytestmark = pytest.mark.gpu


def run_moe(torch, wtype, ws_native, K, N, n_expert, b, ids, expect_rc=0):
    """ws_native uint8 [n_expert*N, row]; b f32 [n_tokens, ne11, K]; ids int32 [n_tokens, n_used]."""
    import ggml_b200 as g
    n_tokens, ne11, _ = b.shape
    n_used = ids.shape[1]
    raw = torch.from_numpy(np.ascontiguousarray(ws_native).reshape(-1)).cuda()
    packed = torch.empty(g.weight_packed_size(wtype, N * n_expert, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(wtype, raw, N * n_expert, K, packed)
    bd = torch.from_numpy(np.ascontiguousarray(b)).cuda()
    idd = torch.from_numpy(np.ascontiguousarray(ids)).cuda()
    dst = torch.full((n_tokens, n_used, N), float("nan"), dtype=torch.float32, device="cuda")
    ws = torch.zeros(g.mul_mat_id_workspace_size(K, N, n_expert, n_used, n_tokens), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = g.mul_mat_id(wtype, packed, K, N, n_expert, bd, K * 4, ne11 * K * 4, ne11, idd, 4, n_used * 4, n_used,
                      n_tokens, dst, N * 4, n_used * N * 4, ws, err)
    torch.cuda.synchronize()
    assert rc == expect_rc
    o, s, t = g.mul_mat_id_route_view(K, n_expert, n_used, n_tokens)
    wsn = ws.cpu().numpy()
    R = n_tokens * n_used
    route = (wsn[o:o + 4 * (n_expert + 1)].view(np.int32), wsn[s:s + 4 * R].view(np.int32),
             wsn[t:t + 4 * R].view(np.int32))
    return dst.cpu().numpy(), int(err.item()), route


def make_case(rng, wtype, K, N, n_expert, n_tokens, n_used, ne11, skew=False):
    w = (rng.standard_normal((n_expert * N, K)) * 0.02).astype(np.float32)
    ws_native = quants.quantize(wtype, w) if wtype != 1 else w.astype(np.float16).view(np.uint8).reshape(n_expert * N, -1)
    b = rng.standard_normal((n_tokens, ne11, K)).astype(np.float32)
    if skew:
        # concentrate on the low experts; the last ones get nothing
        p = np.exp(-np.arange(n_expert) / 2.0)
        p[-2:] = 0
        p /= p.sum()
        ids = np.stack([rng.choice(n_expert, n_used, replace=False, p=p) for _ in range(n_tokens)])
    else:
        ids = np.stack([rng.permutation(n_expert)[:n_used] for _ in range(n_tokens)])
    return ws_native, b, ids.astype(np.int32)


@pytest.mark.parametrize("wtype,K,N,n_expert,n_tokens,n_used,ne11,skew", [
    (12, 256, 128, 16, 64, 4, 1, False),
    (12, 256, 128, 16, 64, 4, 4, False),
    (12, 512, 256, 16, 100, 4, 1, True),
    (8, 256, 64, 8, 33, 2, 2, False),
    (14, 512, 128, 8, 70, 3, 1, True),
    (1, 256, 96, 8, 48, 2, 1, False),
    (12, 2048, 768, 32, 256, 8, 1, False),
    (12, 768, 2048, 32, 256, 8, 8, False),
    (12, 512, 256, 8, 200, 4, 1, False),     # ~100 rows per expert: the 256-token tile
    (14, 512, 128, 8, 300, 4, 4, True),
])
def test_moe_matches_oracle(cuda, wtype, K, N, n_expert, n_tokens, n_used, ne11, skew):
    import torch
    rng = np.random.default_rng(K + N + n_expert * 7 + n_tokens + ne11 + wtype)
    ws_native, b, ids = make_case(rng, wtype, K, N, n_expert, n_tokens, n_used, ne11, skew)
    got, err, route = run_moe(torch, wtype, ws_native, K, N, n_expert, b, ids)
    assert err == 0
    off, slot, tok = oracle.moe_route(ids, n_expert)
    assert np.array_equal(route[0], off)
    assert np.array_equal(route[1], slot)
    assert np.array_equal(route[2], tok)
    want = oracle.mul_mat_id(wtype, ws_native.reshape(n_expert, N, -1), K, N, n_expert, b, ids)
    assert np.all(np.isfinite(got))
    assert rel_err(got, want) <= 1e-2


def test_moe_bad_id_is_reported(cuda):
    import torch
    rng = np.random.default_rng(5)
    ws_native, b, ids = make_case(rng, 12, 256, 64, 8, 20, 2, 1)
    ids[7, 1] = 8
    got, err, route = run_moe(torch, 12, ws_native, 256, 64, 8, b, ids)
    assert err == 100                     # B200_DEV_BAD_IDS
    assert np.all(np.isnan(got))          # nothing written


@pytest.mark.parametrize("wtype,K,Ns,n_expert,n_tokens,n_used,ne11", [
    (12, 2048, (768, 768), 32, 256, 8, 1),      # a MoE layer's gate and up
    (12, 512, (256, 128, 64), 16, 100, 4, 4),   # three members, different N, per-slot b rows
    (14, 512, (128,), 8, 70, 3, 1),             # one member: the plain op
])
def test_moe_group_equals_members(cuda, wtype, K, Ns, n_expert, n_tokens, n_used, ne11):
    """b200_mul_mat_id_group (one route and gather-pack for stacks sharing b and ids) gives every
    member exactly its own b200_mul_mat_id result: the same sorted rows, the same kernels."""
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(5 + wtype + len(Ns))
    _, b, ids = make_case(rng, wtype, K, Ns[0], n_expert, n_tokens, n_used, ne11)
    bd = torch.from_numpy(np.ascontiguousarray(b)).cuda()
    idd = torch.from_numpy(np.ascontiguousarray(ids)).cuda()
    stacks, dsts, wants = [], [], []
    for m, N in enumerate(Ns):
        w = (rng.standard_normal((n_expert * N, K)) * 0.02).astype(np.float32)
        native = quants.quantize(wtype, w)
        raw = torch.from_numpy(np.ascontiguousarray(native).reshape(-1)).cuda()
        packed = torch.empty(g.weight_packed_size(wtype, N * n_expert, K), dtype=torch.uint8, device="cuda")
        g.weight_pack(wtype, raw, N * n_expert, K, packed)
        stacks.append(packed)
        dsts.append(torch.full((n_tokens, n_used, N), float("nan"), dtype=torch.float32, device="cuda"))
        want, err, _ = run_moe(torch, wtype, native, K, N, n_expert, b, ids)
        assert err == 0
        wants.append(want)
    ws = torch.zeros(max(g.mul_mat_id_workspace_size(K, N, n_expert, n_used, n_tokens) for N in Ns),
                     dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = g.mul_mat_id_group(wtype, stacks, list(Ns), K, n_expert, bd, K * 4, ne11 * K * 4, ne11, idd, 4, n_used * 4,
                            n_used, n_tokens, dsts, [N * 4 for N in Ns], [n_used * N * 4 for N in Ns], ws, err)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    for d, want in zip(dsts, wants):
        got = d.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def _packed(torch, g, wtype, native, rows, K):
    raw = torch.from_numpy(np.ascontiguousarray(native).reshape(-1)).cuda()
    out = torch.empty(g.weight_packed_size(wtype, rows, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(wtype, raw, rows, K, out)
    return out


def _native(rng, wtype, rows, K):
    w = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
    return quants.quantize(wtype, w) if wtype != 1 else w.astype(np.float16).view(np.uint8).reshape(rows, -1)


def _ffn_case(torch, g, wt_gu, wt_d, H, F, E, T, n_used, seed, skew=False):
    rng = np.random.default_rng(seed)
    nat = {"gate": _native(rng, wt_gu, E * F, H), "up": _native(rng, wt_gu, E * F, H), "down": _native(rng, wt_d, E * H, F)}
    x = rng.standard_normal((T, 1, H)).astype(np.float32)
    if skew:
        p = np.exp(-np.arange(E) / 2.0)
        p[-2:] = 0
        p /= p.sum()
        ids = np.stack([rng.choice(E, n_used, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    else:
        ids = np.stack([rng.permutation(E)[:n_used] for _ in range(T)]).astype(np.int32)
    pk = {"gate": _packed(torch, g, wt_gu, nat["gate"], E * F, H), "up": _packed(torch, g, wt_gu, nat["up"], E * F, H),
          "down": _packed(torch, g, wt_d, nat["down"], E * H, F)}
    return nat, pk, x, ids


def _ffn_chain(torch, g, wt_gu, wt_d, pk, H, F, E, xd, idd, err):
    """gate / up MUL_MAT_ID group, SWIGLU, down MUL_MAT_ID: the ops the fused call replaces."""
    T, n_used = idd.shape
    yg = torch.empty((T, n_used, F), device="cuda")
    yu = torch.empty_like(yg)
    h = torch.empty_like(yg)
    out = torch.full((T, n_used, H), float("nan"), device="cuda")
    ws = torch.zeros(max(g.mul_mat_id_workspace_size(H, F, E, n_used, T), g.mul_mat_id_workspace_size(F, H, E, n_used, T)),
                     dtype=torch.uint8, device="cuda")
    assert g.mul_mat_id_group(wt_gu, [pk["gate"], pk["up"]], [F, F], H, E, xd, H * 4, H * 4, 1, idd, 4, n_used * 4,
                              n_used, T, [yg, yu], [F * 4, F * 4], [n_used * F * 4] * 2, ws, err) == 0
    assert g.swiglu(yg, yu, h) == 0
    assert g.mul_mat_id(wt_d, pk["down"], F, H, E, h, F * 4, n_used * F * 4, n_used, idd, 4, n_used * 4, n_used, T,
                        out, H * 4, n_used * H * 4, ws, err) == 0
    return out


def _ffn_fused(torch, g, wt_gu, wt_d, pk, H, F, E, xd, idd, err, d_pad=0):
    T, n_used = idd.shape
    Hp = H + d_pad
    out = torch.full((T, n_used, Hp), float("nan"), device="cuda")
    ws = torch.empty(g.mul_mat_id_ffn_workspace_size(H, F, E, n_used, T), dtype=torch.uint8, device="cuda")
    rc = g.mul_mat_id_ffn(wt_gu, pk["gate"], pk["up"], wt_d, pk["down"], H, F, E, xd, H * 4, H * 4, 1, idd, 4,
                          n_used * 4, n_used, T, out, Hp * 4, n_used * Hp * 4, ws, err)
    return rc, out


@pytest.mark.parametrize("wt_gu,wt_d,H,F,E,T,n_used,skew", [
    (12, 12, 512, 768, 32, 200, 8, False),
    (12, 14, 256, 512, 16, 77, 4, True),      # Q6_K down; skewed ids leave experts empty
    (8, 8, 256, 256, 8, 33, 2, False),
    (1, 1, 128, 96, 8, 50, 2, False),         # F16 stacks, F not a multiple of 256
    (12, 12, 2048, 768, 128, 2048, 8, False),
])
def test_mul_mat_id_ffn_matches_the_chain(cuda, wt_gu, wt_d, H, F, E, T, n_used, skew):
    """b200_mul_mat_id_ffn (one route for the three projections, SWIGLU fused into the down
    projection's packing) equals the op chain bit for bit, and the oracle composed op by op
    within the MUL_MAT tolerance (on the first tokens at the full-size case)."""
    import torch
    import ggml_b200 as g
    nat, pk, x, ids = _ffn_case(torch, g, wt_gu, wt_d, H, F, E, T, n_used, H + F + E + T + wt_d, skew)
    xd, idd = torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    want = _ffn_chain(torch, g, wt_gu, wt_d, pk, H, F, E, xd, idd, err)
    rc, got = _ffn_fused(torch, g, wt_gu, wt_d, pk, H, F, E, xd, idd, err)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    assert torch.equal(got, want), float((got - want).abs().max())
    # again with padded dst rows (strides) and the same workspace reused
    rc, got2 = _ffn_fused(torch, g, wt_gu, wt_d, pk, H, F, E, xd, idd, err, d_pad=32)
    torch.cuda.synchronize()
    assert rc == 0 and torch.equal(got2[:, :, :H], want)
    n = min(T, 32)
    og = oracle.mul_mat_id(wt_gu, nat["gate"].reshape(E, F, -1), H, F, E, x[:n], ids[:n])
    ou = oracle.mul_mat_id(wt_gu, nat["up"].reshape(E, F, -1), H, F, E, x[:n], ids[:n])
    od = oracle.mul_mat_id(wt_d, nat["down"].reshape(E, H, -1), F, H, E, oracle.swiglu(og, ou), ids[:n])
    assert rel_err(got[:n].cpu().numpy(), od) <= 1e-2


def test_mul_mat_id_ffn_bad_id_and_declines(cuda):
    import torch
    import ggml_b200 as g
    H, F, E, T, n_used = 256, 256, 8, 16, 2
    nat, pk, x, ids = _ffn_case(torch, g, 12, 12, H, F, E, T, n_used, 4)
    ids[5, 1] = E
    xd, idd = torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc, out = _ffn_fused(torch, g, 12, 12, pk, H, F, E, xd, idd, err)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 100
    assert bool(torch.isnan(out).all())   # a bad-id op writes nothing
    ws = torch.empty(g.mul_mat_id_ffn_workspace_size(H, F, E, n_used, T), dtype=torch.uint8, device="cuda")
    o = torch.empty((T, n_used, H), device="cuda")
    args = (xd, H * 4, H * 4, 1, idd, 4, n_used * 4, n_used, T, o, H * 4, n_used * H * 4)
    assert g.mul_mat_id_ffn(12, pk["gate"], pk["up"], 12, pk["down"], H, 200, E, *args, ws, err) == g.B200_E_UNSUPPORTED
    assert g.mul_mat_id_ffn(12, pk["gate"], pk["up"], 12, pk["down"], H, F, E, *args, ws[:1024], err) == \
        g.B200_E_WORKSPACE


_FFN_GRAPH_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
import ggml_b200 as g
import oracle
from conftest import rel_err
from ggml_b200 import quants
be = g.Backend()
rng = np.random.default_rng(31)
H, F, E, T, U = 512, 768, 32, 96, 8
stacks = [quants.quantize(g.Q4_K, (rng.standard_normal((E * n, k)) * 0.02).astype(np.float32))
          for n, k in ((F, H), (F, H), (H, F))]
ws = [g.make_tensor(g.Q4_K, [H, F, E], stacks[0], name="blk.0.ffn_up_exps.weight"),
      g.make_tensor(g.Q4_K, [H, F, E], stacks[1], name="blk.0.ffn_gate_exps.weight"),
      g.make_tensor(g.Q4_K, [F, H, E], stacks[2], name="blk.0.ffn_down_exps.weight")]
x = rng.standard_normal((T, 1, H)).astype(np.float32)
ids = np.stack([rng.permutation(E)[:U] for _ in range(T)]).astype(np.int32)
buf = g.DeviceBuffer(be, 64 << 20)
o = [i << 23 for i in range(8)]
assert buf.set(o[0], x) == 0 and buf.set(o[1], ids) == 0
tx = buf.tensor(o[0], g.F32, [H, 1, T], name="ffn_moe_in")
ti = buf.tensor(o[1], g.I32, [U, T], name="ffn_moe_topk")

def graph(extra_reader, swapped=False):
    up = buf.tensor(o[2], g.F32, [F, U, T], op=g.OP_MUL_MAT_ID, srcs=[ws[0], tx, ti])
    gate = buf.tensor(o[3], g.F32, [F, U, T], op=g.OP_MUL_MAT_ID, srcs=[ws[1], tx, ti])
    srcs = [up, gate] if swapped else [gate, up]
    h = buf.tensor(o[4], g.F32, [F, U, T], op=g.OP_GLU, srcs=srcs, op_params=[g.GLU_SWIGLU, 1 if swapped else 0])
    down = buf.tensor(o[5], g.F32, [H, U, T], op=g.OP_MUL_MAT_ID, srcs=[ws[2], h, ti])
    nodes = [up, gate, h, down]
    if extra_reader:   # a later node reads h: it must be written, so the chain runs op by op
        nodes.append(buf.tensor(o[6], g.F32, [F, U, T], op=g.OP_UNARY, srcs=[h], op_params=[g.UNARY_SILU]))
    return nodes

for nd in graph(True):
    assert g.supports_op(nd), nd.op
res = {}
for name, extra, sw in (("fused", False, False), ("fused_swapped", False, True), ("chain", True, False)):
    before = be.route_ops("moe_ffn")
    assert be.graph_compute(graph(extra, sw)) == g.STATUS_SUCCESS
    got = np.full((T, U, H), np.nan, np.float32)
    assert buf.get(o[5], got) == 0
    res[name] = got
    print(name.upper(), be.route_ops("moe_ffn") - before)
print("SAME", int(np.array_equal(res["fused"], res["chain"]) and np.array_equal(res["fused_swapped"], res["chain"])))
n = 24
og = oracle.mul_mat_id(g.Q4_K, stacks[1].reshape(E, F, -1), H, F, E, x[:n], ids[:n])
ou = oracle.mul_mat_id(g.Q4_K, stacks[0].reshape(E, F, -1), H, F, E, x[:n], ids[:n])
od = oracle.mul_mat_id(g.Q4_K, stacks[2].reshape(E, H, -1), F, H, E, oracle.swiglu(og, ou), ids[:n])
print("ORACLE", rel_err(res["fused"][:n], od))
assert be.device_errors() == 0 and be.cpu_fallbacks() == 0
buf.free()
be.close()
"""


def test_moe_ffn_through_graph_compute(cuda):
    """With B200_GLUE=1 the MoE FFN node chain (MUL_MAT_ID up, gate, GLU SWIGLU, MUL_MAT_ID down
    on device tensors) runs as one b200_mul_mat_id_ffn, the GLU's swapped form too; when a later
    node reads the SWIGLU output the chain runs op by op, and both give the same bits and match
    the oracle composed op by op."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, B200_GLUE="1")
    p = subprocess.run([sys.executable, "-c", _FFN_GRAPH_CHILD, ROOT], env=env, capture_output=True, text=True,
                       timeout=600)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    out = p.stdout
    assert out.split("FUSED ")[1].split()[0] == "1" and out.split("FUSED_SWAPPED ")[1].split()[0] == "1"
    assert out.split("CHAIN ")[1].split()[0] == "0"
    assert out.split("SAME ")[1].split()[0] == "1"
    assert float(out.split("ORACLE ")[1].split()[0]) <= 1e-2
