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
