"""The combined-N GEMM of a fused MUL_MAT group (b200_gemm_packed_group), through the C ABI.

The reference runs a group of MUL_MATs that share src1 (QKV, gate/up) as one GEMM over the
members' weights side by side, unpacking each member's columns into its own dst
(ggml-rocket.cpp:4956-5020, 5040-5160). Here the members' weight tiles are scheduled by one
launch. Checked against the fp64 oracle per member (max |err| / max |ref| <= 1e-2, the north
star's bound) on small shapes, and against one b200_gemm_packed launch per member (the
single-op path, itself oracle-tested) at the Llama-3-8B group shapes, where only the order of
the fp32 sums may differ: 1e-5.
"""
import numpy as np
import pytest

import oracle
from conftest import rel_err, rk_compare
from test_gpu_mul_mat import _dev, _err_word, _check_err, _weights

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _pack_weight(torch, g, wtype, w_raw, N, K):
    packed = torch.empty(g.weight_packed_size(wtype, N, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(wtype, _dev(torch, w_raw.reshape(-1)), N, K, packed)
    return packed


def _run(torch, wtype, K, Ns, M, seed, ldd_pad=0):
    """Pack one activation, run the group launch and the per-member launches; returns
    (group outputs, per-member outputs, native weights, activation)."""
    import ggml_b200 as g
    rng = np.random.default_rng(seed)
    ws_raw = [_weights(rng, N, K, wtype) for N in Ns]
    a = rng.standard_normal((M, K)).astype(np.float32)
    packed = [_pack_weight(torch, g, wtype, w, N, K) for w, N in zip(ws_raw, Ns)]
    a16 = torch.empty((M, K), dtype=torch.float16, device="cuda")
    scales = torch.empty(M, dtype=torch.float32, device="cuda")
    g.act_pack(_dev(torch, a), M, K, a16, scales)
    lds = [N + ldd_pad for N in Ns]
    outs = [torch.full((M, ld), float("nan"), dtype=torch.float32, device="cuda") for ld in lds]
    wsb = g.gemm_packed_group_workspace_size(M, Ns, K, wtype)
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device="cuda")
    err = _err_word(torch)
    g.gemm_packed_group(wtype, packed, Ns, K, a16, scales, M, outs, ws, err, ldds=lds)
    torch.cuda.synchronize()
    _check_err(err)
    got = [o.cpu().numpy() for o in outs]
    sep = []
    for p, N in zip(packed, Ns):
        o = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        wsm = torch.empty(max(g.gemm_packed_workspace_size(M, N, K, wtype), 256), dtype=torch.uint8, device="cuda")
        g.gemm_packed(wtype, p, N, K, a16, scales, M, o, wsm, err)
        torch.cuda.synchronize()
        _check_err(err)
        sep.append(o.cpu().numpy())
    return got, sep, ws_raw, a


# (wtype, K, member N, M): every weight format, token tiles 32-256, ragged members (N % 128 != 0),
# ragged M, Q8_0's ragged K, and 2-4 members
SMALL = [(1, 1024, [384, 256, 128], 300),
         (12, 512, [256, 160], 100),
         (14, 1024, [512, 512, 256, 128], 64),
         (8, 2080, [512, 48], 33),
         (12, 2048, [1024, 1024], 512),
         (14, 768, [272, 528, 16], 200)]


@pytest.mark.parametrize("wtype,K,Ns,M", SMALL)
def test_gemm_group_vs_oracle(cuda, wtype, K, Ns, M):
    import torch
    got, sep, ws_raw, a = _run(torch, wtype, K, Ns, M, seed=K + sum(Ns) + M + wtype, ldd_pad=16)
    for m, N in enumerate(Ns):
        out = got[m][:, :N]
        assert np.all(np.isfinite(out)), (m, N)
        assert np.all(np.isnan(got[m][:, N:])), "wrote past the member's columns"
        ref = oracle.mul_mat(wtype, ws_raw[m], N, K, a)
        assert rel_err(out, ref) <= TOL, (m, N)
        cos, bad = rk_compare(ref, out)
        assert bad == 0 and cos > 0.9999
        assert rel_err(out, sep[m]) <= 1e-5


@pytest.mark.parametrize("wtype,K,Ns", [(12, 4096, [4096, 1024, 1024]),    # Llama-3-8B Q, K, V
                                        (12, 4096, [14336, 14336]),        # gate, up
                                        (1, 4096, [4096, 1024, 1024])])
def test_gemm_group_llama_shapes(cuda, wtype, K, Ns):
    """The Llama-3-8B groups at the 512-token ubatch: each member equals its own launch up to
    the order of the fp32 sums; a sampled block of rows checked against the oracle."""
    import torch
    M = 512
    got, sep, ws_raw, a = _run(torch, wtype, K, Ns, M, seed=7 + sum(Ns) + wtype)
    for m, N in enumerate(Ns):
        assert np.all(np.isfinite(got[m]))
        assert rel_err(got[m], sep[m]) <= 1e-5, m
        rows = np.arange(0, M, 37)
        ref = oracle.mul_mat(wtype, ws_raw[m], N, K, a[rows])
        assert rel_err(got[m][rows], ref) <= TOL, m


def test_gemm_group_plans(cuda):
    """The planner over the members' tiles takes both schedules that share a tile somewhere in the
    cases above: stream-K (shared K ranges, partials and flags) and the cluster split (two CTAs
    per tile); the group launch twice in a row gives the same bits (the split barriers and the
    stream-K epochs start afresh per call)."""
    import torch
    import ggml_b200 as g
    kinds = set()
    for wtype, K, Ns, M in SMALL + [(12, 4096, [4096, 1024, 1024], 512), (12, 4096, [14336, 14336], 512)]:
        p = g.gemm_packed_group_plan(M, Ns, K, wtype)
        tiles = sum((N + 127) // 128 for N in Ns) * ((M + p["token_tile"] - 1) // p["token_tile"])
        if p["splits"] == 1:
            kinds.add("whole")
        elif p["splits"] == 2 and p["grid"] == 2 * tiles:
            kinds.add("csplit")
        else:
            kinds.add("streamk")
    assert {"csplit", "streamk"} <= kinds, kinds
    first, _, _, _ = _run(torch, 12, 4096, [14336, 14336], 512, seed=5)
    again, _, _, _ = _run(torch, 12, 4096, [14336, 14336], 512, seed=5)
    for x, y in zip(first, again):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_gemm_group_rejects(cuda):
    """Bad member counts and shapes are refused before any launch."""
    import torch
    import ggml_b200 as g
    a16 = torch.zeros((32, 256), dtype=torch.float16, device="cuda")
    sc = torch.ones(32, dtype=torch.float32, device="cuda")
    w = torch.zeros(g.weight_packed_size(1, 128, 256), dtype=torch.uint8, device="cuda")
    o = torch.zeros((32, 128), dtype=torch.float32, device="cuda")
    err = _err_word(torch)
    with pytest.raises(g.B200Error):
        g.gemm_packed_group(1, [w] * 5, [128] * 5, 256, a16, sc, 32, [o] * 5, None, err)
    with pytest.raises(g.B200Error):
        g.gemm_packed_group(1, [w, w], [128, 120], 256, a16, sc, 32, [o, o], None, err)
