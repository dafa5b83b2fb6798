"""Parity at the sizes BASELINE.json names, on the GPU through the C ABI, against the fp64 oracle.

These are the shapes the bench times:
  configs[0]  F16 MUL_MAT, N = K = 4096, M = 512
  configs[1]  Q8_0 / Q4_K / Q6_K MUL_MAT, (K, N) in {(4096, 4096), (4096, 14336), (14336, 4096)},
              M in {32, 128, 512, 2048}
  configs[2]  FLASH_ATTN_EXT, 32 query / 8 KV heads, D 128, n_q 512, causal, n_kv in {1024, 4096, 16384}
  configs[3]  MUL_MAT_ID, 128 experts, top-8 of softmax(N(0, 1) logits), hidden 2048, FFN 768, Q4_K,
              2048 tokens (the gate/up form with ne11 = 1 and the down form with ne11 = n_used)

The whole op runs on the GPU; the fp64 oracle (a restatement of rocket_cpu_matmul_slice,
ggml-rocket.cpp:4053-4084, and of ref_fa, test-rocket-fa.cpp:101-135) checks a seeded sample of the
output that it finishes in seconds: 64 full output rows plus 64 full output columns of every
MUL_MAT, 24 query positions (the first and the last included) of every attention head, and 64 whole
tokens (all their slots) of the MoE layer, besides the route of every row. Tolerance as in
test-rocket-matmul.cpp:316-366: max |err| / max |ref| <= 1e-2 over each sample, plus the
reference's element rule.
"""
import math

import numpy as np
import pytest

import oracle
from conftest import rel_err, rk_compare
from ggml_b200 import quants

pytestmark = pytest.mark.gpu

TOL = 1e-2
M_SWEEP = (32, 128, 512, 2048)
KN_SWEEP = ((4096, 4096), (4096, 14336), (14336, 4096))


def _weights_f32(K, N, seed):
    rng = np.random.default_rng(seed)
    return rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)


def _native(wtype, w):
    if wtype == 1:
        return oracle.fp16_bits(w).view(np.uint8).reshape(w.shape[0], -1)
    return quants.quantize(wtype, w)


def _run_sweep(torch, wtype, w_native, N, K, Ms, seed):
    """Pack the weight once, run b200_mul_mat at every M, check a sample of each output."""
    import ggml_b200 as g
    packed = torch.empty(g.weight_packed_size(wtype, N, K), dtype=torch.uint8, device="cuda")
    raw = torch.from_numpy(np.ascontiguousarray(w_native).reshape(-1)).cuda()
    g.weight_pack(wtype, raw, N, K, packed)
    del raw
    rng = np.random.default_rng(seed)
    for M in Ms:
        a = rng.standard_normal((M, K), dtype=np.float32)
        out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        ws = torch.empty(max(256, g.mul_mat_workspace_size(M, N, K, wtype)), dtype=torch.uint8, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        g.mul_mat(wtype, packed, N, K, torch.from_numpy(a).cuda(), M, out, ws, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, f"device error word {int(err.item())}"
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got)), f"non-finite output at M={M}"
        rows = np.unique(np.concatenate([[0, M - 1], rng.choice(M, min(M, 62), replace=False)]))
        cols = np.unique(np.concatenate([[0, N - 1], rng.choice(N, 62, replace=False)]))
        ref_rows = oracle.mul_mat(wtype, w_native, N, K, a[rows])
        ref_cols = oracle.mul_mat(wtype, np.ascontiguousarray(w_native[cols]), len(cols), K, a)
        for ref, sub in ((ref_rows, got[rows]), (ref_cols, got[:, cols])):
            assert rel_err(sub, ref) <= TOL, f"M={M}: max rel err {rel_err(sub, ref)}"
            cos, bad = rk_compare(ref, sub)
            assert bad == 0 and cos > 0.9999, f"M={M}: cos {cos}, {bad} bad elements"


def test_config0_f16_4096(cuda):
    """F16 weight [4096, 4096], F32 activations [512, 4096]."""
    import torch
    K = N = 4096
    w = _native(1, _weights_f32(K, N, 0xB200))
    _run_sweep(torch, 1, w, N, K, (512,), seed=0xB201)


@pytest.mark.parametrize("wtype", [8, 12, 14], ids=["q8_0", "q4_k", "q6_k"])
@pytest.mark.parametrize("K,N", KN_SWEEP, ids=[f"K{k}_N{n}" for k, n in KN_SWEEP])
def test_config1_quant_sweep(cuda, wtype, K, N):
    """the quantized sweep at every M of the sweep, one weight per (type, K, N)."""
    import torch
    w = _native(wtype, _weights_f32(K, N, 0xB200 ^ (K + 3 * N)))
    _run_sweep(torch, wtype, w, N, K, M_SWEEP, seed=0xB200 + wtype + K + N)


def _f16(x):
    with np.errstate(over="ignore"):
        return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("KV", [1024, 4096, 16384])
def test_config2_flash_attn(cuda, KV):
    """n_q = 512 queries at positions KV-512..KV-1 against KV keys, causal, read from a
    KV-cache view. Checked against ref_fa's own rounding of Q (fp16 of the unscaled q, q_mode 1)
    and against fp16 of the scaled q (q_mode 2), the two readings of "Q narrowed to fp16"."""
    import torch
    from test_gpu_flash_attn import run_fa
    rng = np.random.default_rng(0xFA00 + KV)
    H, HK, D, T = 32, 8, 128, 512
    Q = rng.standard_normal((H, T, D), dtype=np.float32)
    K16 = _f16(rng.standard_normal((HK, KV, D), dtype=np.float32))
    V16 = _f16(rng.standard_normal((HK, KV, D), dtype=np.float32))
    pos = np.arange(KV - T, KV).reshape(T, 1)
    M16 = _f16(np.where(np.arange(KV).reshape(1, KV) <= pos, 0.0, -np.inf).astype(np.float32))
    scale = 1.0 / math.sqrt(D)
    got = run_fa(torch, Q, K16, V16, M16, scale, k_layout="cache")
    assert np.all(np.isfinite(got))
    sub = np.unique(np.concatenate([[0, T - 1], rng.choice(T, 22, replace=False)]))
    for q_mode in (1, 2):
        want = oracle.flash_attn(np.ascontiguousarray(Q[:, sub]), K16, V16, np.ascontiguousarray(M16[sub]), scale,
                                 q_mode=q_mode)
        err = rel_err(got[sub], want)
        assert err <= TOL, f"q_mode {q_mode}: max rel err {err}"
        cos, bad = rk_compare(want, got[sub])
        assert bad == 0 and cos > 0.9999


def _moe_ids(rng, T, E, top):
    logits = rng.standard_normal((T, E), dtype=np.float32)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return np.argsort(-p, axis=-1, kind="stable")[:, :top].astype(np.int32)


@pytest.mark.parametrize("K,N,ne11", [(2048, 768, 1), (768, 2048, 8)], ids=["gate_up", "down"])
def test_config3_moe_layer(cuda, K, N, ne11):
    """128 distinct Q4_K experts, top-8 routing from softmax(N(0,1)) over 2048 tokens."""
    import torch
    from test_gpu_moe import run_moe
    E, top, T = 128, 8, 2048
    rng = np.random.default_rng(0x0E00 + K)
    w = rng.standard_normal((E * N, K), dtype=np.float32) * np.float32(0.02)
    native = quants.quantize(12, w)
    del w
    b = rng.standard_normal((T, ne11, K), dtype=np.float32)
    ids = _moe_ids(rng, T, E, top)
    got, err, route = run_moe(torch, 12, native, K, N, E, b, ids)
    assert err == 0
    off, slot, tok = oracle.moe_route(ids, E)
    assert np.array_equal(route[0], off) and np.array_equal(route[1], slot) and np.array_equal(route[2], tok)
    assert np.all(np.isfinite(got))
    sub = np.unique(np.concatenate([[0, T - 1], rng.choice(T, 62, replace=False)]))
    want = oracle.mul_mat_id(12, native.reshape(E, N, -1), K, N, E, np.ascontiguousarray(b[sub]),
                             np.ascontiguousarray(ids[sub]))
    assert rel_err(got[sub], want) <= TOL
    cos, bad = rk_compare(want, got[sub])
    assert bad == 0 and cos > 0.9999
