"""CPU tests of the oracle (the checker) and of the host-side encoders.

The oracle's dequantizers are pinned bit-for-bit to the golden vectors made from the gguf
package's restatement of ggml's dequantize_row_* (tests/golden/make_golden.py); its fp16
conversion to numpy's; the bench/test encoders to the oracle's C encoders.
"""
import os

import numpy as np
import pytest

import oracle
from conftest import rel_err
from ggml_b200 import quants

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["q8_0", "q4_k", "q6_k"])
def test_oracle_dequant_matches_golden(name):
    z = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    raw, deq, t = z["raw"], z["deq"], int(z["type_id"])
    got = oracle.dequantize(t, raw.reshape(1, -1), deq.size).reshape(deq.shape)
    assert np.array_equal(got.view(np.uint32), deq.view(np.uint32))
    assert str(z["gguf_version"]) == "0.19.0"


def test_oracle_q8_0_quantizer_matches_ggml_reference_rounding():
    z = np.load(os.path.join(GOLDEN, "dequant_q8_0.npz"))
    got = oracle.quantize(8, z["q8_src"])
    assert np.array_equal(got.reshape(-1), z["q8_quant"].reshape(-1))


def test_fp16_conversion_matches_numpy():
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(200000) * np.exp2(rng.uniform(-30, 18, 200000))).astype(np.float32)
    edge = np.array([65504, 65519, 65520, 65535, 65536, 1e-8, 2 ** -24, 2 ** -25, 3 * 2 ** -26, 2 ** -14,
                     np.inf, -np.inf, 0.0, -0.0, 5.96e-8, 6.1e-5], dtype=np.float32)
    x = np.concatenate([x, edge, -edge])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.fp16_bits(x), want)


@pytest.mark.parametrize("t", [8, 12, 14])
def test_numpy_encoders_match_oracle_encoders(t):
    rng = np.random.default_rng(t)
    x = (rng.standard_normal((48, 1024)) * 0.02).astype(np.float32)
    x[3] *= 100
    x[5, :300] = 0
    x[7, :256] = -1.0
    assert np.array_equal(quants.quantize(t, x), oracle.quantize(t, x))


@pytest.mark.parametrize("t,tol", [(8, 0.01), (12, 0.08), (14, 0.03)])
def test_encode_decode_round_trip(t, tol):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((16, 2048)) * 0.02).astype(np.float32)
    y = oracle.dequantize(t, quants.quantize(t, x), 2048)
    assert np.max(np.abs(y - x)) / np.max(np.abs(x)) < tol


def test_pack_act_sandwich():
    """rk_pack_act_row (ggml-rocket.cpp:1451-1475): s = max|row|, A16 = fp16(row * (1/s))."""
    rng = np.random.default_rng(3)
    a = rng.standard_normal((5, 64)).astype(np.float32)
    a[2] = 0.0
    a[3] *= 1e5
    a16, s = oracle.pack_act(a)
    assert s[2] == 1.0
    assert np.all(s[[0, 1, 3, 4]] == np.abs(a[[0, 1, 3, 4]]).max(1))
    inv = (np.float32(1.0) / s).astype(np.float32)
    assert np.array_equal(a16, (a * inv[:, None]).astype(np.float32).astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("t", [1, 8, 12, 14])
def test_oracle_mul_mat_matches_numpy(t):
    rng = np.random.default_rng(t + 100)
    N, K, M = 48, 512, 9
    w = quants.quantize(t, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    a = rng.standard_normal((M, K)).astype(np.float32)
    wf = oracle.dequantize(t, w, K).astype(np.float64)
    ref = (a.astype(np.float64) @ wf.T).astype(np.float32)
    assert np.allclose(oracle.mul_mat(t, w, N, K, a), ref, rtol=0, atol=1e-6)


def _numpy_fa(q, k16, v16, m16, scale):
    H, T, D = q.shape
    HK = k16.shape[0]
    k = k16.view(np.float16).astype(np.float64)
    v = v16.view(np.float16).astype(np.float64)
    m = m16.view(np.float16).astype(np.float64) if m16 is not None else None
    out = np.zeros((T, H, v.shape[2]))
    for h in range(H):
        s = q[h].astype(np.float64) @ k[h // (H // HK)].T * scale
        if m is not None:
            s = s + m[:T]
        mx = s.max(1, keepdims=True)
        p = np.where(np.isfinite(s), np.exp(s - np.where(np.isfinite(mx), mx, 0)), 0.0)
        den = p.sum(1, keepdims=True)
        o = (p @ v[h // (H // HK)]) / np.where(den > 0, den, 1)
        out[:, h] = np.where(den > 0, o, 0)
    return out


def test_oracle_flash_attn_matches_numpy_causal_gqa():
    rng = np.random.default_rng(5)
    H, HK, T, KV, D = 4, 2, 8, 20, 32
    q = rng.standard_normal((H, T, D)).astype(np.float32)
    k = rng.standard_normal((HK, KV, D)).astype(np.float16).view(np.uint16)
    v = rng.standard_normal((HK, KV, D)).astype(np.float16).view(np.uint16)
    mask = np.zeros((T, KV), dtype=np.float32)
    for t in range(T):
        mask[t, KV - T + t + 1:] = -np.inf
    mask[0, :] = -np.inf      # one fully masked row -> zeros
    m16 = mask.astype(np.float16).view(np.uint16)
    got = oracle.flash_attn(q, k, v, m16, 1 / np.sqrt(D), q_mode=0)
    want = _numpy_fa(q, k, v, m16, 1 / np.sqrt(D))
    assert np.allclose(got, want, atol=1e-6)
    assert np.all(got[0] == 0)


def test_oracle_moe_route_is_stable_counting_sort():
    rng = np.random.default_rng(9)
    n_tokens, n_used, n_expert = 37, 4, 9
    ids = np.stack([rng.permutation(n_expert)[:n_used] for _ in range(n_tokens)]).astype(np.int32)
    off, slot, tok = oracle.moe_route(ids, n_expert)
    assert off[0] == 0 and off[-1] == n_tokens * n_used
    for e in range(n_expert):
        rows = list(zip(tok[off[e]:off[e + 1]], slot[off[e]:off[e + 1]]))
        want = [(t, s) for t in range(n_tokens) for s in range(n_used) if ids[t, s] == e]
        assert rows == want
    bad = ids.copy()
    bad[3, 1] = n_expert
    assert oracle.moe_route(bad, n_expert) is None


@pytest.mark.parametrize("ne11", [1, 4])
def test_oracle_mul_mat_id_matches_per_row(ne11):
    rng = np.random.default_rng(ne11)
    K, N, n_expert, n_tokens, n_used = 256, 64, 6, 11, 4
    ws = [quants.quantize(12, (rng.standard_normal((N, K)) * 0.02).astype(np.float32)) for _ in range(n_expert)]
    as_raw = np.stack(ws)
    b = rng.standard_normal((n_tokens, ne11, K)).astype(np.float32)
    ids = np.stack([rng.permutation(n_expert)[:n_used] for _ in range(n_tokens)]).astype(np.int32)
    got = oracle.mul_mat_id(12, as_raw, K, N, n_expert, b, ids)
    for t in range(n_tokens):
        for e in range(n_used):
            x = ids[t, e]
            ref = oracle.mul_mat(12, ws[x], N, K, b[t, e % ne11][None])
            assert np.array_equal(got[t, e], ref[0])


def test_glue_oracle_matches_closed_forms():
    """The glue-op restatements (unpinned: ggml is absent) against float64 closed forms: the
    rope's sequential theta product and f32 rounding stay within 1e-5 of base^(-2j/n) * pos at
    modest positions; rms_norm, silu and swiglu within f32 rounding."""
    rng = np.random.default_rng(9)
    x = rng.standard_normal((5, 3, 128)).astype(np.float32)
    ref = x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True) + 1e-6)
    assert np.max(np.abs(oracle.rms_norm(x, 1e-6) - ref)) < 1e-5
    s = x.astype(np.float64)
    assert np.max(np.abs(oracle.silu(x) - s / (1 + np.exp(-s)))) < 1e-5
    g = rng.standard_normal(x.shape).astype(np.float32)
    assert np.max(np.abs(oracle.swiglu(x, g) - s / (1 + np.exp(-s)) * g)) < 1e-5
    pos = np.array([0, 1, 7, 31, 100], dtype=np.int32)
    for mode in (0, 2):
        for n_dims in (128, 64):
            y = oracle.rope(x, pos, n_dims, mode, 10000.0, 0.5, 1.0)
            half = n_dims // 2
            theta = 0.5 * pos[:, None].astype(np.float64) * 10000.0 ** (-2.0 * np.arange(half) / n_dims)
            c, sn = np.cos(theta)[:, None, :], np.sin(theta)[:, None, :]
            if mode == 2:
                i0, i1 = np.arange(half), np.arange(half) + half
            else:
                i0, i1 = 2 * np.arange(half), 2 * np.arange(half) + 1
            want = s.copy()
            want[..., i0] = s[..., i0] * c - s[..., i1] * sn
            want[..., i1] = s[..., i0] * sn + s[..., i1] * c
            assert np.max(np.abs(y - want)) < 1e-4, (mode, n_dims)
            assert np.array_equal(y[..., n_dims:], x[..., n_dims:])


def test_soft_max_oracle_matches_closed_form():
    rng = np.random.default_rng(10)
    x = (rng.standard_normal((6, 256)) * 4).astype(np.float32)
    w = x.astype(np.float64) * 0.5
    e = np.exp(w - w.max(axis=-1, keepdims=True))
    assert np.max(np.abs(oracle.soft_max(x, 0.5) - e / e.sum(axis=-1, keepdims=True))) < 1e-6


def test_cpu_path_restatement_matches_the_oracle():
    """The timed CPU baseline (oracle/cpu_path.c: 8-bit activation blocks, integer Q4_K block dots)
    stays within the 8-bit activation rounding of the fp64 oracle, its AVX2 and portable dots agree
    exactly, and an all-zero activation row gives zeros."""
    import ctypes
    rng = np.random.default_rng(21)
    N, K, M = 96, 1024, 5
    raw = oracle.quantize(12, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    a = rng.standard_normal((M, K)).astype(np.float32)
    a[2] = 0.0
    got = oracle.cpu_path_mul_mat_q4k(raw, N, K, a)
    want = oracle.mul_mat(12, raw, N, K, a)
    assert rel_err(got, want) <= 2e-2
    assert np.all(got[2] == 0.0)
    L = oracle.path_lib()
    L.orc_cpu_path_scalar_dot_check.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    for n, m in ((0, 0), (7, 4), (95, 1)):
        o = np.zeros(2, np.float32)
        row = np.ascontiguousarray(raw[n])
        assert L.orc_cpu_path_scalar_dot_check(row.ctypes.data, K, np.ascontiguousarray(a[m]).ctypes.data,
                                               o.ctypes.data) == 0
        assert o[0] == o[1]
