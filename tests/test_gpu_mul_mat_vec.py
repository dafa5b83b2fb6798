"""Decode-size MUL_MAT (b200_mul_mat_vec, M = 1..32; Q4_K, Q6_K, Q8_0) on the GPU against the CPU
oracle.

The weights enter the MMA as exact integers (q*sc for Q4_K, q + offset for Q6_K / Q8_0, the offset
cancelled exactly by the MMA's start value) with fp32 scales, the activations as fp16 of a / s
per 256-value block (s the block's absmax); products are exact and summed in fp32, so the only
error beyond fp32 sums is the activations' fp16 rounding (~2^-12 relative), and the bound here,
DECODE_TOL = 2e-3 max relative error, is five times tighter than the prefill MUL_MAT's 1e-2.
Shapes cover every 8-row column-tile count (M = 1..32), N not a multiple of the 16- or 128-row
blocks, K of one super-block, Q8_0 with K not a multiple of 256 (the packed zero padding), strided
src1 / dst rows and unaligned activations (the scalar load paths); repeated calls are
bit-identical. Q4_K at M <= 5 runs on the row-block kernels by default; the schedule test runs
the same cases with each kernel forced."""
import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu

DECODE_TOL = 2e-3
Q8_0, Q4_K, Q6_K = 8, 12, 14


def _pack(torch, wtype, w_raw, N, K):
    import ggml_b200 as g
    raw = torch.from_numpy(np.ascontiguousarray(w_raw).reshape(-1)).cuda()
    packed = torch.empty(g.weight_packed_size(wtype, N, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(wtype, raw, N, K, packed)
    return packed


def _run(torch, wtype, w_raw, N, K, a, lda=None, ldd=None, offset=0):
    import ggml_b200 as g
    M = a.shape[0]
    lda = lda or K
    ldd = ldd or N
    packed = _pack(torch, wtype, w_raw, N, K)
    abuf = torch.zeros(offset + M * lda, dtype=torch.float32, device="cuda")
    av = abuf[offset:offset + M * lda].view(M, lda)
    av[:, :K] = torch.from_numpy(a)
    out = torch.full((M * ldd,), float("nan"), dtype=torch.float32, device="cuda")
    ws = torch.empty(max(256, g.lib().b200_mul_mat_vec_workspace_size(M, N, K)), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = g.mul_mat_vec(wtype, packed, N, K, av, M, out, ws, err, lda=lda, ldd=ldd)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    return out.view(M, ldd)[:, :N].cpu().numpy()


def _case(wtype, N, K, M, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    raw = oracle.quantize(wtype, w)
    a = rng.standard_normal((M, K)).astype(np.float32)
    return raw, a


@pytest.mark.parametrize("wtype", [Q4_K, Q6_K, Q8_0])
@pytest.mark.parametrize("N,K,M", [(4096, 4096, 1), (4096, 14336, 1), (1001, 2816, 1), (14336, 4096, 2),
                                   (4096, 14336, 3), (1000, 512, 4),
                                   (200, 256, 7), (4104, 4096, 8), (64, 2048, 5), (4096, 4096, 9),
                                   (1024, 2048, 16), (520, 1024, 17), (2048, 4096, 24), (1000, 768, 31),
                                   (4096, 4096, 32)])
def test_mul_mat_vec_matches_oracle(cuda, wtype, N, K, M):
    import torch
    if wtype == Q6_K and N % 8:
        N += 8 - N % 8   # the transposed d plane's row pitch is a multiple of 16 bytes
    raw, a = _case(wtype, N, K, M, N + K + M + wtype)
    got = _run(torch, wtype, raw, N, K, a)
    want = oracle.mul_mat(wtype, raw, N, K, a)
    assert np.all(np.isfinite(got))
    assert rel_err(got, want) <= DECODE_TOL, rel_err(got, want)


@pytest.mark.parametrize("N,K,M", [(4096, 4128, 1), (1000, 96, 8), (520, 1056, 12)])
def test_mul_mat_vec_q8_0_ragged_k(cuda, N, K, M):
    """Q8_0 rows whose K is not a multiple of 256: the packed groups are zero-padded and the
    activations past K are zeros."""
    import torch
    raw, a = _case(Q8_0, N, K, M, K + M)
    got = _run(torch, Q8_0, raw, N, K, a)
    assert rel_err(got, oracle.mul_mat(Q8_0, raw, N, K, a)) <= DECODE_TOL


@pytest.mark.parametrize("wtype,M", [(Q4_K, 3), (Q4_K, 11), (Q6_K, 3), (Q8_0, 11)])
def test_mul_mat_vec_strided_and_unaligned(cuda, wtype, M):
    import torch
    N, K = 520, 1024
    raw, a = _case(wtype, N, K, M, 3 + wtype + M)
    want = oracle.mul_mat(wtype, raw, N, K, a)
    # padded rows on both sides, then activations that start 4 bytes past a 16-byte boundary
    first = _run(torch, wtype, raw, N, K, a, lda=K + 8, ldd=N + 24)
    assert rel_err(first, want) <= DECODE_TOL
    assert np.array_equal(first, _run(torch, wtype, raw, N, K, a, lda=K + 8, ldd=N + 24))   # deterministic
    assert rel_err(_run(torch, wtype, raw, N, K, a, lda=K + 1, offset=1), want) <= DECODE_TOL


def test_mul_mat_vec_zero_rows_and_tokens(cuda):
    """An all-zero activation row (s = 1, every fp16 zero) and all-zero weight rows give exact
    zeros beside ordinary rows, on both kernels (M = 3 and M = 12)."""
    import torch
    N, K = 256, 1024
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[:17] = 0.0
    for M in (3, 12):
        a = rng.standard_normal((M, K)).astype(np.float32)
        a[1] = 0.0
        for wtype in (Q4_K, Q6_K, Q8_0):
            raw = oracle.quantize(wtype, w)
            got = _run(torch, wtype, raw, N, K, a)
            assert np.all(got[1] == 0.0) and np.all(got[:, :17] == 0.0)
            assert rel_err(got, oracle.mul_mat(wtype, raw, N, K, a)) <= DECODE_TOL


def test_mul_mat_vec_declines_what_it_does_not_tile(cuda):
    import torch
    import ggml_b200 as g
    x = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    f = torch.zeros(1 << 14, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert g.mul_mat_vec(g.F16, x, 64, 256, f, 1, f, x, err) == g.B200_E_UNSUPPORTED      # dense weight
    assert g.mul_mat_vec(g.Q4_K, x, 64, 256, f, 33, f, x, err) == g.B200_E_UNSUPPORTED    # M > 32
    assert g.mul_mat_vec(g.Q4_K, x, 64, 200, f, 1, f, x, err) == g.B200_E_UNSUPPORTED     # K % 256
    assert g.mul_mat_vec(g.Q4_K, x, 64, 200, f, 12, f, x, err) == g.B200_E_UNSUPPORTED    # K % 256, tiled
    assert g.mul_mat_vec(g.Q6_K, x, 64, 288, f, 1, f, x, err) == g.B200_E_UNSUPPORTED     # K % 256
    assert g.mul_mat_vec(g.Q8_0, x, 64, 200, f, 1, f, x, err) == g.B200_E_UNSUPPORTED     # K % 32
    # workspace too small: the reported size bounds every path, so one byte short of it fails the
    # tiled path (M > 8), and a 255-byte workspace fails the row-block path
    small = x[:g.lib().b200_mul_mat_vec_workspace_size(20, 64, 256) - 1]
    assert g.mul_mat_vec(g.Q4_K, x, 64, 256, f, 20, f, small, err) == g.B200_E_INVALID
    assert g.mul_mat_vec(g.Q4_K, x, 64, 256, f, 2, f, x[:255], err) == g.B200_E_INVALID


def test_mul_mat_vec_back_to_back_shared_workspace(cuda):
    """Calls queued back to back on one stream, sharing one workspace, with different weight
    types, M, N and activations (the backend's pattern: each call's prep rewrites the workspace the
    previous call's kernel read), synchronised only at the end."""
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(11)
    K = 4096
    cases = [(Q4_K, 4096, 1), (Q8_0, 1024, 4), (Q4_K, 14336, 8), (Q6_K, 1024, 20), (Q4_K, 4096, 1),
             (Q8_0, 2048, 32), (Q6_K, 4096, 2), (Q4_K, 2048, 13)]
    need = max(g.lib().b200_mul_mat_vec_workspace_size(M, N, K) for _, N, M in cases)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    runs = []
    for wtype, N, M in cases:
        raw = oracle.quantize(wtype, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        a = rng.standard_normal((M, K)).astype(np.float32)
        packed = _pack(torch, wtype, raw, N, K)
        runs.append((wtype, raw, a, packed, torch.from_numpy(a).cuda(), torch.full((M, N), float("nan"), device="cuda"),
                     N, M))
    torch.cuda.synchronize()
    for wtype, raw, a, packed, ad, out, N, M in runs:
        assert g.mul_mat_vec(wtype, packed, N, K, ad, M, out, ws, err) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for wtype, raw, a, packed, ad, out, N, M in runs:
        e = rel_err(out.cpu().numpy(), oracle.mul_mat(wtype, raw, N, K, a))
        assert e <= DECODE_TOL, (wtype, N, M, e)


@pytest.mark.parametrize("schedule", ["rows", "stream", "tiles"])
def test_mul_mat_vec_each_schedule(cuda, schedule):
    """Each kernel for Q4_K at M <= 8 forced for every such M (B200_GEMV_SCHEDULE, read once per
    process, so in a child; unset, M <= 5 takes the row-block kernel and M >= 6 the tiled one, and
    Q8_0 at M = 1 the one-launch fp32 kernel): the parity cases, the strided cases and the
    back-to-back shared-workspace case under
    each."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    if os.environ.get("B200_GEMV_SCHEDULE") == schedule:
        pytest.skip("this process already runs that schedule")
    env = dict(os.environ, B200_GEMV_SCHEDULE=schedule)
    p = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", __file__,
                        "-k", "matches_oracle or back_to_back or strided"], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=900)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-2000:]
