"""Decode-size MUL_MAT (b200_mul_mat_vec, M = 1..8, Q4_K) on the GPU against the CPU oracle.

The weights enter the MMA as exact integers q*sc with fp32 scales, the activations as fp16 of
a / s per 256-value block (s the block's absmax), products are exact and summed in fp32; so the
only error beyond fp32 sums is the activations' fp16 rounding (~2^-12 relative), and the bound
here, DECODE_TOL = 2e-3 max relative error, is five times tighter than the prefill MUL_MAT's
1e-2. Shapes include N not a multiple of the 16-row block, K of one super-block, strided src1 /
dst rows and unaligned activations (the scalar load path); repeated calls are bit-identical."""
import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu

DECODE_TOL = 2e-3


def _run(torch, w_raw, N, K, a, lda=None, ldd=None, offset=0):
    import ggml_b200 as g
    M = a.shape[0]
    lda = lda or K
    ldd = ldd or N
    raw = torch.from_numpy(np.ascontiguousarray(w_raw).reshape(-1)).cuda()
    packed = torch.empty(g.weight_packed_size(g.Q4_K, N, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(g.Q4_K, raw, N, K, packed)
    abuf = torch.zeros(offset + M * lda, dtype=torch.float32, device="cuda")
    av = abuf[offset:offset + M * lda].view(M, lda)
    av[:, :K] = torch.from_numpy(a)
    out = torch.full((M * ldd,), float("nan"), dtype=torch.float32, device="cuda")
    ws = torch.empty(max(256, g.lib().b200_mul_mat_vec_workspace_size(M, N, K)), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = g.mul_mat_vec(g.Q4_K, packed, N, K, av, M, out, ws, err, lda=lda, ldd=ldd)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    return out.view(M, ldd)[:, :N].cpu().numpy()


@pytest.mark.parametrize("N,K,M", [(4096, 4096, 1), (14336, 4096, 2), (4096, 14336, 3), (1000, 512, 4),
                                   (200, 256, 7), (4104, 4096, 8), (64, 2048, 5)])
def test_mul_mat_vec_matches_oracle(cuda, N, K, M):
    import torch
    rng = np.random.default_rng(N + K + M)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    raw = oracle.quantize(12, w)
    a = rng.standard_normal((M, K)).astype(np.float32)
    got = _run(torch, raw, N, K, a)
    want = oracle.mul_mat(12, raw, N, K, a)
    assert np.all(np.isfinite(got))
    assert rel_err(got, want) <= DECODE_TOL, rel_err(got, want)


def test_mul_mat_vec_strided_and_unaligned(cuda):
    import torch
    rng = np.random.default_rng(3)
    N, K, M = 520, 1024, 3
    raw = oracle.quantize(12, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    a = rng.standard_normal((M, K)).astype(np.float32)
    want = oracle.mul_mat(12, raw, N, K, a)
    # padded rows on both sides, then activations that start 4 bytes past a 16-byte boundary
    first = _run(torch, raw, N, K, a, lda=K + 8, ldd=N + 24)
    assert rel_err(first, want) <= DECODE_TOL
    assert np.array_equal(first, _run(torch, raw, N, K, a, lda=K + 8, ldd=N + 24))   # deterministic
    assert rel_err(_run(torch, raw, N, K, a, lda=K + 1, offset=1), want) <= DECODE_TOL


def test_mul_mat_vec_declines_what_it_does_not_tile(cuda):
    import torch
    import ggml_b200 as g
    x = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    f = torch.zeros(1 << 14, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert g.mul_mat_vec(g.F16, x, 64, 256, f, 1, f, x, err) == g.B200_E_UNSUPPORTED      # not Q4_K
    assert g.mul_mat_vec(g.Q4_K, x, 64, 256, f, 9, f, x, err) == g.B200_E_UNSUPPORTED     # M > 8
    assert g.mul_mat_vec(g.Q4_K, x, 64, 200, f, 1, f, x, err) == g.B200_E_UNSUPPORTED     # K % 256
    small = x[:g.lib().b200_mul_mat_vec_workspace_size(1, 64, 256) - 1]
    assert g.mul_mat_vec(g.Q4_K, x, 64, 256, f, 1, f, small, err) == g.B200_E_INVALID      # workspace too small


def test_mul_mat_vec_back_to_back_shared_workspace(cuda):
    """Calls queued back to back on one stream, sharing one workspace, with different M, N and
    activations (the backend's pattern: each call's prep rewrites the workspace the previous
    call's kernel read), synchronised only at the end."""
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(11)
    K = 4096
    cases = [(4096, 1), (1024, 4), (14336, 8), (1024, 4), (4096, 1), (2048, 2)]
    need = max(g.lib().b200_mul_mat_vec_workspace_size(M, N, K) for N, M in cases)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    runs = []
    for N, M in cases:
        raw = oracle.quantize(12, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
        a = rng.standard_normal((M, K)).astype(np.float32)
        rawd = torch.from_numpy(np.ascontiguousarray(raw).reshape(-1)).cuda()
        packed = torch.empty(g.weight_packed_size(g.Q4_K, N, K), dtype=torch.uint8, device="cuda")
        g.weight_pack(g.Q4_K, rawd, N, K, packed)
        runs.append((raw, a, packed, torch.from_numpy(a).cuda(), torch.full((M, N), float("nan"), device="cuda"), N, M))
    torch.cuda.synchronize()
    for raw, a, packed, ad, out, N, M in runs:
        assert g.mul_mat_vec(g.Q4_K, packed, N, K, ad, M, out, ws, err) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for raw, a, packed, ad, out, N, M in runs:
        e = rel_err(out.cpu().numpy(), oracle.mul_mat(12, raw, N, K, a))
        assert e <= DECODE_TOL, (N, M, e)


def test_mul_mat_vec_stream_schedule(cuda):
    """The other work schedule (B200_GEMV_SCHEDULE, read once per process, so in a child): the
    same parity cases and the back-to-back shared-workspace case under it."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    other = "rows" if os.environ.get("B200_GEMV_SCHEDULE") == "stream" else "stream"
    env = dict(os.environ, B200_GEMV_SCHEDULE=other)
    p = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", __file__,
                        "-k", "matches_oracle or back_to_back or strided"], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-2000:]
