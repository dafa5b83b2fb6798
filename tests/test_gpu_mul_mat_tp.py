"""MUL_MAT with the weight rows split across GPUs (b200_mul_mat_tp / _finish) on the GPU.

The G ranks are emulated inside one process on one B200: rank r's GEMM runs over its row block
of the weight and its epilogue stores its columns into all G dst buffers (separate buffers on
this GPU stand in for the other GPUs'); every rank's signal is issued before any rank's wait, so
no kernel ever waits for a later launch. Every rank's dst must equal the single-GPU b200_mul_mat
result (bit for bit with one rank, where the plan is the same; otherwise up to the order of the
fp32 K-sums) and the CPU oracle within the MUL_MAT tolerance. The op also runs as torchrun ranks
(tp_worker.py) through ggml_b200.tp, with one rank always and with two when two GPUs are present.
"""
import ctypes
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import ROOT, rel_err
from test_gpu_mul_mat import _weights, run_mul_mat

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _emulated(torch, g, wtype, w_raw, N, K, a, G):
    from ggml_b200.tp import shard_rows
    M = a.shape[0]
    lib = g.lib()
    rows_bytes = w_raw.reshape(N, -1)
    dsts = [torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda") for _ in range(G)]
    flags = [torch.zeros((G, 4), dtype=torch.int32, device="cuda") for _ in range(G)]
    peer_dst = torch.tensor([d.data_ptr() for d in dsts], dtype=torch.int64, device="cuda")
    peer_flags = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device="cuda")
    a_dev = torch.from_numpy(np.ascontiguousarray(a.astype(np.float32))).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    keep = []
    for r in range(G):
        lo, hi = shard_rows(N, G, r)
        raw = torch.from_numpy(np.ascontiguousarray(rows_bytes[lo:hi]).reshape(-1)).cuda()
        packed = torch.empty(g.weight_packed_size(wtype, hi - lo, K), dtype=torch.uint8, device="cuda")
        g.weight_pack(wtype, raw, hi - lo, K, packed)
        ws = torch.empty(max(256, lib.b200_mul_mat_tp_workspace_size(wtype, M, hi - lo, K)), dtype=torch.uint8,
                         device="cuda")
        keep += [raw, packed, ws]
        rc = lib.b200_mul_mat_tp(wtype, g._ptr(packed), hi - lo, lo, K, g._ptr(a_dev), K, M, g._ptr(peer_dst), N, G, r,
                                 g._ptr(peer_flags), 1, g._ptr(ws), ws.numel(), g._ptr(err), None)
        assert rc == 0, rc
    for r in range(G):
        assert lib.b200_mul_mat_tp_finish(g._ptr(flags[r]), G, 1, g._ptr(err), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0, int(err.item())
    return [d.cpu().numpy() for d in dsts]


@pytest.mark.parametrize("wtype,K,N,M,G", [
    (1, 1024, 512, 256, 1),
    (12, 2048, 512, 512, 2),
    (12, 4096, 1024, 300, 4),
    (1, 512, 496, 64, 3),        # N = 31 groups of 16: uneven blocks, the last rank smaller
    (14, 1024, 768, 128, 2),
    (8, 2048, 384, 200, 2),
])
def test_tp_emulated_ranks_match_single_gpu(cuda, wtype, K, N, M, G):
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(K + N + M + G + wtype)
    w = _weights(rng, N, K, wtype)
    a = rng.standard_normal((M, K)).astype(np.float32)
    want = run_mul_mat(torch, wtype, w, N, K, a)
    got = _emulated(torch, g, wtype, w, N, K, a, G)
    ref = oracle.mul_mat(wtype, w, N, K, a)
    for r, d in enumerate(got):
        assert np.all(np.isfinite(d)), r
        if G == 1:
            assert np.array_equal(d.view(np.uint32), want.view(np.uint32))
        else:
            assert rel_err(d, want) <= 1e-5, (r, rel_err(d, want))
        assert rel_err(d, ref) <= TOL


def test_tp_rejects_bad_arguments(cuda):
    import torch
    import ggml_b200 as g
    lib = g.lib()
    x = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    p = g._ptr(x)
    # column offset not a multiple of 16, rank out of range, null pointers
    assert lib.b200_mul_mat_tp(1, p, 16, 8, 64, p, 64, 4, p, 64, 1, 0, p, 1, p, 1024, p, None) == g.B200_E_UNSUPPORTED
    assert lib.b200_mul_mat_tp(1, p, 16, 0, 64, p, 64, 4, p, 64, 1, 1, p, 1, p, 1024, p, None) == g.B200_E_INVALID
    assert lib.b200_mul_mat_tp(1, None, 16, 0, 64, p, 64, 4, p, 64, 1, 0, p, 1, p, 1024, p, None) == g.B200_E_INVALID
    assert lib.b200_mul_mat_tp_finish(None, 1, 1, p, None) == g.B200_E_INVALID


def _run_worker(nproc):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "tp_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=360)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert p.stdout.count("TP_OK") == nproc, p.stdout[-2000:]


def test_tp_one_rank(cuda):
    _run_worker(1)


def test_tp_two_gpus(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_worker(2)
