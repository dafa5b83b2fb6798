"""Expert-parallel MUL_MAT_ID kernels (b200_moe_ep_dispatch / _expert / _combine) on the GPU.

The exchanges are emulated inside one process (rank r's send rows for rank q are handed to q
by slicing), so the G-rank kernel contract is checked on a single B200: every rank's dst must
equal the single-GPU b200_mul_mat_id result for its tokens over the full expert stack, and the
CPU oracle within the MUL_MAT tolerance. The op also runs as torchrun ranks (ep_worker.py)
through both exchange paths -- NCCL all-to-all and the kernels' own stores into peer memory --
with one rank always and with two when two GPUs are present.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import ROOT, rel_err
from ggml_b200 import quants

pytestmark = pytest.mark.gpu


def _pack(torch, g, wtype, native, rows, K):
    raw = torch.from_numpy(np.ascontiguousarray(native).reshape(-1)).cuda()
    packed = torch.empty(g.weight_packed_size(wtype, rows, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(wtype, raw, rows, K, packed)
    return packed


def _single_gpu(torch, g, wtype, full_packed, K, N, E, b, ids):
    T, ne11, _ = b.shape
    n_used = ids.shape[1]
    bd, idd = torch.from_numpy(b).cuda(), torch.from_numpy(ids).cuda()
    dst = torch.full((T, n_used, N), float("nan"), device="cuda")
    ws = torch.zeros(g.mul_mat_id_workspace_size(K, N, E, n_used, T), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = g.mul_mat_id(wtype, full_packed, K, N, E, bd, K * 4, ne11 * K * 4, ne11, idd, 4, n_used * 4, n_used, T,
                      dst, N * 4, n_used * N * 4, ws, err)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    return dst.cpu().numpy()


def loopback(torch, g, wtype, native, K, N, E, G, bs, idss):
    """Run the G-rank op in one process; returns each rank's dst and the dispatch counts."""
    from ggml_b200.ep import DeviceOps
    e_loc = E // G
    rows_per_e = native.shape[0] // E
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops = DeviceOps(err)
    stacks = [_pack(torch, g, wtype, native[q * e_loc * rows_per_e:(q + 1) * e_loc * rows_per_e], e_loc * N, K)
              for q in range(G)]
    disp, cnts = [], []
    for r in range(G):
        ne11 = bs[r].shape[1]
        d = ops.dispatch(torch.from_numpy(idss[r]).cuda(), torch.from_numpy(bs[r]).cuda(), ne11, E, G, K)
        disp.append(d)
        cnts.append(d.counts.cpu().numpy().astype(np.int64))
    rets = []
    for q in range(G):
        parts_a, parts_s, parts_h, npairs = [], [], [], 0
        for r in range(G):
            o = int(cnts[r][:q].sum())
            n = int(cnts[r][q])
            parts_a.append(disp[r].a16[o:o + n])
            parts_s.append(disp[r].scale[o:o + n])
            parts_h.append(disp[r].hdr[o:o + n])
            npairs += int(cnts[r][G + q])
        a16, sc, hdr = torch.cat(parts_a), torch.cat(parts_s), torch.cat(parts_h)
        rets.append(ops.expert(wtype, stacks[q], K, N, e_loc, q * e_loc, a16.contiguous(), sc.contiguous(),
                               hdr.contiguous(), npairs))
    outs = []
    for r in range(G):
        parts = []
        for q in range(G):
            o = sum(int(cnts[s][G + q]) for s in range(r))
            parts.append(rets[q][o:o + int(cnts[r][G + q])])
        home = torch.cat(parts).contiguous()
        T, n_used = idss[r].shape
        dst = torch.full((T, n_used, N), float("nan"), device="cuda")
        ops.combine(home, N, disp[r], G, dst)
        outs.append(dst)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return [o.cpu().numpy() for o in outs], cnts


@pytest.mark.parametrize("wtype,K,N,E,G,n_used,ne11,tokens", [
    (12, 512, 128, 16, 2, 4, 1, (64, 37)),
    (12, 512, 128, 16, 2, 4, 4, (40, 21)),
    (8, 256, 64, 8, 4, 2, 1, (33, 1, 17, 8)),
    (1, 256, 96, 8, 2, 2, 2, (48, 30)),
    (12, 2048, 768, 32, 4, 8, 1, (128, 96, 64, 100)),
])
def test_ep_loopback_matches_single_gpu(cuda, wtype, K, N, E, G, n_used, ne11, tokens):
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(K + N + E + G + ne11 + wtype)
    w = (rng.standard_normal((E * N, K)) * 0.02).astype(np.float32)
    native = quants.quantize(wtype, w) if wtype != 1 else w.astype(np.float16).view(np.uint8).reshape(E * N, -1)
    bs = [rng.standard_normal((T, ne11, K)).astype(np.float32) for T in tokens]
    idss = [np.stack([rng.permutation(E)[:n_used] for _ in range(T)]).astype(np.int32) for T in tokens]
    outs, cnts = loopback(torch, g, wtype, native, K, N, E, G, bs, idss)
    full = _pack(torch, g, wtype, native, E * N, K)
    for r in range(G):
        want = _single_gpu(torch, g, wtype, full, K, N, E, bs[r], idss[r])
        assert np.all(np.isfinite(outs[r]))
        assert np.array_equal(outs[r], want), float(np.max(np.abs(outs[r] - want)))
        ref = oracle.mul_mat_id(wtype, native.reshape(E, N, -1), K, N, E, bs[r], idss[r])
        assert rel_err(outs[r], ref) <= 1e-2
        # bookkeeping: every (token, slot) pair returns exactly once
        assert int(cnts[r][2 * G + 1]) == tokens[r] * n_used
        if ne11 == 1:
            assert int(cnts[r][2 * G]) <= tokens[r] * min(n_used, G)


def test_ep_bad_expert_id_sets_error(cuda):
    import torch
    import ggml_b200 as g
    from ggml_b200.ep import DeviceOps
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops = DeviceOps(err)
    ids = torch.tensor([[0, 1], [2, 99]], dtype=torch.int32, device="cuda")
    b = torch.randn(2, 1, 256, device="cuda")
    d = ops.dispatch(ids, b, 1, 8, 2, 256)
    torch.cuda.synchronize()
    assert int(err.item()) == 100
    assert int(d.counts[-2].item()) == 0


def _run_worker(nproc):
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(ROOT, "tests", "ep_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=360)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert p.stdout.count("EP_OK") == nproc, p.stdout[-2000:]


def test_ep_one_rank_nccl_and_peer_paths(cuda):
    """Both exchange paths with a single rank (every expert local): the push, flag, route and
    epilogue-store kernels of the peer-memory path run on one GPU."""
    _run_worker(1)


def test_ep_two_gpus_nccl_and_peer_paths(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_worker(2)
