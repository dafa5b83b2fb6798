"""Expert-parallel MUL_MAT_ID: the exchange logic of ggml_b200.ep as gloo ranks on the CPU.

ExpertParallelMulMatId runs unchanged; its three rank-local steps are host stand-ins (HostOps,
below) that follow the device kernels' contract: send rows grouped by destination rank, then
token, then b row, each with a slot mask and the token's ids; return rows in received order with
a row's slots ascending. Every rank's dst must equal the single-process oracle's MUL_MAT_ID over
the full expert stack (the reference op, ggml-rocket.cpp:6692-6944), for ne11 = 1 (one row per
token and owner rank, deduplicated across slots) and ne11 = n_used (one row per slot), uneven
token counts, and 2 or 4 ranks.
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class HostOps:
    """CPU stand-ins for b200_moe_ep_dispatch / _expert / _combine (same layouts and order)."""

    def __init__(self, w_local):
        self.w_local = w_local          # f32 [n_local, N, K], this rank's experts, decoded

    def dispatch(self, ids, b, ne11, n_expert, n_ranks, K):
        import torch
        from ggml_b200.ep import Dispatched
        ids_n = ids.numpy()
        b_n = b.numpy()
        T, n_used = ids_n.shape
        e_loc = n_expert // n_ranks
        rows = []
        for d in range(n_ranks):
            for t in range(T):
                for j in range(ne11):
                    m = 0
                    for s in range(j, n_used, ne11):
                        if ids_n[t, s] // e_loc == d:
                            m |= 1 << s
                    if m:
                        rows.append((d, t, j, m))
        max_rows = T * n_used
        a16 = np.zeros((max_rows, K), np.float32)
        hdr = np.zeros((max_rows, n_used + 1), np.int32)
        tok = np.zeros(max_rows, np.int32)
        slot = np.zeros(max_rows, np.int32)
        ret = np.zeros(max_rows, np.int32)
        counts = np.zeros(2 * n_ranks + 2, np.int32)
        q = 0
        for p, (d, t, j, m) in enumerate(rows):
            a16[p] = b_n[t, j]
            hdr[p, 0] = m
            hdr[p, 1:] = ids_n[t]
            tok[p] = t
            slot[p] = (m & -m).bit_length() - 1
            ret[p] = q
            q += bin(m).count("1")
            counts[d] += 1
            counts[n_ranks + d] += bin(m).count("1")
        counts[2 * n_ranks] = len(rows)
        counts[2 * n_ranks + 1] = q
        T_ = torch.from_numpy
        return Dispatched(a16=T_(a16), scale=torch.ones(max_rows), hdr=T_(hdr), row_tok=T_(tok), row_slot=T_(slot),
                          row_ret=T_(ret), counts=T_(counts))

    def expert(self, wtype, local_stack, K, N, n_local, expert0, a16, scale, hdr, n_pairs):
        import torch
        out = []
        for r in range(hdr.shape[0]):
            m = int(hdr[r, 0])
            for s in range(32):
                if m >> s & 1:
                    x = int(hdr[r, 1 + s]) - expert0
                    assert 0 <= x < n_local
                    out.append(self.w_local[x].astype(np.float64) @ (a16[r].numpy().astype(np.float64) * float(scale[r])))
        assert len(out) == n_pairs
        return torch.from_numpy(np.array(out, dtype=np.float32).reshape(n_pairs, N))

    def combine(self, ret, N, d, n_ranks, dst):
        S = int(d.counts[2 * n_ranks])
        for p in range(S):
            t, m, k = int(d.row_tok[p]), int(d.hdr[p, 0]), int(d.row_ret[p])
            for s in range(32):
                if m >> s & 1:
                    dst[t, s] = ret[k]
                    k += 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, case, q):
    try:
        sys.path[:0] = [ROOT, os.path.join(ROOT, "ggml-rocket_b200")]
        import datetime
        import torch
        import torch.distributed as dist
        import oracle
        from ggml_b200.ep import ExpertParallelMulMatId
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        wtype, K, N, E, n_used, ne11, tokens = case
        rng = np.random.default_rng(1234)                     # the same weights on every rank
        w = (rng.standard_normal((E * N, K)) * 0.02).astype(np.float32)
        raw = oracle.quantize(wtype, w)
        deq = oracle.dequantize(wtype, raw, K).reshape(E, N, K)
        e_loc = E // world
        rng = np.random.default_rng(99 + rank)                # this rank's tokens
        T = tokens[rank]
        b = rng.standard_normal((T, ne11, K)).astype(np.float32)
        ids = np.stack([rng.permutation(E)[:n_used] for _ in range(T)]).astype(np.int32)
        ep = ExpertParallelMulMatId(ops=HostOps(deq[rank * e_loc:(rank + 1) * e_loc]))
        dst = torch.full((T, n_used, N), float("nan"))
        ep(wtype, None, K, N, E, torch.from_numpy(b), ne11, torch.from_numpy(ids), dst)
        want = oracle.mul_mat_id(wtype, raw.reshape(E, N, -1), K, N, E, b, ids)
        got = dst.numpy()
        err = float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, bool(np.all(np.isfinite(got))), err, ep.last_stats))
    except Exception as e:   # report, do not hang the parent
        q.put((rank, False, repr(e), {}))


@pytest.mark.parametrize("world,case", [
    (2, (8, 256, 64, 8, 3, 1, (20, 13))),
    (2, (8, 256, 64, 8, 3, 3, (17, 9))),
    (4, (8, 256, 32, 16, 4, 1, (7, 11, 1, 5))),
])
def test_ep_exchange_matches_oracle(world, case):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, finite, err, stats in sorted(results, key=lambda x: x[0]):
        assert finite, (rank, err)
        assert isinstance(err, float) and err <= 1e-5, (rank, err)
    if case[5] == 1:
        # ne11 = 1: rows are deduplicated per (token, owner rank), so fewer rows than pairs cross
        tot = [r[3] for r in results]
        assert sum(s["rows_sent"] for s in tot) < sum(s["return_rows"] for s in tot)
