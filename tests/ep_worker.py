"""One rank of the expert-parallel MUL_MAT_ID check (launched by test_gpu_moe_ep.py through
torchrun, one or two GPUs): the NCCL path and the peer-memory path of ggml_b200.ep must both
reproduce, bit for bit, the single-GPU b200_mul_mat_id result for this rank's tokens over the
full expert stack."""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "ggml-rocket_b200"), os.path.join(ROOT, "tests")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import ggml_b200 as g  # noqa: E402
from ggml_b200 import quants  # noqa: E402
from ggml_b200.ep import ExpertParallelMulMatId  # noqa: E402


def ffn_case(rank, world, p2p, wt_gu, wt_down):
    """The expert FFN with its three projections run on the experts' owners
    (PeerExpertParallelMulMatId.ffn) against the single-GPU chain MUL_MAT_ID group (gate, up),
    SWIGLU, MUL_MAT_ID (down) over the full stacks: bit for bit, twice (the buffers are reused),
    and against the CPU oracle composed op by op within the MUL_MAT tolerance."""
    import oracle
    from conftest import rel_err
    E, n_used, H, F = 32, 8, 512, 768
    T = 80 + 29 * rank
    e_loc = E // world
    rng = np.random.default_rng(21 + wt_down)
    nat = {}
    for name, wt, N, K in (("gate", wt_gu, F, H), ("up", wt_gu, F, H), ("down", wt_down, H, F)):
        nat[name] = (wt, N, K, quants.quantize(wt, (rng.standard_normal((E * N, K)) * 0.02).astype(np.float32)))

    def pack(wt, raw_rows, rows, K):
        raw = torch.from_numpy(np.ascontiguousarray(raw_rows).reshape(-1)).cuda()
        out = torch.empty(g.weight_packed_size(wt, rows, K), dtype=torch.uint8, device="cuda")
        g.weight_pack(wt, raw, rows, K, out)
        return out

    full = {k: pack(wt, raw, E * N, K) for k, (wt, N, K, raw) in nat.items()}
    loc = {k: pack(wt, raw[rank * e_loc * N:(rank + 1) * e_loc * N], e_loc * N, K) for k, (wt, N, K, raw) in nat.items()}
    rng = np.random.default_rng(300 + rank)
    x_np = rng.standard_normal((T, 1, H)).astype(np.float32)
    ids_np = np.stack([rng.permutation(E)[:n_used] for _ in range(T)]).astype(np.int32)
    x, ids = torch.from_numpy(x_np).cuda(), torch.from_numpy(ids_np).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    yg = torch.empty((T, n_used, F), device="cuda")
    yu = torch.empty_like(yg)
    hh = torch.empty_like(yg)
    want = torch.full((T, n_used, H), float("nan"), device="cuda")
    ws = torch.zeros(max(g.mul_mat_id_workspace_size(H, F, E, n_used, T), g.mul_mat_id_workspace_size(F, H, E, n_used, T)),
                     dtype=torch.uint8, device="cuda")
    rcs = [g.mul_mat_id_group(wt_gu, [full["gate"], full["up"]], [F, F], H, E, x, H * 4, H * 4, 1, ids, 4, n_used * 4,
                              n_used, T, [yg, yu], [F * 4, F * 4], [n_used * F * 4] * 2, ws, err),
           g.swiglu(yg, yu, hh),
           g.mul_mat_id(wt_down, full["down"], F, H, E, hh, F * 4, n_used * F * 4, n_used, ids, 4, n_used * 4, n_used, T,
                        want, H * 4, n_used * H * 4, ws, err)]
    torch.cuda.synchronize()
    ok = rcs == [0, 0, 0] and int(err.item()) == 0
    for rep in range(2):
        perr = torch.zeros(1, dtype=torch.int32, device="cuda")
        p2p.ops.dev_err = perr
        got = p2p.ffn(wt_gu, loc["gate"], loc["up"], wt_down, loc["down"], H, F, E, x, ids, member=rep % 2)
        torch.cuda.synchronize()
        same = int(perr.item()) == 0 and bool(torch.equal(got, want))
        if not same:
            print(f"rank {rank} ffn {(wt_gu, wt_down)} rep {rep} mismatch: err {int(perr.item())} "
                  f"max {float((got - want).abs().max())}", flush=True)
        ok = ok and same
    # the chain itself against the oracle composed op by op (the first 24 tokens)
    n = 24
    og = oracle.mul_mat_id(wt_gu, nat["gate"][3].reshape(E, F, -1), H, F, E, x_np[:n], ids_np[:n])
    ou = oracle.mul_mat_id(wt_gu, nat["up"][3].reshape(E, F, -1), H, F, E, x_np[:n], ids_np[:n])
    oh = oracle.swiglu(og, ou).astype(np.float32)
    od = oracle.mul_mat_id(wt_down, nat["down"][3].reshape(E, H, -1), F, H, E, oh, ids_np[:n])
    e = rel_err(want[:n].cpu().numpy(), od)
    if e > 1e-2:
        print(f"rank {rank} ffn {(wt_gu, wt_down)} oracle rel err {e}", flush=True)
        ok = False
    return ok


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ok = True
    from ggml_b200.ep import PeerExpertParallelMulMatId
    p2p = PeerExpertParallelMulMatId(n_tokens_max=256, n_used=8, K_max=2048, N_max=768)
    for (wtype, K, N, E, n_used, ne11, T) in [(12, 2048, 768, 32, 8, 1, 256), (12, 768, 256, 32, 8, 8, 96 + 31 * rank)]:
        rng = np.random.default_rng(7)
        w = (rng.standard_normal((E * N, K)) * 0.02).astype(np.float32)
        native = quants.quantize(wtype, w)
        e_loc = E // world
        rpe = native.shape[0] // E

        def pack(nat, rows):
            raw = torch.from_numpy(np.ascontiguousarray(nat).reshape(-1)).cuda()
            out = torch.empty(g.weight_packed_size(wtype, rows, K), dtype=torch.uint8, device="cuda")
            g.weight_pack(wtype, raw, rows, K, out)
            return out

        local_stack = pack(native[rank * e_loc * rpe:(rank + 1) * e_loc * rpe], e_loc * N)
        rng = np.random.default_rng(100 + rank)
        b = torch.from_numpy(rng.standard_normal((T, ne11, K)).astype(np.float32)).cuda()
        ids = torch.from_numpy(np.stack([rng.permutation(E)[:n_used] for _ in range(T)]).astype(np.int32)).cuda()
        dst = torch.full((T, n_used, N), float("nan"), device="cuda")
        ep = ExpertParallelMulMatId()
        ep(wtype, local_stack, K, N, E, b, ne11, ids, dst)
        full = pack(native, E * N)
        want = torch.full_like(dst, float("nan"))
        ws = torch.zeros(g.mul_mat_id_workspace_size(K, N, E, n_used, T), dtype=torch.uint8, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        rc = g.mul_mat_id(wtype, full, K, N, E, b, K * 4, ne11 * K * 4, ne11, ids, 4, n_used * 4, n_used, T,
                          want, N * 4, n_used * N * 4, ws, err)
        torch.cuda.synchronize()
        same = rc == 0 and int(err.item()) == 0 and bool(torch.equal(dst, want))
        if not same:
            print(f"rank {rank} case {(wtype, K, N, E, n_used, ne11, T)} mismatch: "
                  f"{float((dst - want).abs().max())}", flush=True)
        # the same op with both exchanges over peer memory (twice: the buffers are reused)
        for rep in range(2):
            perr = torch.zeros(1, dtype=torch.int32, device="cuda")
            p2p.ops.dev_err = perr
            got = p2p(wtype, local_stack, K, N, E, b, ne11, ids)
            torch.cuda.synchronize()
            p_same = int(perr.item()) == 0 and bool(torch.equal(got, want))
            if not p_same:
                print(f"rank {rank} p2p case {(wtype, K, N, E, n_used, ne11, T)} rep {rep} mismatch: err "
                      f"{int(perr.item())} max {float((got - want).abs().max())}", flush=True)
            same = same and p_same
        # a two-member group (gate and up over the same rows): the second stack is this rank's
        # experts of a second weight; each member must equal its own single-GPU op
        w2 = (np.random.default_rng(8).standard_normal((E * N, K)) * 0.02).astype(np.float32)
        native2 = quants.quantize(wtype, w2)
        local2 = pack(native2[rank * e_loc * rpe:(rank + 1) * e_loc * rpe], e_loc * N)
        want2 = torch.full_like(dst, float("nan"))
        rc = g.mul_mat_id(wtype, pack(native2, E * N), K, N, E, b, K * 4, ne11 * K * 4, ne11, ids, 4, n_used * 4,
                          n_used, T, want2, N * 4, n_used * N * 4, ws, err)
        perr = torch.zeros(1, dtype=torch.int32, device="cuda")
        p2p.ops.dev_err = perr
        g1, g2 = p2p.grouped(wtype, [local_stack, local2], K, [N, N], E, b, ne11, ids)
        torch.cuda.synchronize()
        g_same = rc == 0 and int(perr.item()) == 0 and bool(torch.equal(g1, want)) and bool(torch.equal(g2, want2))
        if not g_same:
            print(f"rank {rank} p2p group case {(wtype, K, N, E, n_used, ne11, T)} mismatch: err {int(perr.item())}",
                  flush=True)
        ok = ok and same and g_same
    ok = ffn_case(rank, world, p2p, 12, 12) and ok
    ok = ffn_case(rank, world, p2p, 12, 14) and ok
    p2p.close()
    dist.barrier()
    dist.destroy_process_group()
    if ok:
        print("EP_OK", flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
