"""One rank of the N-sharded MUL_MAT check (launched by test_gpu_mul_mat_tp.py through torchrun,
one or two GPUs): ggml_b200.tp.PeerShardedMulMat, each rank holding a row block of the weight,
must give every rank the single-GPU b200_mul_mat result over the whole weight (up to the order
of the fp32 K-sums), twice in a row (the epoch flags and buffer reuse)."""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "ggml-rocket_b200"), os.path.join(ROOT, "tests")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import ggml_b200 as g  # noqa: E402
import oracle  # noqa: E402
from conftest import rel_err  # noqa: E402
from ggml_b200.tp import PeerShardedMulMat, shard_rows  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ok = True
    tp = PeerShardedMulMat(M_max=512, N_max=4096)
    for rep in range(2):
        for (wtype, K, N, M) in [(12, 4096, 4096, 512), (1, 2048, 1024, 200), (14, 1024, 2048, 96)]:
            rng = np.random.default_rng(11 + wtype + rep)
            w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
            native = oracle.fp16_bits(w).view(np.uint8).reshape(N, K * 2) if wtype == 1 else oracle.quantize(wtype, w)
            a = rng.standard_normal((M, K)).astype(np.float32)      # the same activation on every rank
            lo, hi = shard_rows(N, world, rank)
            raw = torch.from_numpy(np.ascontiguousarray(native[lo:hi]).reshape(-1)).cuda()
            shard = torch.empty(g.weight_packed_size(wtype, hi - lo, K), dtype=torch.uint8, device="cuda")
            g.weight_pack(wtype, raw, hi - lo, K, shard)
            a_dev = torch.from_numpy(a).cuda()
            got = tp(wtype, shard, N, K, a_dev, M).clone()
            full_raw = torch.from_numpy(np.ascontiguousarray(native).reshape(-1)).cuda()
            full = torch.empty(g.weight_packed_size(wtype, N, K), dtype=torch.uint8, device="cuda")
            g.weight_pack(wtype, full_raw, N, K, full)
            want = torch.full((M, N), float("nan"), device="cuda")
            ws = torch.empty(g.mul_mat_workspace_size(M, N, K, wtype), dtype=torch.uint8, device="cuda")
            err = torch.zeros(1, dtype=torch.int32, device="cuda")
            g.mul_mat(wtype, full, N, K, a_dev, M, want, ws, err)
            torch.cuda.synchronize()
            e = rel_err(got.cpu().numpy(), want.cpu().numpy())
            if int(err.item()) != 0 or int(tp.err.item()) != 0 or not (e <= 1e-5):
                ok = False
                print(f"rank {rank} rep {rep} case {(wtype, K, N, M)}: rel err {e} err {int(err.item())} "
                      f"{int(tp.err.item())}", flush=True)
    tp.close()
    dist.barrier()
    dist.destroy_process_group()
    if ok:
        print("TP_OK", flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
