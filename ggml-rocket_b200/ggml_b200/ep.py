"""Expert-parallel MUL_MAT_ID over several GPUs: one process per GPU, NCCL all-to-all.

The reference runs MUL_MAT_ID (ggml-rocket.cpp:6692-6944) on one device. Here the experts of
one op are split across the ranks of a process group in contiguous blocks of E / n_ranks,
each rank keeps its own tokens, and an op is

    dispatch  (home rank, b200_moe_ep_dispatch)   one fp16 row per (token, b row, owner rank)
    exchange  all_to_all of the row counts, then of rows, row scales and slot-mask headers
    expert    (owner rank, b200_moe_ep_expert)    grouped tcgen05 GEMM over the received rows
    exchange  all_to_all of the f32 output rows back to their home ranks
    combine   (home rank, b200_moe_ep_combine)    scatter into dst[:, slot, token]

A token routed to several experts of one rank crosses the link once (its slot mask names the
slots); outputs return as f32, so every dst row equals the single-GPU op's.

Only the collectives are torch.distributed (plumbing); the device work is the library's. The
`ops` object supplies the three local steps, so the exchange logic also runs with host stand-ins
(tests run it as gloo ranks on the CPU).
"""
from dataclasses import dataclass

import torch
import torch.distributed as dist

import ggml_b200 as g


@dataclass
class Dispatched:
    a16: torch.Tensor        # [max_rows, K] fp16 send rows, grouped by destination rank
    scale: torch.Tensor      # [max_rows] f32
    hdr: torch.Tensor        # [max_rows, n_used + 1] int32 {slot mask, ids of the token}
    row_tok: torch.Tensor    # [max_rows] int32
    row_slot: torch.Tensor   # [max_rows] int32
    row_ret: torch.Tensor    # [max_rows] int32 first return row of each send row
    counts: torch.Tensor     # [2 * n_ranks + 2] int32: rows / return rows per destination, totals


class DeviceOps:
    """The three rank-local steps on this process's GPU, through the C ABI."""

    def __init__(self, dev_err=None):
        self.dev_err = dev_err

    def _err(self, device):
        if self.dev_err is None:
            self.dev_err = torch.zeros(1, dtype=torch.int32, device=device)
        return self.dev_err

    def dispatch(self, ids, b, ne11, n_expert, n_ranks, K, stream=None):
        n_tokens, n_used = ids.shape
        dev = b.device
        max_rows = n_tokens * n_used
        d = Dispatched(
            a16=torch.empty((max_rows, K), dtype=torch.float16, device=dev),
            scale=torch.empty(max_rows, dtype=torch.float32, device=dev),
            hdr=torch.empty((max_rows, n_used + 1), dtype=torch.int32, device=dev),
            row_tok=torch.empty(max_rows, dtype=torch.int32, device=dev),
            row_slot=torch.empty(max_rows, dtype=torch.int32, device=dev),
            row_ret=torch.empty(max_rows, dtype=torch.int32, device=dev),
            counts=torch.zeros(2 * n_ranks + 2, dtype=torch.int32, device=dev))
        scratch = torch.empty(max(256, g.lib().b200_moe_ep_dispatch_scratch_size(n_tokens, ne11, n_ranks)),
                              dtype=torch.uint8, device=dev)
        # ids [n_tokens, n_used] as ggml stores it: the slot stride is ids_nb0, the token stride ids_nb1
        g.check(g.lib().b200_moe_ep_dispatch(
            g._ptr(ids), ids.stride(1) * 4, ids.stride(0) * 4, n_used, n_tokens, n_expert, n_ranks,
            g._ptr(b), b.stride(1) * 4, b.stride(0) * 4, ne11, K,
            g._ptr(d.a16), g._ptr(d.scale), g._ptr(d.hdr), g._ptr(d.row_tok), g._ptr(d.row_slot),
            g._ptr(d.row_ret), g._ptr(d.counts), g._ptr(scratch), scratch.numel(), g._ptr(self._err(dev)),
            g._stream(stream)), "moe_ep_dispatch")
        return d

    def expert(self, wtype, local_stack, K, N, n_local, expert0, a16, scale, hdr, n_pairs, stream=None):
        n_rows, n_used = hdr.shape[0], hdr.shape[1] - 1
        dev = local_stack.device
        ret = torch.empty((max(n_pairs, 1), N), dtype=torch.float32, device=dev)
        if n_rows == 0:
            return ret[:0]
        ws = torch.empty(g.lib().b200_moe_ep_expert_workspace_size(K, n_local, n_used, n_rows),
                         dtype=torch.uint8, device=dev)
        g.check(g.lib().b200_moe_ep_expert(
            wtype, g._ptr(local_stack), K, N, n_local, expert0, g._ptr(a16), g._ptr(scale), g._ptr(hdr), n_rows,
            n_used, n_pairs, g._ptr(ret), g._ptr(ws), ws.numel(), g._ptr(self._err(dev)), g._stream(stream)),
            "moe_ep_expert")
        return ret[:n_pairs]

    def combine(self, ret, N, d, n_ranks, dst, stream=None):
        n_used = d.hdr.shape[1] - 1
        g.check(g.lib().b200_moe_ep_combine(
            g._ptr(ret) if ret.numel() else None, N, g._ptr(d.hdr), n_used, g._ptr(d.row_tok), g._ptr(d.row_ret),
            g._ptr(d.counts), n_ranks, d.row_tok.numel(), g._ptr(dst), dst.stride(1) * 4, dst.stride(0) * 4,
            g._stream(stream)), "moe_ep_combine")


def _a2a(out, inp, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


class ExpertParallelMulMatId:
    """dst[:, s, t] = as[:, :, ids[s, t]] . b[:, s % ne11, t] with the experts split over a group.

    Tensors are this rank's: b [n_tokens, ne11, K] f32, ids [n_tokens, n_used] int32 (global
    expert ids), dst [n_tokens, n_used, N] f32, and local_stack the packed weights of experts
    [rank * E/G, (rank+1) * E/G) as one [E/G * N, K] matrix (b200_weight_pack layout). Every rank
    calls it in the same order (it runs collectives)."""

    def __init__(self, group=None, ops=None):
        self.group = group
        self.ops = ops if ops is not None else DeviceOps()
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.last_stats = {}

    def __call__(self, wtype, local_stack, K, N, n_expert, b, ne11, ids, dst):
        G, ops = self.G, self.ops
        if n_expert % G:
            raise ValueError(f"{n_expert} experts do not split over {G} ranks")
        n_local = n_expert // G
        d = ops.dispatch(ids, b, ne11, n_expert, G, K)
        counts = d.counts.to("cpu", torch.int64)
        rows_to, pairs_to = counts[:G], counts[G:2 * G]
        comm_dev = d.counts.device
        cnt_in = torch.stack([rows_to, pairs_to], 1).reshape(-1).to(comm_dev)
        cnt_out = torch.empty_like(cnt_in)
        _a2a(cnt_out, cnt_in, None, None, self.group)
        cnt_out = cnt_out.cpu().reshape(G, 2)
        rows_from, pairs_from = cnt_out[:, 0].tolist(), cnt_out[:, 1].tolist()
        rows_to, pairs_to = rows_to.tolist(), pairs_to.tolist()
        S, R = sum(rows_to), sum(rows_from)
        recv_a16 = torch.empty((R, d.a16.shape[1]), dtype=d.a16.dtype, device=d.a16.device)
        recv_scale = torch.empty(R, dtype=d.scale.dtype, device=d.scale.device)
        recv_hdr = torch.empty((R, d.hdr.shape[1]), dtype=d.hdr.dtype, device=d.hdr.device)
        _a2a(recv_a16, d.a16[:S], rows_from, rows_to, self.group)
        _a2a(recv_scale, d.scale[:S], rows_from, rows_to, self.group)
        _a2a(recv_hdr, d.hdr[:S], rows_from, rows_to, self.group)
        P_in = sum(pairs_from)
        ret = ops.expert(wtype, local_stack, K, N, n_local, self.rank * n_local, recv_a16, recv_scale, recv_hdr,
                         P_in)
        home = torch.empty((sum(pairs_to), N), dtype=torch.float32, device=ret.device)
        _a2a(home, ret, pairs_to, pairs_from, self.group)
        ops.combine(home, N, d, G, dst)
        self.last_stats = {"rows_sent": S, "rows_received": R, "return_rows": P_in,
                           "wire_bytes_out": S * (d.a16.shape[1] * d.a16.element_size() + 4 + 4 * d.hdr.shape[1])
                           + P_in * N * 4}
        return dst
