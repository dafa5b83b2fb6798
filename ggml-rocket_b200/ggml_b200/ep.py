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


class PeerExpertParallelMulMatId:
    """The same op as ExpertParallelMulMatId with both exchanges done by the library's kernels
    over NVLink peer memory (b200_moe_ep_p2p_*): the dispatch pushes every packed row into its
    owner's receive buffer, the owner's grouped GEMM stores every output row into its home rank's
    return buffer, and flags with a per-op epoch order the steps -- no collective call and no
    host synchronisation per op. torch.distributed is used once, at construction, to exchange
    the buffers' IPC handles.

    Sizes are fixed at construction: at most n_tokens_max tokens per rank, n_used slots, K_max
    input and N_max output columns over the ops it will run. __call__ returns a view of the
    return buffer holding dst [n_tokens, n_used, N] (valid until the next call), and copies it
    into dst when one is given."""

    def __init__(self, n_tokens_max, n_used, K_max, N_max, group=None, device=None, ops=None, n_members_max=2):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.ops = ops if ops is not None else DeviceOps()
        self.n_used, self.K_max, self.N_max = n_used, K_max, N_max
        self.cap = n_tokens_max * n_used
        G, dev = self.G, self.dev
        self.recv_a16 = torch.zeros((G, self.cap, K_max), dtype=torch.float16, device=dev)
        self.recv_meta = torch.zeros((G, self.cap, n_used + 3), dtype=torch.int32, device=dev)
        # one return buffer per member of a group op (gate and up share their rows)
        self.n_members_max = n_members_max
        self.rets = torch.zeros((n_members_max, n_tokens_max, n_used, N_max), dtype=torch.float32, device=dev)
        self.ret = self.rets[0]
        self.flags = torch.zeros((2 * G, 4), dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        mine = [self._export(t) for t in (self.recv_a16, self.recv_meta, self.rets, self.flags)]
        allh = [None] * G
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        ptrs = [[0] * G for _ in range(4)]
        for q in range(G):
            for b, t in enumerate((self.recv_a16, self.recv_meta, self.rets, self.flags)):
                if q == self.rank:
                    ptrs[b][q] = t.data_ptr()
                else:
                    handle, off = allh[q][b]
                    base = g._c.c_void_p(0)
                    hb = g._c.create_string_buffer(handle, len(handle))
                    g.check(g.lib().b200_ep_shared_open(hb, g._c.byref(base)), "ep_shared_open")
                    self._opened.append(base.value)
                    ptrs[b][q] = base.value + off
        self.peer = [torch.tensor(p, dtype=torch.int64, device=dev) for p in ptrs]
        member_bytes = self.rets[0].numel() * 4
        self.peer_rets = [torch.tensor([p + m * member_bytes for p in ptrs[2]], dtype=torch.int64, device=dev)
                          for m in range(n_members_max)]
        self.epoch = 0
        self.last_stats = {}
        dist.barrier(group=group)

    @staticmethod
    def _export(t):
        h = g._c.create_string_buffer(64)
        off = g._c.c_size_t(0)
        g.check(g.lib().b200_ep_shared_export(g._ptr(t), h, g._c.byref(off)), "ep_shared_export")
        return (h.raw, off.value)

    def close(self):
        """Unmap the other ranks' buffers (collective: every rank calls it)."""
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        for base in self._opened:
            g.lib().b200_ep_shared_close(g._c.c_void_p(base))
        self._opened = []

    def __call__(self, wtype, local_stack, K, N, n_expert, b, ne11, ids, dst=None, stream=None, member=0):
        out = self.grouped(wtype, [local_stack], K, [N], n_expert, b, ne11, ids, stream=stream, member0=member)[0]
        if dst is not None:
            dst.copy_(out)
        return out

    def grouped(self, wtype, local_stacks, K, Ns, n_expert, b, ne11, ids, stream=None, member0=0):
        """Several MUL_MAT_IDs over the same b and ids (a layer's gate and up): the rows are
        dispatched and pushed once, each owner routes and gathers them once and runs one grouped
        GEMM per stack. Returns one view of the return buffers per member, [n_tokens, n_used, N]:
        members member0, member0 + 1, ... of the exchange's return buffers, so that ops of a layer
        given distinct members keep their results side by side without copies."""
        G, ops = self.G, self.ops
        n_tokens, n_used = ids.shape
        nm = len(local_stacks)
        if n_expert % G or n_used != self.n_used or K > self.K_max or max(Ns) > self.N_max or \
                n_tokens * n_used > self.cap or member0 < 0 or member0 + nm > self.n_members_max:
            raise ValueError("op outside the sizes this exchange was built for")
        n_local = n_expert // G
        self.epoch += 1
        d = ops.dispatch(ids, b, ne11, n_expert, G, K, stream=stream)
        err = ops._err(self.dev)
        lib = g.lib()
        g.check(lib.b200_moe_ep_p2p_push(
            g._ptr(d.a16), g._ptr(d.scale), g._ptr(d.hdr), g._ptr(d.row_tok), g._ptr(d.counts), G, self.rank,
            n_used, K, self.cap, g._ptr(self.peer[0]), g._ptr(self.peer[1]), g._ptr(self.peer[3]), self.epoch,
            n_tokens * n_used, g._stream(stream)), "moe_ep_p2p_push")
        ws_bytes = lib.b200_moe_ep_p2p_expert_workspace_size(G, self.cap, K, n_local, n_used)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.dev)
        P = g._c.c_void_p * nm
        I = g._c.c_int64 * nm
        g.check(lib.b200_moe_ep_p2p_expert_group(
            nm, wtype, P(*[g._ptr(t) for t in local_stacks]), I(*Ns), K, n_local, self.rank * n_local,
            g._ptr(self.recv_a16), g._ptr(self.recv_meta), g._ptr(self.flags), G, self.rank, n_used, self.cap,
            n_tokens * n_used, P(*[g._ptr(self.peer_rets[member0 + m]) for m in range(nm)]), I(*([self.N_max * 4] * nm)),
            I(*([n_used * self.N_max * 4] * nm)), g._ptr(self.peer[3]), self.epoch, g._ptr(ws), ws_bytes,
            g._ptr(err), g._stream(stream)), "moe_ep_p2p_expert_group")
        g.check(lib.b200_moe_ep_p2p_finish(g._ptr(self.flags), G, self.epoch, g._ptr(err), g._stream(stream)),
                "moe_ep_p2p_finish")
        return [self.rets[member0 + m][:n_tokens, :, :Ns[m]] for m in range(nm)]

    def ffn(self, wtype_gate_up, gate_stack, up_stack, wtype_down, down_stack, H, F, n_expert, x, ids, stream=None,
            member=0):
        """A MoE block's expert FFN, down(swiglu(gate(x), up(x))) per (token, slot), with the
        three expert projections run where the experts are (b200_moe_ep_p2p_expert_ffn): x's
        rows are dispatched and pushed once, each owner keeps gate, up and h in its own memory,
        and only the down projection's rows come back. x is [n_tokens, 1, H] (or [n_tokens, H]);
        gate_stack / up_stack are this rank's experts of [F, H] weights, down_stack of [H, F].
        Returns a view of return buffer `member`, [n_tokens, n_used, H], valid until that member
        is written again; it equals the single-GPU chain MUL_MAT_ID, MUL_MAT_ID, SWIGLU,
        MUL_MAT_ID bit for bit."""
        G, ops = self.G, self.ops
        n_tokens, n_used = ids.shape
        if x.dim() == 2:
            x = x.view(n_tokens, 1, H)
        if n_expert % G or n_used != self.n_used or H > self.K_max or H > self.N_max or \
                n_tokens * n_used > self.cap or not 0 <= member < self.n_members_max:
            raise ValueError("op outside the sizes this exchange was built for")
        n_local = n_expert // G
        self.epoch += 1
        d = ops.dispatch(ids, x, 1, n_expert, G, H, stream=stream)
        err = ops._err(self.dev)
        lib = g.lib()
        g.check(lib.b200_moe_ep_p2p_push(
            g._ptr(d.a16), g._ptr(d.scale), g._ptr(d.hdr), g._ptr(d.row_tok), g._ptr(d.counts), G, self.rank,
            n_used, H, self.cap, g._ptr(self.peer[0]), g._ptr(self.peer[1]), g._ptr(self.peer[3]), self.epoch,
            n_tokens * n_used, g._stream(stream)), "moe_ep_p2p_push")
        ws_bytes = lib.b200_moe_ep_p2p_ffn_workspace_size(G, self.cap, H, F, n_local, n_used)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.dev)
        g.check(lib.b200_moe_ep_p2p_expert_ffn(
            wtype_gate_up, g._ptr(gate_stack), g._ptr(up_stack), wtype_down, g._ptr(down_stack), H, F, n_local,
            self.rank * n_local, g._ptr(self.recv_a16), g._ptr(self.recv_meta), g._ptr(self.flags), G, self.rank,
            n_used, self.cap, n_tokens * n_used, g._ptr(self.peer_rets[member]), self.N_max * 4,
            n_used * self.N_max * 4, g._ptr(self.peer[3]), self.epoch, g._ptr(ws), ws_bytes, g._ptr(err),
            g._stream(stream)), "moe_ep_p2p_expert_ffn")
        g.check(lib.b200_moe_ep_p2p_finish(g._ptr(self.flags), G, self.epoch, g._ptr(err), g._stream(stream)),
                "moe_ep_p2p_finish")
        return self.rets[member][:n_tokens, :, :H]
