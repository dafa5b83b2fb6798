"""MUL_MAT with the weight rows split across GPUs (N-sharded), one process per GPU.

Rank r of G holds rows [r*N/G, (r+1)*N/G) of an [N, K] weight (packed with b200_weight_pack)
and the whole [M, K] activation. Its GEMM's epilogue writes its columns of dst straight into
every rank's dst buffer over NVLink (the buffers are exchanged once, at construction, as CUDA IPC
handles through torch.distributed), then flags every rank; ``finish`` waits for the other ranks'
flags. After a call every rank holds the full [M, N] dst: the all-gather a sharded layer needs,
done by the kernel's own stores, with no collective call and no host synchronisation per op.

The reference runs MUL_MAT (ggml-rocket.cpp:4548-4871) on one device; this is the multi-GPU form
of the same op, bit-for-bit the single-GPU arithmetic per element up to the order of the fp32
K-sums (the stream-K plan of an N/G-row weight can split a tile's K range differently).
"""
import torch
import torch.distributed as dist

import ggml_b200 as g


def shard_rows(N, G, r):
    """Rows [lo, hi) of an N-row weight that rank r of G holds: equal blocks of whole 16-row
    groups (the GEMM's column granularity); the last rank takes the remainder."""
    if N % 16:
        raise ValueError("N must be a multiple of 16")
    groups = N // 16
    per = (groups + G - 1) // G
    lo = min(N, r * per * 16)
    hi = min(N, (r + 1) * per * 16)
    return lo, hi


class PeerShardedMulMat:
    """dst[M, N] = A[M, K] . W[N, K]^T with W's rows split over the ranks of ``group``.

    Sizes are fixed at construction: at most M_max tokens and N_max output columns. __call__
    returns a view of this rank's dst buffer [M, N] (valid until the next call) and copies it into
    ``dst`` when one is given."""

    def __init__(self, M_max, N_max, group=None, device=None):
        self.group = group
        self.G = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.M_max, self.N_max = M_max, N_max
        G, dev = self.G, self.dev
        self.dst = torch.zeros((M_max, N_max), dtype=torch.float32, device=dev)
        self.flags = torch.zeros((G, 4), dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        mine = [self._export(t) for t in (self.dst, self.flags)]
        allh = [None] * G
        dist.all_gather_object(allh, mine, group=group)
        self._opened = []
        ptrs = [[0] * G for _ in range(2)]
        for q in range(G):
            for b, t in enumerate((self.dst, self.flags)):
                if q == self.rank:
                    ptrs[b][q] = t.data_ptr()
                else:
                    handle, off = allh[q][b]
                    base = g._c.c_void_p(0)
                    hb = g._c.create_string_buffer(handle, len(handle))
                    g.check(g.lib().b200_ep_shared_open(hb, g._c.byref(base)), "ep_shared_open")
                    self._opened.append(base.value)
                    ptrs[b][q] = base.value + off
        self.peer_dst = torch.tensor(ptrs[0], dtype=torch.int64, device=dev)
        self.peer_flags = torch.tensor(ptrs[1], dtype=torch.int64, device=dev)
        self.epoch = 0
        self._ws = None
        self._need = {}
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

    def __call__(self, wtype, w_shard, N, K, a, M, dst=None, stream=None, lda=None):
        """w_shard: this rank's packed rows shard_rows(N, G, rank) of the weight; a: [M, K] f32
        on this GPU (row stride lda floats, default K)."""
        if M > self.M_max or N > self.N_max:
            raise ValueError("op outside the sizes this exchange was built for")
        lo, hi = shard_rows(N, self.G, self.rank)
        if hi <= lo:
            raise ValueError("every rank must hold at least one 16-row group of the weight (N >= 16 * G)")
        lib = g.lib()
        self.epoch += 1
        key = (wtype, M, hi - lo, K)
        need = self._need.get(key)
        if need is None:
            need = self._need[key] = lib.b200_mul_mat_tp_workspace_size(wtype, M, hi - lo, K)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.dev)
        g.check(lib.b200_mul_mat_tp(
            wtype, g._ptr(w_shard), hi - lo, lo, K, g._ptr(a), lda if lda else K, M, g._ptr(self.peer_dst),
            self.N_max, self.G, self.rank, g._ptr(self.peer_flags), self.epoch, g._ptr(self._ws), self._ws.numel(),
            g._ptr(self.err), g._stream(stream)), "mul_mat_tp")
        g.check(lib.b200_mul_mat_tp_finish(g._ptr(self.flags), self.G, self.epoch, g._ptr(self.err),
                                           g._stream(stream)), "mul_mat_tp_finish")
        out = self.dst[:M, :N]
        if dst is not None:
            dst.copy_(out)
        return out
