"""Descriptor graphs of whole model layers, built the way llama.cpp builds them, for placement
checks and end-to-end runs of graph_compute.

`llama_layer` returns the nodes of one dense Llama-family prefill layer -- attention norm, Q/K/V
projections, RoPE, the K/V cache writes (CPY into f16 cache views), FLASH_ATTN_EXT, the output
projection and residual, FFN norm, gate/up, SWIGLU, down and residual -- as b200_tensor
descriptors with ggml's shapes, strides and views (llama.cpp's llm_build_llama /
build_attn / build_ffn). With no `alloc`, tensors carry no data (enough for supports_op); with an
`alloc(nbytes) -> (data, on_device)` callback every tensor gets storage, e.g. in a DeviceBuffer.
"""
import ggml_b200 as g


class Layer:
    """The descriptors of one layer: `nodes` in execution order, `inputs` / `weights` /
    `caches` by name, `out` the layer output."""

    def __init__(self):
        self.nodes = []
        self.inputs = {}
        self.weights = {}
        self.caches = {}
        self.out = None
        self._keep = []          # every descriptor, so that the ctypes objects stay alive

    def t(self, *a, **k):
        x = g.make_tensor(*a, **k)
        self._keep.append(x)
        return x


def _contig_nb(ttype, ne):
    be, bb = g.BLOCK.get(ttype, (1, 4))
    nb0 = bb
    nb1 = (ne[0] // be) * bb
    return [nb0, nb1, nb1 * ne[1], nb1 * ne[1] * ne[2]]


def llama_layer(T, E=4096, F=14336, H=32, HK=8, D=128, n_kv=None, wtype=g.Q4_K, eps=1e-5, rope_base=500000.0,
                alloc=None, il=0, rope_mode=0):
    """One prefill layer of T tokens. n_kv: the KV cache length the attention reads (at least T,
    rounded up to 256 like llama.cpp's padded cache views); the new K/V rows are written at its
    start. rope_mode: 0 (normal, what llama.cpp uses for the Llama architecture) or 2 (neox).
    alloc: see the module docstring."""
    n_kv = n_kv or max(256, (T + 255) // 256 * 256)
    L = Layer()

    def new(ttype, ne, op=g.OP_NONE, srcs=(), name="", op_params=None, nb=None, view_of=None, offset=0):
        ne = list(ne) + [1] * (4 - len(ne))
        if view_of is not None:
            data, dev = view_of.data, bool(view_of.on_device)
            if data is not None:
                data += offset
        elif alloc is not None:
            size = _contig_nb(ttype, ne)[3] * ne[3] if nb is None else nb[3] * ne[3]
            data, dev = alloc(size)
        else:
            data, dev = None, False
        return L.t(ttype, ne, data, op=op, srcs=srcs, name=name, on_device=dev, nb=nb, op_params=op_params)

    def weight(name, ne, ttype=wtype):
        w = new(ttype, ne, name=f"blk.{il}.{name}.weight")
        L.weights[name] = w
        return w

    def node(x):
        L.nodes.append(x)
        return x

    x = new(g.F32, [E, T], name="inp")
    pos = new(g.I32, [T], name="inp_pos")
    mask = new(g.F16, [n_kv, (T + 63) // 64 * 64], name="kq_mask")
    L.inputs.update(x=x, pos=pos, mask=mask)
    k_cache = new(g.F16, [D * HK, n_kv], name=f"cache_k_l{il}")
    v_cache = new(g.F16, [D * HK, n_kv], name=f"cache_v_l{il}")
    L.caches.update(k=k_cache, v=v_cache)

    # attention
    an = node(new(g.F32, [E, T], g.OP_RMS_NORM, [x], "attn_norm", op_params=[eps]))
    an = node(new(g.F32, [E, T], g.OP_MUL, [an, weight("attn_norm", [E], g.F32)], "attn_norm_w"))
    q = node(new(g.F32, [E, T], g.OP_MUL_MAT, [weight("attn_q", [E, E]), an], "Qcur"))
    k = node(new(g.F32, [D * HK, T], g.OP_MUL_MAT, [weight("attn_k", [E, D * HK]), an], "Kcur"))
    v = node(new(g.F32, [D * HK, T], g.OP_MUL_MAT, [weight("attn_v", [E, D * HK]), an], "Vcur"))
    rope_params = [0, D, rope_mode, 0, 8192, rope_base, 1.0, 0.0, 1.0, 32.0, 1.0]
    q3 = node(new(g.F32, [D, H, T], g.OP_RESHAPE, [q], "Qcur_3d", view_of=q))
    k3 = node(new(g.F32, [D, HK, T], g.OP_RESHAPE, [k], "Kcur_3d", view_of=k))
    qr = node(new(g.F32, [D, H, T], g.OP_ROPE, [q3, pos], "Qcur_rope", op_params=rope_params))
    kr = node(new(g.F32, [D, HK, T], g.OP_ROPE, [k3, pos], "Kcur_rope", op_params=rope_params))
    # the new rows of the caches: views of their first T rows, written by CPY (f32 -> f16)
    kv_nb = [2, 2 * D, 2 * D * HK, 2 * D * HK * T]
    kc_view = node(new(g.F16, [D, HK, T], g.OP_VIEW, [k_cache], "k_cache_view", nb=kv_nb, view_of=k_cache))
    vc_view = node(new(g.F16, [D, HK, T], g.OP_VIEW, [v_cache], "v_cache_view", nb=kv_nb, view_of=v_cache))
    v3 = node(new(g.F32, [D, HK, T], g.OP_RESHAPE, [v], "Vcur_3d", view_of=v))
    node(new(g.F16, [D, HK, T], g.OP_CPY, [kr, kc_view], "k_cache_cpy", nb=kv_nb, view_of=k_cache))
    node(new(g.F16, [D, HK, T], g.OP_CPY, [v3, vc_view], "v_cache_cpy", nb=kv_nb, view_of=v_cache))
    # attention reads: q permuted to [D, T, H]; k / v the cache as [D, n_kv, HK]
    qp = node(new(g.F32, [D, T, H], g.OP_PERMUTE, [qr], "q", nb=[4, 4 * D * H, 4 * D, 4 * D * H * T],
                  view_of=qr))
    kvv_nb = [2, 2 * D * HK, 2 * D, 2 * D * HK * n_kv]
    kk = node(new(g.F16, [D, n_kv, HK], g.OP_VIEW, [k_cache], "k", nb=kvv_nb, view_of=k_cache))
    vv = node(new(g.F16, [D, n_kv, HK], g.OP_VIEW, [v_cache], "v", nb=kvv_nb, view_of=v_cache))
    scale = 1.0 / D ** 0.5
    fa = node(new(g.F32, [D, H, T], g.OP_FLASH_ATTN_EXT, [qp, kk, vv, mask], "kqv_out",
                  op_params=[scale, 0.0, 0.0, 10]))
    fa2 = node(new(g.F32, [E, T], g.OP_RESHAPE, [fa], "kqv_out_2d", view_of=fa))
    o = node(new(g.F32, [E, T], g.OP_MUL_MAT, [weight("attn_output", [E, E]), fa2], "attn_out"))
    h = node(new(g.F32, [E, T], g.OP_ADD, [o, x], "ffn_inp"))
    # feed-forward
    fn = node(new(g.F32, [E, T], g.OP_RMS_NORM, [h], "ffn_norm", op_params=[eps]))
    fn = node(new(g.F32, [E, T], g.OP_MUL, [fn, weight("ffn_norm", [E], g.F32)], "ffn_norm_w"))
    gt = node(new(g.F32, [F, T], g.OP_MUL_MAT, [weight("ffn_gate", [E, F]), fn], "ffn_gate"))
    up = node(new(g.F32, [F, T], g.OP_MUL_MAT, [weight("ffn_up", [E, F]), fn], "ffn_up"))
    act = node(new(g.F32, [F, T], g.OP_GLU, [gt, up], "ffn_swiglu", op_params=[g.GLU_SWIGLU, 0]))
    dn = node(new(g.F32, [E, T], g.OP_MUL_MAT, [weight("ffn_down", [F, E]), act], "ffn_out"))
    L.out = node(new(g.F32, [E, T], g.OP_ADD, [dn, h], "l_out"))
    return L
