"""The glue ops of a layer (RMS_NORM, ADD, MUL, SILU, SWIGLU, ROPE, GET_ROWS, CPY) on the GPU.

The kernels follow ggml's CPU definitions (restated in the oracle, unpinned since ggml is absent):
ADD, MUL, GET_ROWS and CPY are exact, so they are compared bit for bit; RMS_NORM (tree-ordered
double sum), SILU / SWIGLU (device expf) and ROPE (device cosf / sinf on the same f32 angles)
within GLUE_TOL = 1e-5 max relative error. Then a chain of them runs through graph_compute
(B200_GLUE=1, read once per process, so in a child) on tensors in a device buffer and on host
tensors, including a strided host destination."""
import ctypes

import numpy as np
import pytest

import oracle
from conftest import rel_err

pytestmark = pytest.mark.gpu

GLUE_TOL = 1e-5


def _shape(t):
    """ggml ne / nb (bytes) of a torch tensor whose dims are listed outermost first."""
    ne = list(reversed(t.shape)) + [1] * (4 - t.dim())
    nb = [s * t.element_size() for s in reversed(t.stride())]
    last = nb[-1] * ne[t.dim() - 1] if t.dim() else t.element_size()
    nb = nb + [last] * (4 - t.dim())
    return (ctypes.c_int64 * 4)(*ne), (ctypes.c_size_t * 4)(*nb)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def test_rms_norm_silu_swiglu(cuda):
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(1)
    x = rng.standard_normal((7, 4096)).astype(np.float32) * 3
    xd = torch.from_numpy(x).cuda()
    y = torch.empty_like(xd)
    ne, nb = _shape(xd)
    assert lib.b200_rms_norm(_ptr(xd), ne, nb, 1e-5, _ptr(y), None) == 0
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.rms_norm(x, 1e-5)) <= GLUE_TOL
    # a strided view: every other row
    xs = xd[::2]
    ne, nb = _shape(xs)
    y2 = torch.empty(xs.shape, dtype=torch.float32, device="cuda")
    assert lib.b200_rms_norm(_ptr(xs), ne, nb, 1e-6, _ptr(y2), None) == 0
    torch.cuda.synchronize()
    assert rel_err(y2.cpu().numpy(), oracle.rms_norm(x[::2], 1e-6)) <= GLUE_TOL
    gt = rng.standard_normal(x.shape).astype(np.float32)
    gd = torch.from_numpy(gt).cuda()
    ne, nb = _shape(xd)
    assert lib.b200_silu(_ptr(xd), ne, nb, _ptr(y), None) == 0
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.silu(x)) <= GLUE_TOL
    _, gnb = _shape(gd)
    assert lib.b200_swiglu(_ptr(xd), nb, _ptr(gd), gnb, ne, _ptr(y), None) == 0
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.swiglu(x, gt)) <= GLUE_TOL


def test_add_mul_broadcast_exact(cuda):
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(2)
    a = rng.standard_normal((2, 3, 6, 64)).astype(np.float32)
    b = rng.standard_normal((1, 3, 1, 64)).astype(np.float32)
    ad, bd = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    out = torch.empty_like(ad)
    ane, anb = _shape(ad)
    bne, bnb = _shape(bd)
    for op, want in ((0, a + b), (1, a * b)):   # B200_BIN_ADD, B200_BIN_MUL
        assert lib.b200_binary(op, _ptr(ad), ane, anb, _ptr(bd), bne, bnb, _ptr(out), None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), want)
    # a transposed (strided) first operand
    at = ad.transpose(2, 3)
    ane, anb = _shape(at)
    out2 = torch.empty(at.shape, dtype=torch.float32, device="cuda")
    b1 = torch.from_numpy(rng.standard_normal((1, 1, 64, 1)).astype(np.float32)).cuda()
    bne, bnb = _shape(b1)
    assert lib.b200_binary(0, _ptr(at), ane, anb, _ptr(b1), bne, bnb, _ptr(out2), None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(out2.cpu().numpy(), at.cpu().numpy() + b1.cpu().numpy())
    # b that does not repeat over a is refused
    bad = torch.zeros((1, 1, 1, 5), dtype=torch.float32, device="cuda")
    bne, bnb = _shape(bad)
    assert lib.b200_binary(0, _ptr(at), ane, anb, _ptr(bad), bne, bnb, _ptr(out2), None) == g.B200_E_INVALID


@pytest.mark.parametrize("mode,n_dims,base,fscale", [(0, 128, 10000.0, 1.0), (2, 128, 500000.0, 1.0),
                                                     (2, 64, 10000.0, 0.25), (0, 96, 1000000.0, 0.5)])
def test_rope(cuda, mode, n_dims, base, fscale):
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(n_dims + mode)
    T, H, D = 33, 8, 128
    x = rng.standard_normal((T, H, D)).astype(np.float32)
    pos = rng.integers(0, 8192, T).astype(np.int32)
    xd = torch.from_numpy(x).cuda()
    pd = torch.from_numpy(pos).cuda()
    y = torch.empty_like(xd)
    ne, nb = _shape(xd)
    assert lib.b200_rope(_ptr(xd), ne, nb, _ptr(pd), n_dims, mode, base, fscale, 1.0, _ptr(y), None) == 0
    torch.cuda.synchronize()
    want = oracle.rope(x, pos, n_dims, mode, base, fscale, 1.0)
    assert rel_err(y.cpu().numpy(), want) <= GLUE_TOL
    assert np.array_equal(y.cpu().numpy()[..., n_dims:], x[..., n_dims:])
    assert lib.b200_rope(_ptr(xd), ne, nb, _ptr(pd), n_dims, 8, base, fscale, 1.0, _ptr(y), None) == \
        g.B200_E_UNSUPPORTED   # multi-section / vision modes stay on the host


@pytest.mark.parametrize("T,H,pad,n_dims", [(512, 32, 0, 128), (512, 8, 0, 128), (65, 32, 2, 128), (40, 4, 6, 64)])
def test_rope_normal_mode_rows(cuda, T, H, pad, n_dims):
    """Normal-mode ROPE at Llama-3-8B's query / key shapes (the 8-byte pair kernel), on dense rows and
    on a view whose head rows are wider than D, partial rotation included; against the oracle."""
    import torch
    import ggml_b200 as g
    lib = g.lib()
    D = 128
    rng = np.random.default_rng(T * H + pad)
    full = rng.standard_normal((T, H, D + pad)).astype(np.float32)
    pos = rng.integers(0, 8192, T).astype(np.int32)
    xd = torch.from_numpy(full).cuda()
    view = xd[..., :D]
    pd = torch.from_numpy(pos).cuda()
    y = torch.empty((T, H, D), dtype=torch.float32, device="cuda")
    ne = (ctypes.c_int64 * 4)(D, H, T, 1)
    nb = (ctypes.c_size_t * 4)(4, (D + pad) * 4, H * (D + pad) * 4, T * H * (D + pad) * 4)
    assert lib.b200_rope(_ptr(view), ne, nb, _ptr(pd), n_dims, 0, 500000.0, 1.0, 1.0, _ptr(y), None) == 0
    torch.cuda.synchronize()
    x = np.ascontiguousarray(full[..., :D])
    want = oracle.rope(x, pos, n_dims, 0, 500000.0, 1.0, 1.0)
    assert rel_err(y.cpu().numpy(), want) <= GLUE_TOL
    assert np.array_equal(y.cpu().numpy()[..., n_dims:], x[..., n_dims:])


@pytest.mark.parametrize("T,HK,n_kv,row0", [(512, 8, 1024, 512), (37, 2, 64, 3)])
def test_rope_into_f16_cache_view(cuda, T, HK, n_kv, row0):
    """ROPE of K written as fp16 straight into a KV-cache view (b200_rope_f16): bit-identical to
    b200_rope followed by the f32 -> f16 CPY into the same view, and nothing outside the view
    changes."""
    import torch
    import ggml_b200 as g
    lib = g.lib()
    D = 128
    rng = np.random.default_rng(T + HK)
    x = torch.from_numpy(rng.standard_normal((T, HK, D)).astype(np.float32)).cuda()
    pos = torch.from_numpy(rng.integers(0, 8192, T).astype(np.int32)).cuda()
    ne, nb = _shape(x)
    # the cache: [n_kv rows of HK * D fp16]; the view: rows row0 .. row0 + T as [D, HK, T]
    def cache():
        return torch.from_numpy(rng.standard_normal((n_kv, HK * D)).astype(np.float16)).cuda()
    fused = cache()
    ref = fused.clone()
    vnb = (ctypes.c_size_t * 4)(2, 2 * D, 2 * D * HK, 2 * D * HK * T)
    base = lambda c: ctypes.c_void_p(c.data_ptr() + row0 * HK * D * 2)   # noqa: E731
    assert lib.b200_rope_f16(_ptr(x), ne, nb, _ptr(pos), D, 0, 500000.0, 1.0, 1.0, base(fused), vnb, None) == 0
    y = torch.empty_like(x)
    assert lib.b200_rope(_ptr(x), ne, nb, _ptr(pos), D, 0, 500000.0, 1.0, 1.0, _ptr(y), None) == 0
    vne = (ctypes.c_int64 * 4)(D, HK, T, 1)
    assert lib.b200_cpy(0, _ptr(y), ne, nb, 1, base(ref), vne, vnb, None) == 0
    torch.cuda.synchronize()
    assert torch.equal(fused.view(torch.int16), ref.view(torch.int16))
    # neox mode is not the pair kernel's: refused, nothing written
    assert lib.b200_rope_f16(_ptr(x), ne, nb, _ptr(pos), D, 2, 500000.0, 1.0, 1.0, base(fused), vnb, None) == \
        g.B200_E_UNSUPPORTED


def test_get_rows_and_cpy(cuda):
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(4)
    table = rng.standard_normal((100, 256)).astype(np.float32)
    idx = np.array([[3, 99, 0, 3, 57]], dtype=np.int32)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for ttype, tab in ((0, table), (1, table.astype(np.float16))):
        td = torch.from_numpy(tab).cuda()
        idd = torch.from_numpy(idx).cuda()
        out = torch.empty((1, 5, 256), dtype=torch.float32, device="cuda")
        sne, snb = _shape(td)
        ine, inb = _shape(idd)
        assert lib.b200_get_rows(ttype, _ptr(td), sne, snb, _ptr(idd), ine, inb, _ptr(out), _ptr(err), None) == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert np.array_equal(out.cpu().numpy()[0], tab[idx[0]].astype(np.float32))
    # an index past the table: error word set, zero row, the others intact
    bad = torch.from_numpy(np.array([[1, 100]], dtype=np.int32)).cuda()
    ine, inb = _shape(bad)
    td = torch.from_numpy(table).cuda()
    sne, snb = _shape(td)
    out = torch.full((1, 2, 256), 7.0, dtype=torch.float32, device="cuda")
    assert lib.b200_get_rows(0, _ptr(td), sne, snb, _ptr(bad), ine, inb, _ptr(out), _ptr(err), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) != 0
    o = out.cpu().numpy()[0]
    assert np.array_equal(o[0], table[1]) and np.all(o[1] == 0)
    # CPY: f32 -> f16 (round to nearest even), f16 -> f32, a transposed source into a contiguous
    # destination, and a same-shape strided destination
    x = (rng.standard_normal((64, 48)) * 100).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    h = torch.empty((64, 48), dtype=torch.float16, device="cuda")
    sne, snb = _shape(xd)
    dne, dnb = _shape(h)
    assert lib.b200_cpy(0, _ptr(xd), sne, snb, 1, _ptr(h), dne, dnb, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy(), x.astype(np.float16))
    back = torch.empty((64, 48), dtype=torch.float32, device="cuda")
    sne, snb = _shape(h)
    dne, dnb = _shape(back)
    assert lib.b200_cpy(1, _ptr(h), sne, snb, 0, _ptr(back), dne, dnb, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(back.cpu().numpy(), x.astype(np.float16).astype(np.float32))
    xt = xd.t()                                               # [48, 64] strided
    flat = torch.empty(48 * 64, dtype=torch.float32, device="cuda")
    sne, snb = _shape(xt)
    dne, dnb = _shape(flat)
    assert lib.b200_cpy(0, _ptr(xt), sne, snb, 0, _ptr(flat), dne, dnb, None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(flat.cpu().numpy(), np.ascontiguousarray(x.T).reshape(-1))
    big = torch.zeros((64, 96), dtype=torch.float32, device="cuda")
    view = big[:, ::2]                                        # same shape as x, strided
    sne, snb = _shape(xd)
    dne, dnb = _shape(view)
    assert lib.b200_cpy(0, _ptr(xd), sne, snb, 0, _ptr(view), dne, dnb, None) == 0
    torch.cuda.synchronize()
    bb = big.cpu().numpy()
    assert np.array_equal(bb[:, ::2], x) and np.all(bb[:, 1::2] == 0)


def test_router_ops_soft_max_argsort_sum_rows_div(cuda):
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((37, 128)) * 3).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty_like(xd)
    ne, nb = _shape(xd)
    assert lib.b200_soft_max(_ptr(xd), ne, nb, 0.7, _ptr(y), None) == 0
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), oracle.soft_max(x, 0.7)) <= GLUE_TOL
    s = torch.empty((37, 1), dtype=torch.float32, device="cuda")
    assert lib.b200_sum_rows(_ptr(xd), ne, nb, _ptr(s), None) == 0
    torch.cuda.synchronize()
    assert np.array_equal(s.cpu().numpy()[:, 0], x.astype(np.float64).sum(axis=1).astype(np.float32))
    q = torch.empty_like(xd)
    sne, snb = _shape(s)
    assert lib.b200_binary(2, _ptr(xd), ne, nb, _ptr(s), sne, snb, _ptr(q), None) == 0   # B200_BIN_DIV
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), x / s.cpu().numpy())
    for n in (8, 128, 200, 1000):
        v = rng.standard_normal((5, n)).astype(np.float32)
        v[:, 1] = v[:, 0]                                  # a tie: index order
        v[1, 2], v[1, 3], v[1, 4], v[1, 5] = -0.0, 0.0, np.inf, -np.inf   # -0 ties +0; infinities
        v[2, 3], v[2, 6] = np.nan, np.nan                  # NaNs after every number, either order
        vd = torch.from_numpy(v).cuda()
        ids = torch.empty((5, n), dtype=torch.int32, device="cuda")
        vne, vnb = _shape(vd)
        for desc in (0, 1):
            assert lib.b200_argsort(_ptr(vd), vne, vnb, desc, _ptr(ids), None) == 0
            torch.cuda.synchronize()
            want = np.argsort(-v if desc else v, axis=1, kind="stable")
            assert np.array_equal(ids.cpu().numpy(), want), (n, desc)
    wide = torch.zeros((1, 2048), dtype=torch.float32, device="cuda")
    wne, wnb = _shape(wide)
    assert lib.b200_argsort(_ptr(wide), wne, wnb, 1, _ptr(ids), None) == g.B200_E_UNSUPPORTED


_ROUTER_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
import ggml_b200 as g
import oracle
from conftest import rel_err
be = g.Backend()
rng = np.random.default_rng(12)
E, T, K = 64, 48, 8
logits = (rng.standard_normal((T, E)) * 2).astype(np.float32)
buf = g.DeviceBuffer(be, 1 << 20)
o = [i << 16 for i in range(8)]
assert buf.set(o[0], logits) == 0
tl = buf.tensor(o[0], g.F32, [E, T], name="ffn_moe_logits")
pr = buf.tensor(o[1], g.F32, [E, T], op=g.OP_SOFT_MAX, srcs=[tl], op_params=[1.0, 0.0])
srt = buf.tensor(o[2], g.I32, [E, T], op=g.OP_ARGSORT, srcs=[pr], op_params=[1])
sel = g.make_tensor(g.I32, [K, T], srt.data, op=g.OP_VIEW, srcs=[srt], on_device=True, nb=[4, 4 * E, 4 * E * T, 4 * E * T])
pv = g.make_tensor(g.F32, [1, E, T], pr.data, op=g.OP_VIEW, srcs=[pr], on_device=True)
wts = buf.tensor(o[3], g.F32, [1, K, T], op=g.OP_GET_ROWS, srcs=[pv, sel])
w2 = g.make_tensor(g.F32, [K, T], wts.data, op=g.OP_VIEW, srcs=[wts], on_device=True)
sm = buf.tensor(o[4], g.F32, [1, T], op=g.OP_SUM_ROWS, srcs=[w2])
nw = buf.tensor(o[5], g.F32, [K, T], op=g.OP_DIV, srcs=[w2, sm])
for nd in (pr, srt, wts, sm, nw):
    assert g.supports_op(nd), nd.op
assert be.graph_compute([pr, srt, sel, pv, wts, w2, sm, nw]) == g.STATUS_SUCCESS
ids = np.zeros((T, E), np.int32)
got = np.zeros((T, K), np.float32)
assert buf.get(o[2], ids) == 0 and buf.get(o[5], got) == 0
p = oracle.soft_max(logits, 1.0)
want_ids = np.argsort(-p, axis=1, kind="stable")
print("IDS", int(np.array_equal(ids, want_ids)))
top = np.take_along_axis(p, want_ids[:, :K], axis=1)
want = top / top.astype(np.float64).sum(axis=1, keepdims=True).astype(np.float32)
print("WEIGHTS", rel_err(got, want))
assert be.route_ops("glue") == 5 and be.device_errors() == 0
buf.free()
be.close()
"""


def test_moe_router_through_graph_compute(cuda):
    """The MoE router of a llama.cpp graph (soft_max -> argsort desc -> top-k view -> get_rows ->
    sum_rows -> div) on a device buffer under B200_GLUE=1: the expert ids exactly, the
    normalised weights within GLUE_TOL."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, B200_GLUE="1")
    p = subprocess.run([sys.executable, "-c", _ROUTER_CHILD, ROOT], env=env, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert p.stdout.split("IDS")[1].split()[0] == "1"
    assert float(p.stdout.split("WEIGHTS")[1].split()[0]) <= GLUE_TOL


_CHILD = r"""
import ctypes, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
import ggml_b200 as g
import oracle
from conftest import rel_err
be = g.Backend()
rng = np.random.default_rng(6)
T, H, D, E = 40, 4, 64, 256
x = rng.standard_normal((T, E)).astype(np.float32)
wn = rng.standard_normal(E).astype(np.float32)
pos = np.arange(T, dtype=np.int32) * 3
# in a device buffer: xn = rms_norm(x) * wn; q = rope(xn viewed [D, H, T]); s = swiglu(q, q)
buf = g.DeviceBuffer(be, 1 << 22)
offs = [i << 18 for i in range(8)]
assert buf.set(offs[0], x) == 0 and buf.set(offs[1], wn) == 0 and buf.set(offs[2], pos) == 0
tx = buf.tensor(offs[0], g.F32, [E, T], name="x")
tw = buf.tensor(offs[1], g.F32, [E], name="attn_norm.weight")
tp = buf.tensor(offs[2], g.I32, [T], name="pos")
n1 = buf.tensor(offs[3], g.F32, [E, T], op=g.OP_RMS_NORM, srcs=[tx], op_params=[1e-5])
n2 = buf.tensor(offs[4], g.F32, [E, T], op=g.OP_MUL, srcs=[n1, tw])
v = g.make_tensor(g.F32, [D, H, T], n2.data, op=g.OP_VIEW, srcs=[n2], on_device=True)
r = buf.tensor(offs[5], g.F32, [D, H, T], op=g.OP_ROPE, srcs=[v, tp],
               op_params=[0, D, 2, 0, 4096, 10000.0, 1.0, 0.0, 1.0, 32.0, 1.0])
s = buf.tensor(offs[6], g.F32, [D, H, T], op=g.OP_GLU, srcs=[r, r], op_params=[g.GLU_SWIGLU, 0])
nodes = [n1, n2, v, r, s]
for nd in (n1, n2, r, s):
    assert g.supports_op(nd), nd.op
assert be.graph_compute(nodes) == g.STATUS_SUCCESS
got = np.zeros((T, H, D), np.float32)
assert buf.get(offs[6], got) == 0
xn = oracle.rms_norm(x, 1e-5) * wn
q = oracle.rope(xn.reshape(T, H, D), pos, D, 2, 10000.0, 1.0, 1.0)
want = oracle.swiglu(q, q)
print("CHAIN", rel_err(got, want))
assert be.route_ops("glue") == 4 and be.route_ops("norm_mul") == 1   # RMS_NORM * weight fused
# the norm's own output read again later: the fused launch writes it too
m2 = buf.tensor(offs[7], g.F32, [E, T], op=g.OP_ADD, srcs=[n1, n2])
assert be.graph_compute([n1, n2, m2]) == g.STATUS_SUCCESS
got2 = np.zeros((T, E), np.float32)
assert buf.get(offs[7], got2) == 0
nrm = oracle.rms_norm(x, 1e-5)
print("NORMREUSE", rel_err(got2, nrm + nrm * wn))
assert be.route_ops("norm_mul") == 2
# residual ADD -> RMS_NORM -> MUL: one launch; the sum (the next residual) is written
ra = buf.tensor(offs[3], g.F32, [E, T], op=g.OP_ADD, srcs=[tx, n2])
rn = buf.tensor(offs[5], g.F32, [E, T], op=g.OP_RMS_NORM, srcs=[ra], op_params=[1e-5])
rm = buf.tensor(offs[6], g.F32, [E, T], op=g.OP_MUL, srcs=[rn, tw])
assert be.graph_compute([n1, n2, ra, rn, rm]) == g.STATUS_SUCCESS
got_s, got_m = np.zeros((T, E), np.float32), np.zeros((T, E), np.float32)
assert buf.get(offs[3], got_s) == 0 and buf.get(offs[6], got_m) == 0
hsum = x + nrm * wn
print("ADDNORM", max(rel_err(got_s, hsum), rel_err(got_m, oracle.rms_norm(hsum, 1e-5) * wn)))
assert be.route_ops("add_norm_mul") == 1
# host tensors: CPY into a strided host destination (the bytes between its elements survive)
a = rng.standard_normal((8, 32)).astype(np.float32)
dst = np.full((8, 64), 5.0, np.float32)
ta = g.make_tensor(g.F32, [32, 8], a)
td = g.make_tensor(g.F32, [32, 8], dst, op=g.OP_CPY, srcs=[ta], nb=[4, 256, 2048, 2048])
assert g.supports_op(td)
assert be.graph_compute([td]) == g.STATUS_SUCCESS
assert np.array_equal(dst[:, :32], a) and np.all(dst[:, 32:] == 5.0)
print("HOSTCPY ok")
assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
buf.free()
be.close()
"""


def test_glue_chain_through_graph_compute(cuda):
    import os
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, B200_GLUE="1")
    p = subprocess.run([sys.executable, "-c", _CHILD, ROOT], env=env, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert float(p.stdout.split("CHAIN")[1].split()[0]) <= GLUE_TOL
    assert float(p.stdout.split("NORMREUSE")[1].split()[0]) <= GLUE_TOL
    assert float(p.stdout.split("ADDNORM")[1].split()[0]) <= GLUE_TOL
    assert "HOSTCPY ok" in p.stdout


def test_dense_fast_paths_match_the_general_kernels(cuda):
    """Dense f32 operands take 16-byte-access kernels without per-element index arithmetic; the same
    values laid out with a row pitch wider than the row take the general strided kernels. Both
    must give the same bits (the same f32 operation per element), and match ggml's definitions."""
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(21)
    R, C = 96, 1024
    x = rng.standard_normal((R, C)).astype(np.float32)
    y = rng.standard_normal((R, C)).astype(np.float32)
    w = rng.standard_normal(C).astype(np.float32)
    xd, yd, wd = (torch.from_numpy(v).cuda() for v in (x, y, w))
    wide = torch.zeros((R, 2 * C), dtype=torch.float32, device="cuda")
    wide[:, :C] = xd
    xs = wide[:, :C]                                   # the same values, row pitch 2C: strided
    wide2 = torch.zeros((R, 2 * C), dtype=torch.float32, device="cuda")
    wide2[:, :C] = yd
    ys = wide2[:, :C]

    def run(fn, *args):
        out = torch.empty((R, C), dtype=torch.float32, device="cuda")
        assert fn(*args, _ptr(out), None) == 0
        torch.cuda.synchronize()
        return out.cpu().numpy()

    for op, want in ((0, x + y), (1, x * y), (2, x / y)):
        d = run(lib.b200_binary, op, _ptr(xd), *_shape(xd), _ptr(yd), *_shape(yd))
        st = run(lib.b200_binary, op, _ptr(xs), *_shape(xs), _ptr(ys), *_shape(ys))
        assert np.array_equal(d.view(np.uint32), st.view(np.uint32)) and np.array_equal(d, want)
    wne, wnb = _shape(wd)
    for op, want in ((0, x + w), (1, x * w)):      # the norm weight: one row repeated
        d = run(lib.b200_binary, op, _ptr(xd), *_shape(xd), _ptr(wd), wne, wnb)
        st = run(lib.b200_binary, op, _ptr(xs), *_shape(xs), _ptr(wd), wne, wnb)
        assert np.array_equal(d.view(np.uint32), st.view(np.uint32)) and np.array_equal(d, want)
    d = run(lib.b200_silu, _ptr(xd), *_shape(xd))
    st = run(lib.b200_silu, _ptr(xs), *_shape(xs))
    assert np.array_equal(d.view(np.uint32), st.view(np.uint32)) and rel_err(d, oracle.silu(x)) <= GLUE_TOL
    ne, nb = _shape(xd)
    d = run(lib.b200_swiglu, _ptr(xd), nb, _ptr(yd), _shape(yd)[1], ne)
    st = run(lib.b200_swiglu, _ptr(xs), _shape(xs)[1], _ptr(ys), _shape(ys)[1], _shape(xs)[0])
    assert np.array_equal(d.view(np.uint32), st.view(np.uint32)) and rel_err(d, oracle.swiglu(x, y)) <= GLUE_TOL
    d = run(lib.b200_rms_norm, _ptr(xd), *_shape(xd), ctypes.c_float(1e-5))
    st = run(lib.b200_rms_norm, _ptr(xs), *_shape(xs), ctypes.c_float(1e-5))
    assert rel_err(d, st) <= 1e-6 and rel_err(d, oracle.rms_norm(x, 1e-5)) <= GLUE_TOL
    # f32 -> f16, dense and strided sources
    for src in (xd, xs):
        h = torch.empty((R, C), dtype=torch.float16, device="cuda")
        assert lib.b200_cpy(0, _ptr(src), *_shape(src), 1, _ptr(h), *_shape(h), None) == 0
        torch.cuda.synchronize()
        assert np.array_equal(h.cpu().numpy().view(np.uint16), x.astype(np.float16).view(np.uint16))


def test_rms_norm_mul_matches_the_two_ops(cuda):
    """b200_rms_norm_mul (RMS_NORM and the MUL by one weight row as one launch) gives the same bits
    as b200_rms_norm then b200_binary(MUL), with and without the normalised rows written, for dense
    and row-padded inputs."""
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(31)
    E, T = 4096, 37
    w = torch.from_numpy(rng.standard_normal(E).astype(np.float32)).cuda()
    wne, wnb = _shape(w.view(1, E))
    for pad in (0, 4, 3):
        xb = torch.from_numpy(rng.standard_normal((T, E + pad)).astype(np.float32)).cuda()
        x = xb[:, :E]
        ne, nb = _shape(x)
        ref_n = torch.empty((T, E), device="cuda")
        ref = torch.empty((T, E), device="cuda")
        cne, cnb = _shape(ref_n)
        assert lib.b200_rms_norm(_ptr(x), ne, nb, 1e-6, _ptr(ref_n), None) == 0
        assert lib.b200_binary(1, _ptr(ref_n), cne, cnb, _ptr(w), wne, wnb, _ptr(ref), None) == 0
        got_n = torch.full((T, E), float("nan"), device="cuda")
        got = torch.full((T, E), float("nan"), device="cuda")
        assert lib.b200_rms_norm_mul(_ptr(x), ne, nb, 1e-6, _ptr(w), _ptr(got_n), _ptr(got), None) == 0
        got2 = torch.full((T, E), float("nan"), device="cuda")
        assert lib.b200_rms_norm_mul(_ptr(x), ne, nb, 1e-6, _ptr(w), None, _ptr(got2), None) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref) and torch.equal(got_n, ref_n) and torch.equal(got2, ref), pad
    assert lib.b200_rms_norm_mul(_ptr(x), ne, nb, 1e-6, None, None, _ptr(got), None) == g.B200_E_INVALID


def _sylvester(n):
    i = np.arange(n)
    return np.where(np.bitwise_count(i[:, None] & i[None, :]) % 2 == 1, -1.0, 1.0)


@pytest.mark.parametrize("n", [32, 64, 128, 256, 512, 1024])
def test_hadamard_transform_matches_the_dense_product(cuda, n):
    """b200_hadamard (the fast transform of a Hadamard-tagged MUL_MAT) against the dense product
    with the Sylvester-ordered matrix in fp64, within GLUE_TOL; row-padded input too."""
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(n)
    T = 37
    scale = np.float32(1.0 / np.sqrt(n))
    for pad in (0, 8):
        xb = torch.from_numpy(rng.standard_normal((T, n + pad)).astype(np.float32)).cuda()
        x = xb[:, :n]
        ne, nb = _shape(x)
        y = torch.full((T, n), float("nan"), device="cuda")
        assert lib.b200_hadamard(_ptr(x), ne, nb, float(scale), _ptr(y), None) == 0
        torch.cuda.synchronize()
        want = x.cpu().numpy().astype(np.float64) @ (_sylvester(n) * np.float64(scale)).T
        assert rel_err(y.cpu().numpy(), want) <= GLUE_TOL, (n, pad)
    bad = torch.zeros((2, 48), device="cuda")
    bne, bnb = _shape(bad)
    assert lib.b200_hadamard(_ptr(bad), bne, bnb, 1.0, _ptr(bad), None) == g.B200_E_UNSUPPORTED   # not 2^k


_HADAMARD_CHILD = r"""
import sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
import ggml_b200 as g
from conftest import rel_err
be = g.Backend()
rng = np.random.default_rng(9)
n, T = 128, 40
i = np.arange(n)
h = np.where(np.bitwise_count(i[:, None] & i[None, :]) % 2 == 1, -1.0, 1.0) / np.sqrt(n)
worst = 0.0
for wt, arr in ((g.F32, h.astype(np.float32)), (g.F16, h.astype(np.float16))):
    x = rng.standard_normal((T, n)).astype(np.float32)
    out = np.full((T, n), np.nan, np.float32)
    w = g.make_tensor(wt, [n, n], arr, name="hadamard_%d" % wt)
    tx = g.make_tensor(g.F32, [n, T], x)
    d = g.make_tensor(g.F32, [n, T], out, op=g.OP_MUL_MAT, srcs=[w, tx], op_params=[0, g.HINT_SRC0_IS_HADAMARD])
    assert g.supports_op(d)
    assert be.graph_compute([d]) == g.STATUS_SUCCESS
    want = x.astype(np.float64) @ arr.astype(np.float64).T
    worst = max(worst, rel_err(out, want))
assert be.route_ops("hadamard") == 2 and be.cpu_fallbacks() == 0 and be.device_errors() == 0
be.close()
print("HADAMARD", worst)
"""


def test_hadamard_mul_mat_through_graph_compute(cuda):
    """With B200_GLUE=1 a Hadamard-tagged MUL_MAT (src0 the scaled Sylvester matrix, F32 and F16)
    runs through graph_compute on the transform kernel and matches the dense product."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, B200_GLUE="1")
    p = subprocess.run([sys.executable, "-c", _HADAMARD_CHILD, ROOT], env=env, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert float(p.stdout.split("HADAMARD")[1].split()[0]) <= GLUE_TOL


def test_add_rms_norm_mul_matches_the_three_ops(cuda):
    """b200_add_rms_norm_mul (residual ADD, RMS_NORM and the MUL by the norm weight as one launch)
    gives the same bits as b200_binary(ADD), b200_rms_norm and b200_binary(MUL), the sum included,
    with and without the normalised rows written; and refuses an unaligned operand."""
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(41)
    E, T = 4096, 29
    a = torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).cuda()
    r = torch.from_numpy(rng.standard_normal((T, E)).astype(np.float32)).cuda()
    w = torch.from_numpy(rng.standard_normal(E).astype(np.float32)).cuda()
    ne, nb = _shape(a)
    wne, wnb = _shape(w.view(1, E))
    s_ref, n_ref, o_ref = (torch.empty((T, E), device="cuda") for _ in range(3))
    assert lib.b200_binary(0, _ptr(a), ne, nb, _ptr(r), ne, nb, _ptr(s_ref), None) == 0
    assert lib.b200_rms_norm(_ptr(s_ref), ne, nb, 1e-5, _ptr(n_ref), None) == 0
    assert lib.b200_binary(1, _ptr(n_ref), ne, nb, _ptr(w), wne, wnb, _ptr(o_ref), None) == 0
    for with_norm in (True, False):
        s, n, o = (torch.full((T, E), float("nan"), device="cuda") for _ in range(3))
        assert lib.b200_add_rms_norm_mul(_ptr(a), _ptr(r), ne, 1e-5, _ptr(w), _ptr(s), _ptr(n) if with_norm else None,
                                         _ptr(o), None) == 0
        torch.cuda.synchronize()
        assert torch.equal(s, s_ref) and torch.equal(o, o_ref)
        assert torch.equal(n, n_ref) if with_norm else bool(torch.isnan(n).all())
    odd = torch.empty(T * E + 1, device="cuda")[1:].view(T, E)
    assert lib.b200_add_rms_norm_mul(_ptr(odd), _ptr(r), ne, 1e-5, _ptr(w), _ptr(s), None, _ptr(o), None) == \
        g.B200_E_UNSUPPORTED
