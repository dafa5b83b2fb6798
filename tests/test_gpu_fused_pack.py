"""Glue ops fused with the activation pack of the MUL_MAT that reads them, through the C ABI: the
dense FFN's SWIGLU (b200_swiglu_act_pack) and the [ADD ->] RMS_NORM * weight row in front of a
Q/K/V or gate/up group (b200_rms_norm_mul_act_pack). Their fp16 rows and row scales must equal the
unfused ops followed by b200_act_pack bit for bit (the same per-element arithmetic, and the
reference's activation sandwich, rk_pack_act_row in ggml-rocket.cpp:1451-1475), for the Llama-3-8B
widths and ragged shapes, with a zero row and large-magnitude rows."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,F,pad", [(512, 14336, 0), (77, 2816, 8), (33, 768, 4), (5, 1024, 0), (300, 16384, 0)])
def test_swiglu_act_pack_equals_chain(cuda, M, F, pad):
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(M * 7 + F)
    gate = torch.from_numpy(rng.standard_normal((M, F + pad), dtype=np.float32) * 3).cuda()
    up = torch.from_numpy(rng.standard_normal((M, F + pad), dtype=np.float32)).cuda()
    gate[0] = 0.0                                   # a row whose SWIGLU is all zero (scale 1)
    up[M - 1] *= 1e4                                # a row far outside fp16 range before the scale
    a16 = torch.empty((M, F), dtype=torch.float16, device="cuda")
    sc = torch.empty(M, dtype=torch.float32, device="cuda")
    g.swiglu_act_pack(gate, up, M, F, a16, sc, ldg=F + pad, ldu=F + pad)
    h = torch.empty((M, F), dtype=torch.float32, device="cuda")
    g.swiglu(gate[:, :F].contiguous(), up[:, :F].contiguous(), h)
    a16_ref = torch.empty_like(a16)
    sc_ref = torch.empty_like(sc)
    g.act_pack(h, M, F, a16_ref, sc_ref)
    torch.cuda.synchronize()
    assert torch.equal(a16.view(torch.int16), a16_ref.view(torch.int16))
    assert torch.equal(sc.view(torch.int32), sc_ref.view(torch.int32))
    assert float(sc[0]) == 1.0


def test_swiglu_act_pack_rejects_unsupported(cuda):
    import torch
    import ggml_b200 as g
    x = torch.zeros((4, 16392), dtype=torch.float32, device="cuda")
    a16 = torch.empty((4, 16392), dtype=torch.float16, device="cuda")
    sc = torch.empty(4, dtype=torch.float32, device="cuda")
    with pytest.raises(g.B200Error):                # wider than the register rows hold
        g.swiglu_act_pack(x, x, 4, 16392, a16, sc)
    with pytest.raises(g.B200Error):                # F not a multiple of 4
        g.swiglu_act_pack(x, x, 4, 1022, a16, sc)


@pytest.mark.parametrize("M,E,with_res,outs", [(512, 4096, True, False), (512, 4096, False, False),
                                               (77, 2048, True, True), (3, 16384, False, True), (33, 1028, True, True)])
def test_norm_mul_act_pack_equals_chain(cuda, M, E, with_res, outs):
    import ctypes
    import torch
    import ggml_b200 as g
    lib = g.lib()
    rng = np.random.default_rng(M + E + with_res)
    x = torch.from_numpy(rng.standard_normal((M, E), dtype=np.float32) * 2).cuda()
    res = torch.from_numpy(rng.standard_normal((M, E), dtype=np.float32)).cuda()
    w = torch.from_numpy((1.0 + 0.1 * rng.standard_normal(E)).astype(np.float32)).cuda()
    x[M // 2] *= 1e5                                 # a row far outside fp16 range before the scale
    ne = (ctypes.c_int64 * 4)(E, M, 1, 1)
    nb = (ctypes.c_size_t * 4)(4, E * 4, M * E * 4, M * E * 4)
    eps = 1e-5
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None   # noqa: E731
    a16 = torch.empty((M, E), dtype=torch.float16, device="cuda")
    sc = torch.empty(M, dtype=torch.float32, device="cuda")
    s_out = torch.full((M, E), float("nan"), device="cuda") if with_res else None
    n_out = torch.full((M, E), float("nan"), device="cuda") if outs else None
    d_out = torch.full((M, E), float("nan"), device="cuda") if outs else None
    rc = lib.b200_rms_norm_mul_act_pack(P(x), P(res) if with_res else None, ne, eps, P(w), P(s_out), P(n_out),
                                        P(d_out), P(a16), P(sc), None)
    assert rc == 0
    # the unfused chain: [ADD ->] RMS_NORM * w, then the activation pack of the product
    s_ref = torch.empty((M, E), device="cuda")
    n_ref = torch.empty((M, E), device="cuda")
    d_ref = torch.empty((M, E), device="cuda")
    if with_res:
        assert lib.b200_add_rms_norm_mul(P(x), P(res), ne, ctypes.c_float(eps), P(w), P(s_ref), P(n_ref), P(d_ref),
                                         None) == 0
    else:
        assert lib.b200_rms_norm_mul(P(x), ne, nb, ctypes.c_float(eps), P(w), P(n_ref), P(d_ref), None) == 0
    a16_ref = torch.empty_like(a16)
    sc_ref = torch.empty_like(sc)
    g.act_pack(d_ref, M, E, a16_ref, sc_ref)
    torch.cuda.synchronize()
    assert torch.equal(a16.view(torch.int16), a16_ref.view(torch.int16))
    assert torch.equal(sc.view(torch.int32), sc_ref.view(torch.int32))
    if with_res:
        assert torch.equal(s_out.view(torch.int32), s_ref.view(torch.int32))
    if outs:
        assert torch.equal(n_out.view(torch.int32), n_ref.view(torch.int32))
        assert torch.equal(d_out.view(torch.int32), d_ref.view(torch.int32))
