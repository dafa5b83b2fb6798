"""The dense FFN's SWIGLU fused into the down projection's activation pack (b200_swiglu_act_pack),
through the C ABI: its fp16 rows and row scales must equal b200_swiglu followed by b200_act_pack
bit for bit (the same per-element SWIGLU, ggml_swiglu_split, and the reference's activation
sandwich, rk_pack_act_row in ggml-rocket.cpp:1451-1475), for the Llama-3-8B FFN width and ragged
shapes, with row strides wider than the rows, a zero row and large-magnitude rows."""
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
