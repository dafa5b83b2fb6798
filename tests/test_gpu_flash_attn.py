"""FLASH_ATTN_EXT parity on the GPU through b200_flash_attn_ext, against the fp64 oracle.

Mirrors test-rocket-fa.cpp: its cases (:174-182) -- analytic one-hot "overflow" logits (raw q.k
60000-135000), typical causal attention, the scaled-logit overflow and the Q-range cases (which
the reference must send to its host reference and which run on the GPU here) -- with their
tolerances, plus the BASELINE FA shape (32/8 heads, D 128, causal), KV-cache views with
interleaved heads, ragged KV / T, soft-capping, no mask, and fully masked rows.
"""
import math

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

OVERFLOW, TYPICAL, SCALED, QRANGE = range(4)


def fill_case(D, T, H, KV, HK, kind, seed):
    """The constructions of test-rocket-fa.cpp:137-170 (own generator)."""
    rng = np.random.default_rng(seed)
    Q = np.zeros((H, T, D), np.float32)
    K = np.zeros((HK, KV, D), np.float32)
    V = rng.uniform(-1, 1, (HK, KV, D)).astype(np.float32)
    M = np.zeros((T, KV), np.float32)
    if kind != TYPICAL:
        qa = 500.0 * math.sqrt(D) if kind == SCALED else (1.0e6 if kind == QRANGE else 1000.0)
        k0 = 140.0 if kind == SCALED else 60.0
        kd = 1000.0 if kind == QRANGE else 1.0
        for h in range(H):
            for t in range(T):
                Q[h, t, (t + h) % D] = qa
        for hk in range(HK):
            for j in range(KV):
                K[hk, j, j % D] = (k0 + 5.0 * (j // D)) / kd
    else:
        Q[:] = rng.uniform(-1, 1, Q.shape)
        K[:] = rng.uniform(-1, 1, K.shape)
        for t in range(T):
            M[t, KV - T + t + 1:] = -np.inf
    return Q, K, V, M


def run_fa(torch, Q, K16, V16, M16, scale, softcap=0.0, k_layout="dense", D=None):
    """Q f32 [H,T,D]; K16/V16 fp16 bits [HK,KV,D]; M16 fp16 bits [T,KV] or None. Returns [T,H,DV]."""
    import ggml_b200 as g
    H, T, Dq = Q.shape
    HK, KV, DV = V16.shape
    q = torch.from_numpy(np.ascontiguousarray(Q)).cuda()
    if k_layout == "dense":
        k = torch.from_numpy(np.ascontiguousarray(K16)).cuda()
        v = torch.from_numpy(np.ascontiguousarray(V16)).cuda()
        k_nb1, k_nb2 = Dq * 2, KV * Dq * 2
        v_nb1, v_nb2 = DV * 2, KV * DV * 2
    else:
        # llama.cpp KV-cache view: rows are [HK * D] per position, heads interleaved, room for more
        # positions than KV
        cap = KV + 64
        kc = np.zeros((cap, HK, Dq), np.uint16)
        vc = np.zeros((cap, HK, DV), np.uint16)
        kc[:KV] = np.transpose(K16, (1, 0, 2))
        vc[:KV] = np.transpose(V16, (1, 0, 2))
        k = torch.from_numpy(kc).cuda()
        v = torch.from_numpy(vc).cuda()
        k_nb1, k_nb2 = HK * Dq * 2, Dq * 2
        v_nb1, v_nb2 = HK * DV * 2, DV * 2
    m = None
    m_nb1 = 0
    if M16 is not None:
        # ggml pads the mask's token dim; give it 3 extra rows of garbage
        Tp = T + 3
        mp = np.full((Tp, M16.shape[1]), 0x3C00, np.uint16)
        mp[:T] = M16
        m = torch.from_numpy(mp).cuda()
        m_nb1 = M16.shape[1] * 2
    dst = torch.full((T, H, DV), float("nan"), dtype=torch.float32, device="cuda")
    ws = torch.empty(g.flash_attn_workspace_size(Dq, DV, T, H, KV, HK), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    g.flash_attn_ext(q, Dq * 4, T * Dq * 4, k, k_nb1, k_nb2, v, v_nb1, v_nb2, m, m_nb1, dst, Dq, DV, T, H, KV, HK,
                     scale, softcap, ws, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"device error {int(err.item())}"
    return dst.cpu().numpy()


def f16(x):
    with np.errstate(over="ignore"):
        return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


# (name, D, T, H, KV, HK, kind, tol) from test-rocket-fa.cpp:174-182
REF_CASES = [
    ("overflow d64", 64, 32, 4, 1024, 2, OVERFLOW, 1e-3),
    ("overflow d128", 128, 32, 4, 1024, 2, OVERFLOW, 1e-3),
    ("typical d64", 64, 64, 8, 1024, 2, TYPICAL, 2e-2),
    ("typical d128", 128, 64, 4, 1536, 4, TYPICAL, 2e-2),
    ("scaled d64", 64, 32, 4, 1024, 2, SCALED, 1e-3),
    ("scaled d128", 128, 32, 4, 1024, 2, SCALED, 1e-3),
    ("q range d64", 64, 32, 4, 1024, 2, QRANGE, 1e-3),
]


@pytest.mark.parametrize("case", REF_CASES, ids=[c[0] for c in REF_CASES])
def test_fa_reference_cases(cuda, case):
    import torch
    name, D, T, H, KV, HK, kind, tol = case
    Q, K, V, M = fill_case(D, T, H, KV, HK, kind, seed=D * 131 + KV)
    K16, V16, M16 = f16(K), f16(V), f16(M)
    scale = 1.0 / math.sqrt(D)
    got = run_fa(torch, Q, K16, V16, M16, scale)
    # ref_fa reads Q as fp16 except for the two range cases, which read it as F32
    q_mode = 0 if kind in (SCALED, QRANGE) else 1
    want = oracle.flash_attn(Q, K16, V16, M16, scale, q_mode=q_mode)
    assert np.all(np.isfinite(got))
    assert float(np.max(np.abs(got - want))) <= tol


@pytest.mark.parametrize("KV", [1024, 4096])
def test_fa_baseline_shape_causal(cuda, KV):
    """32 query heads, 8 KV heads, D 128, n_q 512 at the end of the context."""
    import torch
    rng = np.random.default_rng(KV)
    H, HK, D, T = 32, 8, 128, 512
    Q = rng.standard_normal((H, T, D)).astype(np.float32)
    K16 = f16(rng.standard_normal((HK, KV, D)))
    V16 = f16(rng.standard_normal((HK, KV, D)))
    M = np.zeros((T, KV), np.float32)
    for t in range(T):
        M[t, KV - T + t + 1:] = -np.inf
    M16 = f16(M)
    scale = 1.0 / math.sqrt(D)
    got = run_fa(torch, Q, K16, V16, M16, scale, k_layout="cache")
    want = oracle.flash_attn(Q, K16, V16, M16, scale, q_mode=2)
    den = np.max(np.abs(want))
    assert float(np.max(np.abs(got - want))) / den <= 1e-2


@pytest.mark.parametrize("D,DV,H,HK,T,KV", [(128, 128, 8, 2, 50, 1100), (64, 64, 6, 3, 37, 1500),
                                            (128, 64, 4, 4, 20, 700), (64, 128, 16, 1, 33, 1030)])
def test_fa_ragged_shapes(cuda, D, DV, H, HK, T, KV):
    import torch
    rng = np.random.default_rng(D + H + T + KV)
    Q = rng.standard_normal((H, T, D)).astype(np.float32)
    K16 = f16(rng.standard_normal((HK, KV, D)))
    V16 = f16(rng.standard_normal((HK, KV, DV)))
    M = np.where(rng.uniform(size=(T, KV)) < 0.3, -np.inf, rng.uniform(-2, 0, (T, KV))).astype(np.float32)
    M[0, :] = -np.inf          # a fully masked row -> zeros
    M16 = f16(M)
    scale = 1.0 / math.sqrt(D)
    got = run_fa(torch, Q, K16, V16, M16, scale)
    want = oracle.flash_attn(Q, K16, V16, M16, scale, q_mode=2)
    assert np.all(got[0] == 0.0)
    assert float(np.max(np.abs(got - want))) / np.max(np.abs(want)) <= 1e-2


def test_fa_softcap_and_unmasked(cuda):
    import torch
    rng = np.random.default_rng(77)
    H, HK, D, T, KV = 8, 4, 128, 40, 1200
    Q = (rng.standard_normal((H, T, D)) * 3).astype(np.float32)
    K16 = f16(rng.standard_normal((HK, KV, D)))
    V16 = f16(rng.standard_normal((HK, KV, D)))
    scale = 1.0 / math.sqrt(D)
    for softcap, M16 in ((30.0, None), (0.0, None), (50.0, f16(np.zeros((T, KV), np.float32)))):
        got = run_fa(torch, Q, K16, V16, M16, scale, softcap=softcap)
        want = oracle.flash_attn(Q, K16, V16, M16, scale, softcap=softcap, q_mode=2)
        assert float(np.max(np.abs(got - want))) / np.max(np.abs(want)) <= 1e-2


def _q4_0(x):
    """x f32 [rows, n] -> Q4_0 blocks [rows, n / 32 * 18] (fp16 d, then 16 bytes: value j in the low
    nibble of byte j, value j + 16 in the high nibble) and the values those blocks decode to."""
    rows, n = x.shape
    v = x.reshape(rows, n // 32, 32).astype(np.float32)
    idx = np.argmax(np.abs(v), axis=-1)
    vmax = np.take_along_axis(v, idx[..., None], axis=-1)[..., 0]
    d = (vmax / -8.0).astype(np.float16)
    df = d.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(df[..., None] != 0, np.floor(v / df[..., None] + 8.5), 8).clip(0, 15).astype(np.uint8)
    out = np.zeros((rows, n // 32, 18), np.uint8)
    out[..., 0:2] = d.view(np.uint8).reshape(rows, n // 32, 2)
    out[..., 2:] = q[..., :16] | (q[..., 16:] << 4)
    dec = ((q.astype(np.float32) - 8.0) * df[..., None]).reshape(rows, n)
    return out.reshape(rows, -1), dec


@pytest.mark.parametrize("qtype", [8, 2])
def test_kv_to_f16_matches_the_decoders(cuda, qtype):
    """b200_kv_to_f16: a Q8_0 / Q4_0 KV-cache view with interleaved heads (rows nb1 apart, heads nb2)
    decodes to exactly ggml's dequantized values rounded to fp16."""
    import torch
    import ggml_b200 as g
    rng = np.random.default_rng(qtype)
    HK, KV, D = 4, 96, 128
    x = rng.standard_normal((KV, HK * D)).astype(np.float32)   # one cache row holds every head
    if qtype == 8:
        raw = oracle.quantize(8, x)
        dec = oracle.dequantize(8, raw, HK * D)
        bpb = 34
    else:
        raw, dec = _q4_0(x)
        bpb = 18
    src = torch.from_numpy(np.ascontiguousarray(raw).reshape(-1)).cuda()
    out = torch.empty(HK * KV * D, dtype=torch.float16, device="cuda")
    nb1, nb2 = raw.shape[1], D // 32 * bpb
    assert g.lib().b200_kv_to_f16(qtype, src.data_ptr(), D, KV, HK, nb1, nb2, out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    want = dec.reshape(KV, HK, D).transpose(1, 0, 2).astype(np.float16)
    assert np.array_equal(out.cpu().numpy().reshape(HK, KV, D).view(np.uint16), want.view(np.uint16))


_QKV_FA_CHILD = r"""
import math, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import numpy as np
import ggml_b200 as g
import oracle
from test_gpu_flash_attn import _q4_0
be = g.Backend()
rng = np.random.default_rng(5)
H, HK, D, T, KV = 8, 2, 128, 64, 1024
Q = rng.standard_normal((H, T, D)).astype(np.float32)
kf = rng.standard_normal((HK * KV, D)).astype(np.float32)
vf = rng.standard_normal((HK * KV, D)).astype(np.float32)
kraw = oracle.quantize(8, kf)                      # Q8_0 K, [HK][KV] rows of D
vraw, vdec = _q4_0(vf)                             # Q4_0 V
kdec = oracle.dequantize(8, kraw, D)
M = np.zeros((T, KV), np.float32)
for t in range(T):
    M[t, KV - T + t + 1:] = -np.inf
M16 = M.astype(np.float16)
out = np.full((T, H, D), np.nan, np.float32)
qt = g.make_tensor(g.F32, [D, T, H], np.ascontiguousarray(Q.transpose(0, 1, 2)), nb=[4, 4 * D, 4 * D * T, 4 * D * T * H])
kt = g.make_tensor(g.Q8_0, [D, KV, HK], kraw)
vt = g.make_tensor(g.Q4_0, [D, KV, HK], vraw)
mt = g.make_tensor(g.F16, [KV, T], M16)
d = g.make_tensor(g.F32, [D, H, T], out, op=g.OP_FLASH_ATTN_EXT, srcs=[qt, kt, vt, mt],
                  op_params=[1.0 / math.sqrt(D), 0.0, 0.0, 0])
assert g.supports_op(d)
assert be.graph_compute([d]) == g.STATUS_SUCCESS
K16 = kdec.reshape(HK, KV, D).astype(np.float16).view(np.uint16)
V16 = vdec.reshape(HK, KV, D).astype(np.float16).view(np.uint16)
want = oracle.flash_attn(Q, K16, V16, M16.view(np.uint16), 1.0 / math.sqrt(D), q_mode=2)
print("QKVFA", float(np.max(np.abs(out - want)) / np.max(np.abs(want))))
assert be.route_ops("fa_quant_kv") == 1 and be.device_errors() == 0 and be.cpu_fallbacks() == 0
be.close()
"""


def test_fa_over_a_quantized_kv_cache(cuda):
    """B200_FA_QUANT_KV=1: FLASH_ATTN_EXT with a Q8_0 K cache and a Q4_0 V cache runs through
    graph_compute (the cache converted to fp16 tiles, then the fp16 kernel) and matches the oracle on
    the decoded cache within the FA bound."""
    import os
    import subprocess
    import sys
    from conftest import ROOT
    env = dict(os.environ, B200_FA_QUANT_KV="1")
    p = subprocess.run([sys.executable, "-c", _QKV_FA_CHILD, ROOT], env=env, capture_output=True, text=True,
                       timeout=300)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]
    assert float(p.stdout.split("QKVFA")[1].split()[0]) <= 1e-2
