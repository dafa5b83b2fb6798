"""Host-only claim-rule tests (no GPU), mirroring test-rocket-placement.cpp:415-557.

Differences from the reference are B200 facts, each stated at its case: the accumulator is
fp32 in tensor memory, so F32/BF16 accumulator declarations are met; the quantized floor
defaults to the dense one (the fused device dequant has no per-call host cost); attention needs
head dims of 64 or 128. Knob states are read once per process (as the reference's statics are),
so the knob cases run in child processes.
"""
import json
import os
import subprocess
import sys

import pytest

import ggml_b200 as g

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def mm(K, N, M, wt, op_params=None, src0_op=g.OP_NONE, readable=True):
    w = g.make_tensor(wt, [K, N], name="blk.0.attn_q.weight", op=src0_op, readable=readable)
    x = g.make_tensor(g.F32, [K, M])
    d = g.make_tensor(g.F32, [N, M], op=g.OP_MUL_MAT, srcs=[w, x], op_params=op_params)
    return d, (w, x)


def supported(*a, **k):
    d, keep = mm(*a, **k)
    return g.supports_op(d)


K, N, M, MQ = 256, 128, 256, 512


def test_mul_mat_weight_types():
    assert supported(K, N, M, g.F16)
    assert supported(K, N, M, g.F32)
    assert supported(K, N, M, g.BF16)
    assert supported(K, N, MQ, g.Q8_0)
    assert supported(K, N, MQ, g.Q4_K)
    assert supported(K, N, MQ, g.Q6_K)
    # B200: the quant floor defaults to the dense one (16, from a measured crossover), so M=256 is
    # claimed too
    assert supported(K, N, M, g.Q4_K)
    assert not supported(K, N, MQ, 2)          # Q4_0: no device decoder -> CPU


def test_mul_mat_shape_gates():
    assert not supported(80, N, M, g.F16)      # K % 32 != 0
    assert not supported(K, 70, M, g.F16)      # N % 16 != 0
    assert supported(K, 112, M, g.F16)         # N % 16 == 0
    assert not supported(32, N, M, g.F16)      # K < 64
    assert not supported(K, 48, M, g.F16)      # N < 64
    assert not supported(K, N, 1, g.F16)       # decode GEMV stays on the CPU
    assert supported(K, N, 16, g.F16)          # the default floor (16)
    assert not supported(K, N, 8, g.F16)       # below it
    assert not supported(384, N, MQ, g.Q4_K)   # K % 256 != 0 for a K-quant


def test_mul_mat_source_gates():
    assert not supported(K, N, M, g.F16, src0_op=g.OP_OTHER)   # computed (non-leaf) weight
    assert not supported(K, N, M, g.F16, readable=False)       # repacked bytes without a source
    d, keep = mm(K, N, M, g.F16)
    assert g.offload_op(d)
    a = g.make_tensor(g.F32, [K, M])
    add = g.make_tensor(g.F32, [K, M], op=g.OP_OTHER, srcs=[a, a])
    assert not g.offload_op(add)


def test_mul_mat_precision_declarations():
    # accumulator declarations: fp32 accumulation meets all of them (the reference declines F32/BF16)
    assert supported(K, N, M, g.F16, op_params=[10])
    assert supported(K, N, M, g.F16, op_params=[15])
    assert supported(K, N, M, g.F16, op_params=[20])
    # activation declarations: the activation is rounded to fp16
    assert not supported(K, N, M, g.F16, op_params=[0, 0, 0, 10])
    assert not supported(K, N, M, g.F16, op_params=[0, 0, 0, 15])
    assert supported(K, N, M, g.F16, op_params=[0, 0, 0, 20])
    assert supported(K, N, M, g.F16, op_params=[0, 0, 0, 30])
    # a Walsh-Hadamard src0 stays on the CPU's exact transform
    assert supported(128, 128, M, g.F32)
    assert not supported(128, 128, M, g.F32, op_params=[0, g.HINT_SRC0_IS_HADAMARD])


def fa(D, T, H, KV, HK, kv_type=g.F16, max_bias=0.0, masked=True, sinks=False, acc=0, DV=None):
    DV = D if DV is None else DV
    q = g.make_tensor(g.F32, [D, T, H])
    k = g.make_tensor(kv_type, [D, KV, HK])
    v = g.make_tensor(kv_type, [DV, KV, HK])
    m = g.make_tensor(g.F16, [KV, T + 3]) if masked else None
    s = g.make_tensor(g.F32, [H]) if sinks else None
    d = g.make_tensor(g.F32, [DV, H, T], op=g.OP_FLASH_ATTN_EXT, srcs=[q, k, v, m, s],
                      op_params=[0.125, float(max_bias), 0.0, acc])
    return g.supports_op(d)


def test_flash_attn_gates():
    assert fa(64, 256, 8, 1024, 2)
    assert fa(64, 256, 8, 1024, 2, acc=10)     # F32 accumulator declared: met
    assert fa(128, 512, 32, 4096, 8)           # the BASELINE shape
    assert not fa(64, 1, 8, 1024, 2)           # decode
    assert not fa(64, 256, 8, 512, 2)          # short context
    assert not fa(48, 256, 8, 1024, 2)         # head_dim % 32 != 0
    assert not fa(96, 256, 8, 1024, 2)         # B200: head dims 64 / 128 only
    assert not fa(64, 256, 8, 1024, 2, kv_type=g.F32)
    assert not fa(64, 256, 8, 1024, 2, kv_type=g.Q8_0)   # a quantized cache needs B200_FA_QUANT_KV=1
    assert not fa(64, 256, 8, 1024, 2, max_bias=8.0)
    assert not fa(64, 256, 8, 1024, 2, masked=False)   # unmasked needs B200_FLASH_ATTN_UNMASKED=1
    assert not fa(64, 256, 8, 1024, 2, sinks=True)     # attention sinks: a different softmax
    assert not fa(64, 256, 6, 1024, 4)                 # GQA does not divide


def moe(n_tokens, n_used, n_expert, K=2048, N=768, wt=g.Q4_K, name="blk.0.ffn_up_exps.weight"):
    a = g.make_tensor(wt, [K, N, n_expert], name=name)
    b = g.make_tensor(g.F32, [K, 1, n_tokens])
    ids = g.make_tensor(g.I32, [n_used, n_tokens])
    d = g.make_tensor(g.F32, [N, n_used, n_tokens], op=g.OP_MUL_MAT_ID, srcs=[a, b, ids])
    return g.supports_op(d)


def test_moe_auto_defaults():
    assert moe(2048, 8, 128)                   # M_e = 128
    assert moe(512, 4, 32, K=2880, N=2880, wt=g.Q8_0)   # gpt-oss-like shape (K % 32)
    assert not moe(16, 8, 128)                 # below the token floor
    assert not moe(64, 1, 128)                 # M_e = 0 < bucket floor
    assert not moe(2048, 8, 128, K=2000)       # K % 256 != 0 for Q4_K


def glue(kind):
    """Descriptors of the glue ops the B200_GLUE claim rules accept or decline."""
    x = g.make_tensor(g.F32, [128, 8, 4])
    pos = g.make_tensor(g.I32, [4])
    if kind == "rms":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_RMS_NORM, srcs=[x], op_params=[1e-5])
    elif kind == "add_bcast":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_ADD, srcs=[x, g.make_tensor(g.F32, [128])])
    elif kind == "add_norepeat":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_ADD, srcs=[x, g.make_tensor(g.F32, [100])])
    elif kind == "silu":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_UNARY, srcs=[x], op_params=[g.UNARY_SILU])
    elif kind == "gelu":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_UNARY, srcs=[x], op_params=[-1])
    elif kind == "swiglu1":
        d = g.make_tensor(g.F32, [64, 8, 4], op=g.OP_GLU, srcs=[x], op_params=[g.GLU_SWIGLU, 0])
    elif kind in ("rope", "rope_yarn", "rope_mrope"):
        ext = 1.0 if kind == "rope_yarn" else 0.0
        mode = 8 if kind == "rope_mrope" else 2
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_ROPE, srcs=[x, pos],
                          op_params=[0, 128, mode, 0, 4096, 10000.0, 1.0, ext, 1.0, 32.0, 1.0])
    elif kind == "get_rows_q4k":
        d = g.make_tensor(g.F32, [256, 4], op=g.OP_GET_ROWS,
                          srcs=[g.make_tensor(g.Q4_K, [256, 100]), g.make_tensor(g.I32, [4])])
    elif kind == "get_rows_f16":
        d = g.make_tensor(g.F32, [256, 4], op=g.OP_GET_ROWS,
                          srcs=[g.make_tensor(g.F16, [256, 100]), g.make_tensor(g.I32, [4])])
    elif kind == "cpy_f16":
        d = g.make_tensor(g.F16, [128, 8, 4], op=g.OP_CPY, srcs=[x])
    elif kind == "soft_max":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_SOFT_MAX, srcs=[x], op_params=[1.0, 0.0])
    elif kind == "soft_max_mask":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_SOFT_MAX, srcs=[x, g.make_tensor(g.F32, [128, 8])],
                          op_params=[1.0, 0.0])
    elif kind == "argsort":
        d = g.make_tensor(g.I32, [128, 8, 4], op=g.OP_ARGSORT, srcs=[x], op_params=[1])
    elif kind == "argsort_wide":
        d = g.make_tensor(g.I32, [2048, 3], op=g.OP_ARGSORT, srcs=[g.make_tensor(g.F32, [2048, 3])], op_params=[1])
    elif kind == "sum_rows":
        d = g.make_tensor(g.F32, [1, 8, 4], op=g.OP_SUM_ROWS, srcs=[x])
    elif kind == "div":
        d = g.make_tensor(g.F32, [128, 8, 4], op=g.OP_DIV, srcs=[x, g.make_tensor(g.F32, [1, 8, 4])])
    else:
        raise ValueError(kind)
    return g.supports_op(d)


GLUE_KINDS = ("rms", "add_bcast", "add_norepeat", "silu", "gelu", "swiglu1", "rope", "rope_yarn", "rope_mrope",
              "get_rows_q4k", "get_rows_f16", "cpy_f16", "soft_max", "soft_max_mask", "argsort", "argsort_wide",
              "sum_rows", "div")


_CHILD = r"""
import json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import test_placement as t
print(json.dumps({"q4k_m256": t.supported(256, 128, 256, 12), "q4k_m512": t.supported(256, 128, 512, 12),
                  "f16_m16": t.supported(256, 128, 16, 1), "f16_m3": t.supported(256, 128, 3, 1),
                  "q4k_m1": t.supported(256, 128, 1, 12), "q4k_m8": t.supported(256, 128, 8, 12),
                  "q4k_m9": t.supported(256, 128, 9, 12), "q8_m1": t.supported(256, 128, 1, 8),
                  "q6k_m12": t.supported(256, 128, 12, 14), "f16_m1": t.supported(256, 128, 1, 1),
                  "q4k_m40": t.supported(256, 128, 40, 12),
                  "moe": t.moe(2048, 8, 128), "fa_unmasked": t.fa(64, 256, 8, 1024, 2, masked=False),
                  "fa": t.fa(64, 256, 8, 1024, 2), "glue": {k: t.glue(k) for k in t.GLUE_KINDS}}))
"""


def child(env):
    e = dict(os.environ)
    for k in list(e):
        if k.startswith("B200_"):
            del e[k]
    e.update(env)
    out = subprocess.run([sys.executable, "-c", _CHILD, ROOT], env=e, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_knobs_in_children():
    r = child({"B200_MIN_M_QUANT": "512"})
    assert not r["q4k_m256"] and r["q4k_m512"]
    r = child({"B200_MIN_M": "32"})                # the reference's default
    assert not r["f16_m16"]
    r = child({"B200_MIN_M": "1"})                 # floor of 4
    assert not r["f16_m3"]
    r = child({"B200_MIN_M": ""})                  # set-but-empty reads as unset (16)
    assert r["f16_m16"]
    r = child({"B200_MOE": "0"})
    assert not r["moe"]
    r = child({"B200_MOE": "1"})
    assert r["moe"]
    r = child({"B200_MOE_MIN_WORK": "1000"})       # 128 * 2048 * 768 = 201 MMAC < 1000
    assert not r["moe"]
    r = child({"B200_FLASH_ATTN_UNMASKED": "1"})
    assert r["fa_unmasked"]
    r = child({"B200_FLASH_ATTN": "0"})
    assert not r["fa"]
    r = child({"B200_FLASH_ATTN_MIN_KV": "2048"})
    assert not r["fa"]
    r = child({})                                  # decode-size MUL_MAT stays on the host by default
    assert not r["q4k_m1"] and not r["q4k_m8"]
    assert not any(r["glue"].values())             # glue ops stay on the host by default
    r = child({"B200_GLUE": "1"})
    assert r["glue"] == {"rms": True, "add_bcast": True, "add_norepeat": False, "silu": True, "gelu": False,
                         "swiglu1": True, "rope": True, "rope_yarn": False, "rope_mrope": False,
                         "get_rows_q4k": False, "get_rows_f16": True, "cpy_f16": True, "soft_max": True,
                         "soft_max_mask": False, "argsort": True, "argsort_wide": False, "sum_rows": True,
                         "div": True}
    r = child({"B200_DECODE": "1"})                # quantized weights below the floor, M <= 32
    assert r["q4k_m1"] and r["q4k_m8"] and r["q4k_m9"] and r["q8_m1"] and r["q6k_m12"] and not r["f16_m1"]
    r = child({"B200_DECODE": "1", "B200_MIN_M_QUANT": "64"})
    assert r["q4k_m9"] and not r["q4k_m40"]        # M = 33 .. 63: neither the decode kernel nor the GEMM


def test_moe_ledger_budget_in_child():
    code = r"""
import sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import test_placement as t
# four 113 MB Q4_K stacks against a 300 MB budget: two fit; each stack is decided once
r = [t.moe(2048, 8, 128, name=f"blk.{i}.ffn_up_exps.weight") for i in range(4)]
again = t.moe(2048, 8, 128, name="blk.0.ffn_up_exps.weight")
print(sum(r), r[0], again)
"""
    e = dict(os.environ)
    e["B200_WEIGHT_BUDGET_MB"] = "300"
    out = subprocess.run([sys.executable, "-c", code, ROOT], env=e, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    n, first, again = out.stdout.split()
    assert n == "2" and first == "True" and again == "True"


def test_weight_key_identity():
    import numpy as np
    a = np.arange(4096, dtype=np.uint8)
    b = (a + 1).astype(np.uint8)               # new bytes throughout (the fingerprint samples 16 x 64 B)
    w1 = g.make_tensor(g.F16, [64, 32], a, name="blk.3.ffn_down.weight")
    w2 = g.make_tensor(g.F16, [64, 32], b, name="blk.3.ffn_down.weight")
    w3 = g.make_tensor(g.F16, [64, 32], a, name="B200#blk.3.ffn_down.weight#1")
    k1, k2, k3 = g.weight_key(w1), g.weight_key(w2), g.weight_key(w3)
    assert k1 != k2                            # same name, new bytes -> a different key
    assert k1 == k3                            # the scheduler's copy name maps to the weight
    assert g.weight_key(g.make_tensor(g.F16, [64, 32], a, name="leaf_12")) == ""
    assert g.weight_key(g.make_tensor(g.F16, [64, 32], a, name="")) == ""


def test_breaker_semantics():
    """ggml-rocket.cpp:263-307 / test-rocket-internals.cpp:535-561: three consecutive device
    failures open the route for 64 calls; a failed probe doubles the interval (cap 4096); a
    structural decline (unsupported) does not count; a success closes it."""
    DEV, UNS = -4, -2
    r = g.breaker_replay([DEV, DEV, DEV] + [0] * 64 + [DEV] + [0] * 130 + [0])
    assert r[:3] == [1, 1, 1]
    assert r[3:67] == [0] * 64                 # open for 64 calls
    assert r[67] == 1                          # the probe (fails)
    assert r[68:68 + 128] == [0] * 128         # reopened for twice as long
    assert r[196] == 1
    r = g.breaker_replay([UNS] * 10 + [0])
    assert all(x == 1 for x in r)              # declines never open it
    r = g.breaker_replay([DEV, DEV, 0, DEV, DEV, 0])
    assert all(x == 1 for x in r)              # a success resets the count


_HADAMARD_CHILD = r"""
import json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200")
import numpy as np
import ggml_b200 as g


def sylvester(n):
    i = np.arange(n)
    return np.where(np.bitwise_count(i[:, None] & i[None, :]) % 2 == 1, -1.0, 1.0)


def claim(h, wt, n, hint=True, m=7):
    arr = np.ascontiguousarray(h.astype(np.float16 if wt == g.F16 else np.float32))   # alive while claimed
    w = g.make_tensor(wt, [n, n], arr)
    x = g.make_tensor(g.F32, [n, m])
    d = g.make_tensor(g.F32, [n, m], op=g.OP_MUL_MAT, srcs=[w, x],
                      op_params=[0, g.HINT_SRC0_IS_HADAMARD if hint else 0])
    return g.supports_op(d)


out = {}
for n in (32, 128, 1024):
    h = sylvester(n) / np.sqrt(n)
    out[f"f32_{n}"] = claim(h, g.F32, n)
    out[f"f16_{n}"] = claim(h.astype(np.float16), g.F16, n)
h = sylvester(128)
out["unscaled"] = claim(h, g.F32, 128)
out["permuted"] = claim(h[::-1].copy(), g.F32, 128)                   # not the Sylvester order
bad = h.copy(); bad[5, 9] *= 0.5
out["one_entry_off"] = claim(bad, g.F32, 128)
out["n_16"] = claim(sylvester(16), g.F32, 16)
print(json.dumps(out))
"""


@pytest.mark.parametrize("glue", ["0", "1"])
def test_hadamard_tagged_mul_mat_claim(glue):
    """A MUL_MAT under ggml's Walsh-Hadamard hint: declined by default, as the reference does;
    with the glue ops claimed (B200_GLUE=1) claimed exactly when src0 is c times the
    Sylvester-ordered Hadamard matrix of order 32..1024 (F32 or F16), for the device transform."""
    e = dict(os.environ, B200_GLUE=glue)
    p = subprocess.run([sys.executable, "-c", _HADAMARD_CHILD, ROOT], env=e, capture_output=True, text=True,
                       timeout=120)
    assert p.returncode == 0, p.stderr[-2000:]
    r = json.loads(p.stdout.strip().splitlines()[-1])
    on = glue == "1"
    for n in (32, 128, 1024):
        assert r[f"f32_{n}"] == on and r[f"f16_{n}"] == on, (n, r)
    assert r["unscaled"] == on
    assert not r["permuted"] and not r["one_entry_off"] and not r["n_16"]


_QKV_CHILD = r"""
import json, sys
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/ggml-rocket_b200"); sys.path.insert(0, sys.argv[1] + "/tests")
import ggml_b200 as g
import test_placement as t
print(json.dumps({"q8": t.fa(64, 256, 8, 1024, 2, kv_type=g.Q8_0), "q4_0": t.fa(128, 512, 32, 4096, 8, kv_type=g.Q4_0),
                  "q4k": t.fa(128, 512, 32, 4096, 8, kv_type=g.Q4_K), "f16": t.fa(64, 256, 8, 1024, 2)}))
"""


def test_flash_attn_quantized_kv_claim_in_child():
    """B200_FA_QUANT_KV=1: FLASH_ATTN_EXT over a Q8_0 or Q4_0 KV cache is claimed (converted to fp16
    tiles on the device); other quantized cache types stay declined, F16 is unchanged."""
    e = dict(os.environ, B200_FA_QUANT_KV="1")
    p = subprocess.run([sys.executable, "-c", _QKV_CHILD, ROOT], env=e, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr[-2000:]
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert r == {"q8": True, "q4_0": True, "q4k": False, "f16": True}, r
