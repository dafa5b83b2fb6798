"""ctypes loader for the CPU oracle (oracle.c) -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs use this,
and only as the checker or the timed CPU baseline; the product never imports it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SO = os.path.join(HERE, "_build", "liboracle.so")
# the CPU MUL_MAT path restated for timing (cpu_path.c): its AVX2 kernel is chosen at run time, so
# the .so runs on whichever host it travels to
SO_PATH = os.path.join(HERE, "_build", "libcpupath.so")


def build():
    os.makedirs(os.path.dirname(SO), exist_ok=True)
    src = os.path.join(HERE, "oracle.c")
    hdr = os.path.join(HERE, "oracle.h")
    if not (os.path.exists(SO) and os.path.getmtime(SO) >= max(os.path.getmtime(src), os.path.getmtime(hdr))):
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-Wall", "-Wextra",
                               "-o", SO, src, "-lm"])
    psrc = os.path.join(HERE, "cpu_path.c")
    if not (os.path.exists(SO_PATH) and os.path.getmtime(SO_PATH) >= os.path.getmtime(psrc)):
        subprocess.check_call(["gcc", "-O3", "-ffp-contract=off", "-fPIC", "-shared", "-fopenmp", "-Wall", "-Wextra",
                               "-o", SO_PATH, psrc, "-lm"])
    return SO


_L = None
_LP = None
_vp, _i64, _int, _f = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float


def lib():
    global _L
    if _L is None:
        if not os.path.exists(SO):
            build()
        L = ctypes.CDLL(SO)
        L.orc_fp32_to_fp16_row.argtypes = [_vp, _vp, _i64]
        L.orc_fp16_to_fp32_row.argtypes = [_vp, _vp, _i64]
        L.orc_row_size.restype = ctypes.c_size_t
        L.orc_row_size.argtypes = [_int, _i64]
        L.orc_dequantize_row.argtypes = [_int, _vp, _vp, _i64]
        L.orc_quantize_row.argtypes = [_int, _vp, _vp, _i64]
        L.orc_pack_act.argtypes = [_vp, _i64, _i64, _i64, _vp, _vp]
        L.orc_mul_mat_f64.argtypes = [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _int]
        L.orc_flash_attn_f64.argtypes = [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
                                         _vp, _i64, _vp, _int, _int, _int, _int, _int, _int, _f, _f, _int, _int]
        L.orc_moe_route.argtypes = [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp]
        L.orc_mul_mat_id_f64.argtypes = [_int, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
                                         _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _int]
        L.orc_rms_norm.argtypes = [_vp, _i64, _i64, _f, _vp]
        L.orc_silu.argtypes = [_vp, _i64, _vp]
        L.orc_swiglu.argtypes = [_vp, _vp, _i64, _vp]
        L.orc_rope.argtypes = [_vp, _i64, _i64, _i64, _vp, _int, _int, _f, _f, _f, _vp]
        L.orc_soft_max.argtypes = [_vp, _i64, _i64, _f, _vp]
        _L = L
    return _L


def path_lib():
    global _LP
    if _LP is None:
        if not os.path.exists(SO_PATH):
            build()
        L = ctypes.CDLL(SO_PATH)
        L.orc_cpu_path_mul_mat_q4k.argtypes = [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _int]
        _LP = L
    return _LP


def cpu_path_mul_mat_q4k(w_raw, N, K, a, nthreads=0):
    """The host CPU's Q4_K MUL_MAT path restated for timing (cpu_path.c): activations quantized to
    8-bit blocks of 256, integer block dot products. Within ~1e-2 of mul_mat()."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    w_raw = np.ascontiguousarray(w_raw)
    M = a.shape[0]
    c = np.zeros((M, N), dtype=np.float32)
    rc = path_lib().orc_cpu_path_mul_mat_q4k(_p(w_raw), N, K, _p(a), K, M, _p(c), N, nthreads)
    assert rc == 0
    return c


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def row_size(t, k):
    return lib().orc_row_size(t, k)


def quantize(t, x):
    """x: float32 [N, K] -> uint8 [N, row_size] ggml blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    N, K = x.shape
    out = np.zeros((N, row_size(t, K)), dtype=np.uint8)
    for n in range(N):
        rc = lib().orc_quantize_row(t, ctypes.c_void_p(x[n].ctypes.data), ctypes.c_void_p(out[n].ctypes.data), K)
        assert rc == 0
    return out


def dequantize(t, raw, K):
    raw = np.ascontiguousarray(raw)
    N = raw.shape[0]
    out = np.zeros((N, K), dtype=np.float32)
    for n in range(N):
        rc = lib().orc_dequantize_row(t, ctypes.c_void_p(raw[n].ctypes.data), ctypes.c_void_p(out[n].ctypes.data), K)
        assert rc == 0
    return out


def fp16_bits(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros(x.shape, dtype=np.uint16)
    lib().orc_fp32_to_fp16_row(_p(x), _p(y), x.size)
    return y


def pack_act(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    M, K = a.shape
    a16 = np.zeros((M, K), dtype=np.uint16)
    s = np.zeros(M, dtype=np.float32)
    lib().orc_pack_act(_p(a), M, K, K, _p(a16), _p(s))
    return a16, s


def mul_mat(t, w_raw, N, K, a, nthreads=0):
    a = np.ascontiguousarray(a, dtype=np.float32)
    w_raw = np.ascontiguousarray(w_raw)
    M = a.shape[0]
    c = np.zeros((M, N), dtype=np.float32)
    rc = lib().orc_mul_mat_f64(t, _p(w_raw), N, K, _p(a), K, M, _p(c), N, nthreads)
    assert rc == 0
    return c


def flash_attn(q, k, v, mask, scale, softcap=0.0, q_mode=0, nthreads=0):
    """q F32 [H, T, D] (ggml [D, T, H]), k/v fp16 bits [HK, KV, D], mask fp16 bits [T, KV] or None.
    Returns F32 [T, H, DV] (ggml dst [DV, H, T])."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    H, T, D = q.shape
    HK, KV, DV = v.shape
    out = np.zeros((T, H, DV), dtype=np.float32)
    m_nb1 = 0
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint16)
        m_nb1 = mask.shape[1] * 2
    rc = lib().orc_flash_attn_f64(_p(q), 4, D * 4, T * D * 4, _p(k), 2, D * 2, KV * D * 2,
                                  _p(v), 2, DV * 2, KV * DV * 2, _p(mask), m_nb1, _p(out),
                                  D, DV, T, H, KV, HK, scale, softcap, q_mode, nthreads)
    assert rc == 0
    return out


def moe_route(ids, n_expert):
    """ids int32 [n_tokens, n_used] (ggml [n_used, n_tokens]) -> (off, slot, tok) or None on a bad id."""
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n_tokens, n_used = ids.shape
    off = np.zeros(n_expert + 1, dtype=np.int32)
    slot = np.zeros(max(1, n_tokens * n_used), dtype=np.int32)
    tok = np.zeros(max(1, n_tokens * n_used), dtype=np.int32)
    rc = lib().orc_moe_route(_p(ids), 4, n_used * 4, n_used, n_tokens, n_expert, _p(off), _p(slot), _p(tok))
    if rc:
        return None
    return off, slot[:n_tokens * n_used], tok[:n_tokens * n_used]


def mul_mat_id(t, as_raw, K, N, n_expert, b, ids, nthreads=0):
    """as_raw uint8 [n_expert, N, row_size]; b F32 [n_tokens, ne11, K]; ids int32 [n_tokens, n_used].
    Returns F32 [n_tokens, n_used, N] (ggml dst [N, n_used, n_tokens])."""
    as_raw = np.ascontiguousarray(as_raw)
    b = np.ascontiguousarray(b, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    n_tokens, ne11, _ = b.shape
    n_used = ids.shape[1]
    dst = np.zeros((n_tokens, n_used, N), dtype=np.float32)
    rb = row_size(t, K)
    rc = lib().orc_mul_mat_id_f64(t, _p(as_raw), N * rb, K, N, n_expert, _p(b), K * 4, ne11 * K * 4, ne11,
                                  _p(ids), 4, n_used * 4, n_used, n_tokens, _p(dst), N * 4, n_used * N * 4, nthreads)
    if rc:
        return None
    return dst


# ---- glue ops (ggml CPU definitions; unpinned: ggml is absent) ----------------------------------

def rms_norm(x, eps):
    """x [..., n] f32 -> ggml rms_norm over the last axis."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    n = x.shape[-1]
    lib().orc_rms_norm(_p(x), x.size // n, n, eps, _p(y))
    return y


def silu(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_silu(_p(x), x.size, _p(y))
    return y


def swiglu(a, g):
    a = np.ascontiguousarray(a, dtype=np.float32)
    g = np.ascontiguousarray(g, dtype=np.float32)
    y = np.empty_like(a)
    lib().orc_swiglu(_p(a), _p(g), a.size, _p(y))
    return y


def rope(x, pos, n_dims, mode, freq_base, freq_scale=1.0, attn_factor=1.0):
    """x [n_tokens, n_head, head_dim] f32, pos [n_tokens] i32 -> ggml rope (ext_factor 0)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    y = np.empty_like(x)
    T, H, D = x.shape
    lib().orc_rope(_p(x), D, H, T, _p(pos), n_dims, mode, freq_base, freq_scale, attn_factor, _p(y))
    return y


def soft_max(x, scale=1.0):
    """x [..., n] f32 -> ggml soft_max (no mask) over the last axis."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    n = x.shape[-1]
    lib().orc_soft_max(_p(x), x.size // n, n, scale, _p(y))
    return y
