"""Python binding of libggml-b200.so (ctypes over the C ABI in include/).

The library is the product; this module only declares its entry points so tests, the
bench and the smoke check can call them with device pointers from torch tensors. Loading
fails loudly when the library has not been built: there is no Python or CPU fallback.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libggml-b200.so")

# ggml_type numbering
F32, F16, Q8_0, Q4_K, Q6_K, I32, BF16 = 0, 1, 8, 12, 14, 26, 30
TYPE_NAMES = {F32: "f32", F16: "f16", Q8_0: "q8_0", Q4_K: "q4_K", Q6_K: "q6_K", I32: "i32", BF16: "bf16"}
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

B200_OK = 0
STATUS = {0: "ok", -1: "invalid", -2: "unsupported", -3: "cuda", -4: "device", -5: "workspace",
          -6: "bad_ids", -7: "no_device"}


class B200Error(RuntimeError):
    pass


def row_size(t, k):
    be, bb = BLOCK[t]
    return (k // be) * bb


_lib = None

_c = ctypes
_vp, _i64, _int, _sz, _f = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_size_t, _c.c_float

_SIGS = {
    "b200_weight_packed_size": (_sz, [_int, _i64, _i64]),
    "b200_weight_pack": (_int, [_int, _vp, _i64, _i64, _vp, _vp]),
    "b200_dequantize": (_int, [_int, _vp, _i64, _i64, _int, _vp, _vp]),
    "b200_mul_mat_workspace_size": (_sz, [_i64, _i64, _i64]),
    "b200_mul_mat": (_int, [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp, _vp]),
}


def lib():
    """The loaded library; raises B200Error when it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise B200Error(f"{LIB_PATH} is not built (run ggml-rocket_b200/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            if hasattr(L, name):
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
        _lib = L
    return _lib


def declared_symbols():
    return sorted(_SIGS)


def check(rc, what):
    if rc != B200_OK:
        raise B200Error(f"{what} failed: {STATUS.get(rc, rc)}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


# ---- thin wrappers over torch device tensors -------------------------------------------------

def weight_packed_size(t, N, K):
    return lib().b200_weight_packed_size(t, N, K)


def weight_pack(t, src, N, K, dst, stream=None):
    check(lib().b200_weight_pack(t, _ptr(src), N, K, _ptr(dst), _stream(stream)), "weight_pack")


def dequantize(t, src, N, K, dst, f16_out=False, stream=None):
    check(lib().b200_dequantize(t, _ptr(src), N, K, 1 if f16_out else 0, _ptr(dst), _stream(stream)), "dequantize")


def mul_mat_workspace_size(M, N, K):
    return lib().b200_mul_mat_workspace_size(M, N, K)


def mul_mat(wtype, w_packed, N, K, a, M, out, workspace, dev_err, lda=None, ldd=None, stream=None):
    lda = K if lda is None else lda
    ldd = N if ldd is None else ldd
    check(lib().b200_mul_mat(wtype, _ptr(w_packed), N, K, _ptr(a), lda, M, _ptr(out), ldd,
                             _ptr(workspace), workspace.numel() * workspace.element_size(), _ptr(dev_err),
                             _stream(stream)), "mul_mat")
