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
Q4_0 = 2
TYPE_NAMES = {F32: "f32", F16: "f16", Q8_0: "q8_0", Q4_K: "q4_K", Q6_K: "q6_K", I32: "i32", BF16: "bf16"}
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

B200_OK = 0
STATUS = {0: "ok", -1: "invalid", -2: "unsupported", -3: "cuda", -4: "device", -5: "workspace",
          -6: "bad_ids", -7: "no_device", -8: "too_large"}
B200_E_INVALID, B200_E_UNSUPPORTED, B200_E_WORKSPACE, B200_E_TOO_LARGE = -1, -2, -5, -8


class B200Error(RuntimeError):
    pass


def row_size(t, k):
    be, bb = BLOCK[t]
    return (k // be) * bb


_lib = None

_c = ctypes
_vp, _i64, _int, _sz, _f = _c.c_void_p, _c.c_int64, _c.c_int, _c.c_size_t, _c.c_float
_pint = _c.POINTER(_c.c_int)

_SIGS = {
    "b200_weight_packed_size": (_sz, [_int, _i64, _i64]),
    "b200_weight_pack": (_int, [_int, _vp, _i64, _i64, _vp, _vp]),
    "b200_dequantize": (_int, [_int, _vp, _i64, _i64, _int, _vp, _vp]),
    "b200_mul_mat_workspace_size": (_sz, [_int, _i64, _i64, _i64]),
    "b200_mul_mat": (_int, [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp, _vp]),
    "b200_act_pack": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "b200_swiglu_act_pack": (_int, [_vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _vp]),
    "b200_gemm_packed_workspace_size": (_sz, [_int, _i64, _i64, _i64]),
    "b200_gemm_packed": (_int, [_int, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _sz, _vp, _vp]),
    "b200_mul_mat_plan": (_int, [_int, _i64, _i64, _i64, _pint, _pint, _pint, _pint]),
    "b200_gemm_packed_group_workspace_size": (_sz, [_int, _int, _i64, _vp, _i64]),
    "b200_gemm_packed_group": (_int, [_int, _int, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _vp, _sz, _vp, _vp]),
    "b200_gemm_packed_group_plan": (_int, [_int, _int, _i64, _vp, _i64, _pint, _pint, _pint]),
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


# codes kernels record in a device error word (first writer wins)
DEVICE_ERRORS = {1: "wait_producer", 2: "wait_mma", 3: "wait_epilogue", 4: "wait_dequant", 5: "wait_drain",
                 6: "bad_index", 7: "wait_peer", 8: "wait_stream", 100: "bad_ids"}


def check_device(err, what):
    """Read a device error word (synchronises with the work that wrote it) and raise on a nonzero code."""
    code = int(err.item())
    if code != 0:
        raise B200Error(f"{what}: device error {DEVICE_ERRORS.get(code, code)}")


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


def mul_mat_workspace_size(M, N, K, wtype=F16):
    return lib().b200_mul_mat_workspace_size(wtype, M, N, K)


def mul_mat(wtype, w_packed, N, K, a, M, out, workspace, dev_err, lda=None, ldd=None, stream=None):
    lda = K if lda is None else lda
    ldd = N if ldd is None else ldd
    check(lib().b200_mul_mat(wtype, _ptr(w_packed), N, K, _ptr(a), lda, M, _ptr(out), ldd,
                             _ptr(workspace), workspace.numel() * workspace.element_size(), _ptr(dev_err),
                             _stream(stream)), "mul_mat")


def act_pack(a, M, K, a16, scales, lda=None, stream=None):
    lda = K if lda is None else lda
    check(lib().b200_act_pack(_ptr(a), lda, M, K, _ptr(a16), _ptr(scales), _stream(stream)), "act_pack")


def swiglu_act_pack(gate, up, M, F, a16, scales, ldg=None, ldu=None, stream=None):
    """a16 / scales = the activation pack of silu(gate) * up (b200_swiglu_act_pack)."""
    ldg = F if ldg is None else ldg
    ldu = F if ldu is None else ldu
    check(lib().b200_swiglu_act_pack(_ptr(gate), ldg, _ptr(up), ldu, M, F, _ptr(a16), _ptr(scales), _stream(stream)),
          "swiglu_act_pack")


def gemm_packed_workspace_size(M, N, K, wtype=F16):
    return lib().b200_gemm_packed_workspace_size(wtype, M, N, K)


def gemm_packed(wtype, w_packed, N, K, a16, scales, M, out, workspace, dev_err, ldd=None, stream=None):
    ldd = N if ldd is None else ldd
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().b200_gemm_packed(wtype, _ptr(w_packed), N, K, _ptr(a16), _ptr(scales), M, _ptr(out), ldd,
                                 _ptr(workspace), wsb, _ptr(dev_err), _stream(stream)), "gemm_packed")


def _i64_array(vals):
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def gemm_packed_group_workspace_size(M, Ns, K, wtype=F16):
    return lib().b200_gemm_packed_group_workspace_size(len(Ns), wtype, M, _i64_array(Ns), K)


def gemm_packed_group(wtype, w_packed, Ns, K, a16, scales, M, outs, workspace, dev_err, ldds=None, stream=None):
    """One combined-N GEMM launch over several weights (the fused group) against one packed
    activation: outs[m] = scales * (a16 . W_m^T)."""
    n = len(Ns)
    ldds = list(Ns) if ldds is None else ldds
    ws_arr = (ctypes.c_void_p * n)(*[_ptr(w) for w in w_packed])
    out_arr = (ctypes.c_void_p * n)(*[_ptr(o) for o in outs])
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(lib().b200_gemm_packed_group(n, wtype, ws_arr, _i64_array(Ns), K, _ptr(a16), _ptr(scales), M, out_arr,
                                       _i64_array(ldds), _ptr(workspace), wsb, _ptr(dev_err), _stream(stream)),
          "gemm_packed_group")


def gemm_packed_group_plan(M, Ns, K, wtype=F16):
    vals = [ctypes.c_int(0) for _ in range(3)]
    check(lib().b200_gemm_packed_group_plan(len(Ns), wtype, M, _i64_array(Ns), K, *[ctypes.byref(v) for v in vals]),
          "gemm_packed_group_plan")
    return dict(token_tile=vals[0].value, splits=vals[1].value, grid=vals[2].value)


def mul_mat_plan(M, N, K, wtype=F16):
    vals = [ctypes.c_int(0) for _ in range(4)]
    check(lib().b200_mul_mat_plan(wtype, M, N, K, *[ctypes.byref(v) for v in vals]), "mul_mat_plan")
    return dict(token_tile=vals[0].value, splits=vals[1].value, grid=vals[2].value, launches=vals[3].value)


# ---- backend-level API (include/ggml-b200.h) -------------------------------------------------

OP_NONE, OP_RESHAPE, OP_VIEW, OP_PERMUTE, OP_TRANSPOSE, OP_MUL_MAT, OP_MUL_MAT_ID, OP_FLASH_ATTN_EXT, OP_OTHER = range(9)
OP_RMS_NORM, OP_ADD, OP_MUL, OP_UNARY, OP_GLU, OP_ROPE, OP_GET_ROWS, OP_CPY = range(9, 17)
OP_SOFT_MAX, OP_ARGSORT, OP_SUM_ROWS, OP_DIV = range(17, 21)
UNARY_SILU, GLU_SWIGLU = 1, 2
STATUS_SUCCESS, STATUS_FAILED = 0, -1
PREC_F32, PREC_BF16, PREC_F16, PREC_Q8, PREC_Q4 = 10, 15, 20, 30, 40
HINT_SRC0_IS_HADAMARD = 1


class Tensor(ctypes.Structure):
    pass


Tensor._fields_ = [
    ("type", ctypes.c_int32),
    ("op", ctypes.c_int32),
    ("ne", ctypes.c_int64 * 4),
    ("nb", ctypes.c_size_t * 4),
    ("op_params", ctypes.c_int32 * 16),
    ("src", ctypes.POINTER(Tensor) * 10),
    ("data", ctypes.c_void_p),
    ("on_device", ctypes.c_int32),
    ("readable", ctypes.c_int32),
    ("name", ctypes.c_char * 64),
]

_TP = ctypes.POINTER(Tensor)
_BACKEND_SIGS = {
    "ggml_backend_b200_reg_name": (ctypes.c_char_p, []),
    "ggml_backend_b200_reg_device_count": (_int, []),
    "ggml_backend_b200_op_from_name": (_int, [ctypes.c_char_p]),
    "ggml_backend_b200_device_name": (ctypes.c_char_p, [_int]),
    "ggml_backend_b200_device_description": (_int, [_int, ctypes.c_char_p, _sz]),
    "ggml_backend_b200_device_memory": (_int, [_int, _c.POINTER(_sz), _c.POINTER(_sz)]),
    "ggml_backend_b200_supports_op": (ctypes.c_bool, [_TP]),
    "ggml_backend_b200_offload_op": (ctypes.c_bool, [_TP]),
    "ggml_backend_b200_init": (_vp, []),
    "ggml_backend_b200_free": (None, [_vp]),
    "ggml_backend_is_b200": (ctypes.c_bool, [_vp]),
    "ggml_backend_b200_set_n_gpus": (None, [_vp, _int]),
    "ggml_backend_b200_moe_stats": (None, [_vp, _c.POINTER(_c.c_long), _c.POINTER(_c.c_long)]),
    "ggml_backend_b200_route_ops": (_c.c_long, [_vp, ctypes.c_char_p]),
    "ggml_backend_b200_cpu_fallbacks": (_c.c_long, [_vp]),
    "ggml_backend_b200_device_errors": (_c.c_long, [_vp]),
    "ggml_backend_b200_graph_compute": (_int, [_vp, _c.POINTER(_TP), _int]),
    "ggml_backend_b200_weight_cache_bytes": (_sz, [_vp, _c.POINTER(_c.c_long)]),
    "ggml_backend_b200_weight_key": (_sz, [_TP, ctypes.c_char_p, _sz]),
    "ggml_backend_b200_breaker_replay": (None, [_c.POINTER(_int), _int, _c.POINTER(_int)]),
    "ggml_backend_b200_subop_from_name": (_int, [ctypes.c_char_p]),
    "b200_rms_norm": (_int, [_vp, _vp, _vp, _f, _vp, _vp]),
    "b200_rms_norm_mul": (_int, [_vp, _vp, _vp, _f, _vp, _vp, _vp, _vp]),
    "b200_add_rms_norm_mul": (_int, [_vp, _vp, _vp, _f, _vp, _vp, _vp, _vp, _vp]),
    "b200_rms_norm_mul_act_pack": (_int, [_vp, _vp, _vp, _f, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "b200_hadamard": (_int, [_vp, _vp, _vp, _f, _vp, _vp]),
    "b200_kv_to_f16": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp]),
    "b200_binary": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "b200_silu": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "b200_swiglu": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "b200_rope": (_int, [_vp, _vp, _vp, _vp, _int, _int, _f, _f, _f, _vp, _vp]),
    "b200_rope_f16": (_int, [_vp, _vp, _vp, _vp, _int, _int, _f, _f, _f, _vp, _vp, _vp]),
    "b200_get_rows": (_int, [_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "b200_cpy": (_int, [_int, _vp, _vp, _vp, _int, _vp, _vp, _vp, _vp]),
    "b200_soft_max": (_int, [_vp, _vp, _vp, _f, _vp, _vp]),
    "b200_argsort": (_int, [_vp, _vp, _vp, _int, _vp, _vp]),
    "b200_sum_rows": (_int, [_vp, _vp, _vp, _vp, _vp]),
    "ggml_backend_b200_buffer_type_name": (ctypes.c_char_p, []),
    "ggml_backend_b200_buffer_type_alignment": (_sz, []),
    "ggml_backend_b200_buffer_type_max_size": (_sz, [_int]),
    "ggml_backend_b200_buffer_type_alloc_size": (_sz, [_TP]),
    "ggml_backend_b200_buffer_type_is_host": (ctypes.c_bool, []),
    "ggml_backend_b200_buffer_alloc": (_vp, [_vp, _sz]),
    "ggml_backend_b200_buffer_free": (None, [_vp]),
    "ggml_backend_b200_buffer_base": (_vp, [_vp]),
    "ggml_backend_b200_buffer_size": (_sz, [_vp]),
    "ggml_backend_b200_buffer_set": (_int, [_vp, _sz, _vp, _sz]),
    "ggml_backend_b200_buffer_get": (_int, [_vp, _sz, _vp, _sz]),
    "ggml_backend_b200_buffer_memset": (_int, [_vp, _sz, _c.c_uint8, _sz]),
    "ggml_backend_b200_buffer_clear": (_int, [_vp, _c.c_uint8]),
    "ggml_backend_b200_buffer_copy": (_int, [_vp, _sz, _vp, _sz, _sz]),
    "ggml_backend_b200_host_alloc": (_vp, [_sz]),
    "ggml_backend_b200_host_free": (None, [_vp]),
    "ggml_backend_b200_set_async": (_int, [_vp, _vp, _sz, _vp, _sz]),
    "ggml_backend_b200_get_async": (_int, [_vp, _vp, _sz, _vp, _sz]),
    "ggml_backend_b200_copy_async": (_int, [_vp, _vp, _sz, _vp, _sz, _sz]),
    "ggml_backend_b200_synchronize": (_int, [_vp]),
    "ggml_backend_b200_event_new": (_vp, [_vp]),
    "ggml_backend_b200_event_free": (None, [_vp]),
    "ggml_backend_b200_event_record": (_int, [_vp, _vp]),
    "ggml_backend_b200_event_wait": (_int, [_vp, _vp]),
    "ggml_backend_b200_event_synchronize": (_int, [_vp]),
    "ggml_backend_b200_device_caps": (None, [_int, _c.POINTER(ctypes.c_bool), _c.POINTER(ctypes.c_bool),
                                             _c.POINTER(ctypes.c_bool), _c.POINTER(ctypes.c_bool)]),
    "b200_flash_attn_workspace_size": (_sz, [_int] * 6),
    "b200_flash_attn_ext": (_int, [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp,
                                   _int, _int, _int, _int, _int, _int, _f, _f, _f, _vp, _sz, _vp, _vp]),
    "b200_mul_mat_id_workspace_size": (_sz, [_i64] * 5),
    "b200_mul_mat_id": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
                               _vp, _i64, _i64, _vp, _sz, _vp, _vp]),
    "b200_mul_mat_vec_workspace_size": (_sz, [_i64, _i64, _i64]),
    "b200_mul_mat_vec": (_int, [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _sz, _vp, _vp]),
    "b200_mul_mat_id_group": (_int, [_int, _int, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64,
                                     _i64, _i64, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "b200_mul_mat_id_route_view": (_int, [_i64, _i64, _i64, _i64, _c.POINTER(_sz), _c.POINTER(_sz),
                                          _c.POINTER(_sz)]),
}
_SIGS.update(_BACKEND_SIGS)
_SIGS.update({
    "b200_moe_ep_dispatch_scratch_size": (_sz, [_i64, _i64, _i64]),
    "b200_moe_ep_dispatch": (_int, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
                                    _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "b200_moe_ep_expert_workspace_size": (_sz, [_i64] * 4),
    "b200_moe_ep_expert": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64,
                                  _vp, _vp, _sz, _vp, _vp]),
    "b200_moe_ep_combine": (_int, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _vp]),
})
_SIGS.update({
    "b200_ep_shared_export": (_int, [_vp, _vp, _c.POINTER(_sz)]),
    "b200_ep_shared_open": (_int, [_vp, _c.POINTER(_vp)]),
    "b200_ep_shared_close": (_int, [_vp]),
    "b200_moe_ep_p2p_push": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _int,
                                    _i64, _vp]),
    "b200_moe_ep_p2p_expert_workspace_size": (_sz, [_i64] * 5),
    "b200_moe_ep_p2p_expert": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _i64,
                                      _i64, _vp, _i64, _i64, _vp, _int, _vp, _sz, _vp, _vp]),
    "b200_moe_ep_p2p_finish": (_int, [_vp, _i64, _int, _vp, _vp]),
    "b200_moe_ep_p2p_expert_group": (_int, [_int, _int, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i64,
                                            _i64, _i64, _vp, _vp, _vp, _vp, _int, _vp, _sz, _vp, _vp]),
    "b200_moe_ep_p2p_ffn_workspace_size": (_sz, [_i64] * 6),
    "b200_mul_mat_id_ffn_workspace_size": (_sz, [_i64] * 5),
    "b200_mul_mat_id_ffn": (_int, [_int, _vp, _vp, _int, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64,
                                   _i64, _i64, _vp, _i64, _i64, _vp, _sz, _vp, _vp]),
    "b200_moe_ep_p2p_expert_ffn": (_int, [_int, _vp, _vp, _int, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _vp, _i64,
                                          _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _int, _vp, _sz, _vp, _vp]),
    "b200_mul_mat_tp_workspace_size": (_sz, [_int, _i64, _i64, _i64]),
    "b200_mul_mat_tp": (_int, [_int, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _int, _vp,
                               _sz, _vp, _vp]),
    "b200_mul_mat_tp_finish": (_int, [_vp, _i64, _int, _vp, _vp]),
    "b200_set_peer_wait_limit_ns": (None, [_c.c_uint64]),
    "b200_peer_wait_limit_ns": (_c.c_uint64, []),
})
_SIGS.update({
    "ggml_backend_b200_builder_new": (_vp, []),
    "ggml_backend_b200_builder_free": (None, [_vp]),
    "ggml_backend_b200_builder_reset": (None, [_vp]),
    "ggml_backend_b200_builder_find": (_TP, [_vp, _vp]),
    "ggml_backend_b200_builder_add": (_TP, [_vp, _vp, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int32,
                                            _c.POINTER(_i64), _c.POINTER(_sz), _c.POINTER(ctypes.c_int32),
                                            _c.POINTER(_vp), _vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_char_p]),
    "ggml_backend_b200_builder_push_node": (_int, [_vp, _vp]),
    "ggml_backend_b200_builder_nodes": (_int, [_vp, _c.POINTER(_c.POINTER(_TP))]),
    "ggml_backend_b200_builder_compute": (_int, [_vp, _vp]),
})
_SIGS.update({
    "b200_mul_mat_noalloc_max_workspace": (_sz, []),
    "b200_mul_mat_noalloc": (_int, [_int, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _vp, _vp]),
    "b200_mul_mat_noalloc_error": (_int, [_vp, _c.POINTER(_int)]),
})


def _elem_size(t):
    be, bb = BLOCK.get(t, (1, 4 if t == I32 else 0))
    return bb / be


def make_tensor(t, ne, data=None, op=OP_NONE, srcs=(), name="", on_device=False, nb=None, readable=True,
                op_params=None):
    """A b200_tensor with ggml semantics: ne[0] innermost; contiguous strides unless nb is given."""
    ne = list(ne) + [1] * (4 - len(ne))
    x = Tensor()
    x.type = t
    x.op = op
    for i in range(4):
        x.ne[i] = int(ne[i])
    if nb is None:
        be, bb = BLOCK.get(t, (1, 4 if t == I32 else 4))
        nb0 = bb if be == 1 else bb
        nb1 = (ne[0] // be) * bb
        nb = [nb0, nb1, nb1 * ne[1], nb1 * ne[1] * ne[2]]
    for i in range(4):
        x.nb[i] = int(nb[i])
    for i, s in enumerate(srcs):
        if s is not None:
            x.src[i] = ctypes.pointer(s)
    if data is not None:
        x.data = data if isinstance(data, int) else data.ctypes.data
    x.on_device = 1 if on_device else 0
    x.readable = 1 if readable else 0
    x.name = name.encode()[:63]
    if op_params:
        for i, v in enumerate(op_params):
            if isinstance(v, float):
                import struct
                v = struct.unpack("<i", struct.pack("<f", v))[0]
            x.op_params[i] = int(v)
    return x


def supports_op(op):
    return bool(lib().ggml_backend_b200_supports_op(ctypes.byref(op)))


def offload_op(op):
    return bool(lib().ggml_backend_b200_offload_op(ctypes.byref(op)))


class Backend:
    """An owning wrapper of a b200_backend_t."""

    def __init__(self):
        self.h = lib().ggml_backend_b200_init()
        if not self.h:
            raise B200Error("ggml_backend_b200_init returned NULL (no CUDA device)")

    def close(self):
        if self.h:
            lib().ggml_backend_b200_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def graph_compute(self, nodes):
        arr = (_TP * len(nodes))(*[ctypes.pointer(n) for n in nodes])
        return lib().ggml_backend_b200_graph_compute(self.h, arr, len(nodes))

    def route_ops(self, route=None):
        return lib().ggml_backend_b200_route_ops(self.h, route.encode() if route else None)

    def cpu_fallbacks(self):
        return lib().ggml_backend_b200_cpu_fallbacks(self.h)

    def device_errors(self):
        return lib().ggml_backend_b200_device_errors(self.h)

    def moe_stats(self):
        a, b = ctypes.c_long(0), ctypes.c_long(0)
        lib().ggml_backend_b200_moe_stats(self.h, ctypes.byref(a), ctypes.byref(b))
        return a.value, b.value

    def weight_cache(self):
        n = ctypes.c_long(0)
        by = lib().ggml_backend_b200_weight_cache_bytes(self.h, ctypes.byref(n))
        return by, n.value


class DeviceBuffer:
    """A b200 device buffer (the backend's buffer type): tensors placed in it are passed with
    on_device = 1 and data = base + offset, and graph_compute uses them in place."""

    def __init__(self, backend, size):
        self.backend = backend
        self.h = lib().ggml_backend_b200_buffer_alloc(backend.h, size)
        if not self.h:
            raise B200Error("ggml_backend_b200_buffer_alloc failed")
        self.size = size
        self.base = lib().ggml_backend_b200_buffer_base(self.h)

    def free(self):
        if self.h:
            lib().ggml_backend_b200_buffer_free(self.h)
            self.h = None

    def set(self, offset, arr):
        import numpy as np
        a = np.ascontiguousarray(arr)
        return lib().ggml_backend_b200_buffer_set(self.h, offset, a.ctypes.data, a.nbytes)

    def get(self, offset, out):
        return lib().ggml_backend_b200_buffer_get(self.h, offset, out.ctypes.data, out.nbytes)

    def tensor(self, offset, ttype, ne, op=OP_NONE, srcs=(), name="", op_params=None):
        """A descriptor of a contiguous tensor at `offset` in this buffer."""
        return make_tensor(ttype, ne, self.base + offset, op=op, srcs=srcs, name=name, on_device=True,
                           op_params=op_params)


class GraphBuilder:
    """The converter a ggml adapter drives (ggml_backend_b200_builder_*): host tensors declared by
    key with ggml's op names, one descriptor per key, nodes pushed in execution order."""

    def __init__(self):
        self.h = lib().ggml_backend_b200_builder_new()

    def close(self):
        if self.h:
            lib().ggml_backend_b200_builder_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def add(self, key, op_name, type_, ne, nb, op_params=None, src_keys=(), data=None, on_device=False,
            readable=True, name="", subop_name=None):
        ne4 = (ctypes.c_int64 * 4)(*(list(ne) + [1] * (4 - len(ne))))
        nb4 = (ctypes.c_size_t * 4)(*nb)
        opp = (ctypes.c_int32 * 16)(*(list(op_params or []) + [0] * (16 - len(op_params or []))))
        srcs = (ctypes.c_void_p * 10)(*(list(src_keys) + [None] * (10 - len(src_keys))))
        r = lib().ggml_backend_b200_builder_add(self.h, key, op_name.encode(),
                                                subop_name.encode() if subop_name else None, type_, ne4, nb4, opp,
                                                srcs, data, 1 if on_device else 0, 1 if readable else 0,
                                                name.encode())
        return r.contents if r else None

    def find(self, key):
        r = lib().ggml_backend_b200_builder_find(self.h, key)
        return r.contents if r else None

    def push(self, key):
        return lib().ggml_backend_b200_builder_push_node(self.h, key)

    def nodes(self):
        arr = ctypes.POINTER(_TP)()
        n = lib().ggml_backend_b200_builder_nodes(self.h, ctypes.byref(arr))
        return [arr[i].contents for i in range(n)]

    def compute(self, backend):
        return lib().ggml_backend_b200_builder_compute(backend.h, self.h)


def weight_key(t):
    buf = ctypes.create_string_buffer(256)
    lib().ggml_backend_b200_weight_key(ctypes.byref(t), buf, 256)
    return buf.value.decode()


def breaker_replay(rcs):
    n = len(rcs)
    a = (ctypes.c_int * n)(*rcs)
    out = (ctypes.c_int * n)()
    lib().ggml_backend_b200_breaker_replay(a, n, out)
    return list(out)


def flash_attn_ext(q, q_nb1, q_nb2, k, k_nb1, k_nb2, v, v_nb1, v_nb2, mask, m_nb1, dst, D, DV, T, H, KV, HK,
                   scale, softcap, workspace, dev_err, max_bias=0.0, stream=None):
    check(lib().b200_flash_attn_ext(_ptr(q), q_nb1, q_nb2, _ptr(k), k_nb1, k_nb2, _ptr(v), v_nb1, v_nb2,
                                    _ptr(mask), m_nb1, _ptr(dst), D, DV, T, H, KV, HK, scale, max_bias, softcap,
                                    _ptr(workspace), workspace.numel() * workspace.element_size(), _ptr(dev_err),
                                    _stream(stream)), "flash_attn_ext")


def flash_attn_workspace_size(D, DV, T, H, KV, HK):
    return lib().b200_flash_attn_workspace_size(D, DV, T, H, KV, HK)


def mul_mat_id_workspace_size(K, N, n_expert, n_used, n_tokens):
    return lib().b200_mul_mat_id_workspace_size(K, N, n_expert, n_used, n_tokens)


def mul_mat_id(wtype, as_packed, K, N, n_expert, b, b_nb1, b_nb2, ne11, ids, ids_nb0, ids_nb1, n_used, n_tokens,
               dst, d_nb1, d_nb2, workspace, dev_err, stream=None):
    return lib().b200_mul_mat_id(wtype, _ptr(as_packed), K, N, n_expert, _ptr(b), b_nb1, b_nb2, ne11, _ptr(ids),
                                 ids_nb0, ids_nb1, n_used, n_tokens, _ptr(dst), d_nb1, d_nb2, _ptr(workspace),
                                 workspace.numel() * workspace.element_size(), _ptr(dev_err), _stream(stream))


def mul_mat_vec(wtype, w_packed, N, K, a, M, out, workspace, dev_err, lda=None, ldd=None, stream=None):
    """Decode-size MUL_MAT (M <= 32; Q4_K, Q6_K, Q8_0): out[M, N] = a[M, K] . W^T (b200_mul_mat_vec)."""
    return lib().b200_mul_mat_vec(wtype, _ptr(w_packed), N, K, _ptr(a), lda if lda else K, M, _ptr(out),
                                  ldd if ldd else N, _ptr(workspace), workspace.numel() * workspace.element_size(),
                                  _ptr(dev_err), _stream(stream))


def mul_mat_id_group(wtype, stacks, Ns, K, n_expert, b, b_nb1, b_nb2, ne11, ids, ids_nb0, ids_nb1, n_used, n_tokens,
                     dsts, d_nb1s, d_nb2s, workspace, dev_err, stream=None):
    """MUL_MAT_IDs over several expert stacks sharing b and ids: one route and gather-pack, one
    grouped GEMM per stack (b200_mul_mat_id_group)."""
    n = len(stacks)
    P = ctypes.c_void_p * n
    I = ctypes.c_int64 * n
    return lib().b200_mul_mat_id_group(n, wtype, P(*[_ptr(t) for t in stacks]), I(*Ns), K, n_expert, _ptr(b), b_nb1,
                                       b_nb2, ne11, _ptr(ids), ids_nb0, ids_nb1, n_used, n_tokens,
                                       P(*[_ptr(t) for t in dsts]), I(*d_nb1s), I(*d_nb2s), _ptr(workspace),
                                       workspace.numel() * workspace.element_size(), _ptr(dev_err), _stream(stream))


def swiglu(a, gt, dst, stream=None):
    """dst = silu(a) * gt over contiguous f32 tensors of one shape (b200_swiglu, ggml's
    SWIGLU with separate gate and up tensors)."""
    n = a.numel()
    inner = a.shape[-1] if a.dim() else 1
    ne = (ctypes.c_int64 * 4)(inner, n // inner, 1, 1)
    nb = (ctypes.c_size_t * 4)(4, inner * 4, n * 4, n * 4)
    return lib().b200_swiglu(_ptr(a), nb, _ptr(gt), nb, ne, _ptr(dst), _stream(stream))


def mul_mat_id_ffn_workspace_size(H, F, n_expert, n_used, n_tokens):
    return lib().b200_mul_mat_id_ffn_workspace_size(H, F, n_expert, n_used, n_tokens)


def mul_mat_id_ffn(wtype_gate_up, gate, up, wtype_down, down, H, F, n_expert, x, x_nb1, x_nb2, ne11, ids, ids_nb0,
                   ids_nb1, n_used, n_tokens, dst, d_nb1, d_nb2, workspace, dev_err, stream=None):
    """A MoE block's expert FFN, down(swiglu(gate(x), up(x))), over one route (b200_mul_mat_id_ffn)."""
    return lib().b200_mul_mat_id_ffn(wtype_gate_up, _ptr(gate), _ptr(up), wtype_down, _ptr(down), H, F, n_expert,
                                     _ptr(x), x_nb1, x_nb2, ne11, _ptr(ids), ids_nb0, ids_nb1, n_used, n_tokens,
                                     _ptr(dst), d_nb1, d_nb2, _ptr(workspace),
                                     workspace.numel() * workspace.element_size(), _ptr(dev_err), _stream(stream))


def mul_mat_id_route_view(K, n_expert, n_used, n_tokens):
    a, b, c = ctypes.c_size_t(0), ctypes.c_size_t(0), ctypes.c_size_t(0)
    check(lib().b200_mul_mat_id_route_view(K, n_expert, n_used, n_tokens, ctypes.byref(a), ctypes.byref(b),
                                           ctypes.byref(c)), "route_view")
    return a.value, b.value, c.value
