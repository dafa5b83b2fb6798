"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed)."""
import ctypes
import os
import re

import ggml_b200 as g

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    names = set()
    for h in ("ggml-b200.h", "ggml-b200-kernels.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b((?:ggml_backend|b200)_\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(g.LIB_PATH)
    names = declared()
    assert len(names) >= 35
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_declares_every_symbol():
    assert declared() <= set(g._SIGS)


def test_library_answers_without_a_gpu():
    lib = g.lib()
    assert lib.ggml_backend_b200_reg_name() == b"B200"
    assert lib.ggml_backend_b200_op_from_name(b"MUL_MAT") == g.OP_MUL_MAT
    assert lib.ggml_backend_b200_op_from_name(b"FLASH_ATTN_EXT") == g.OP_FLASH_ATTN_EXT
    assert lib.ggml_backend_b200_op_from_name(b"ADD") == g.OP_ADD
    assert lib.ggml_backend_b200_op_from_name(b"CONV_2D") == g.OP_OTHER
    assert lib.ggml_backend_b200_subop_from_name(b"SILU") == g.UNARY_SILU
    assert lib.ggml_backend_b200_subop_from_name(b"SWIGLU") == g.GLU_SWIGLU
    assert lib.ggml_backend_b200_subop_from_name(b"GELU") == -1
    assert g.weight_packed_size(g.Q4_K, 4096, 4096) == 4096 * 16 * 144
    assert g.weight_packed_size(g.Q4_K, 4096, 4000) == 0       # K % 256 != 0


def test_multi_gpu_and_group_entry_points_reject_bad_arguments_without_a_gpu():
    """The N-sharded, grouped MUL_MAT_ID and grouped expert-parallel entry points check their
    arguments before any CUDA call, so malformed calls fail with a status even on a host with
    no GPU."""
    lib = g.lib()
    p = ctypes.c_void_p(16)
    # b200_mul_mat_tp: null weight, rank out of range, column offset not a multiple of 16
    assert lib.b200_mul_mat_tp(12, None, 16, 0, 256, p, 256, 4, p, 64, 1, 0, p, 1, p, 0, p, None) == \
        g.B200_E_INVALID
    assert lib.b200_mul_mat_tp(12, p, 16, 0, 256, p, 256, 4, p, 64, 2, 2, p, 1, p, 0, p, None) == g.B200_E_INVALID
    assert lib.b200_mul_mat_tp(12, p, 16, 8, 256, p, 256, 4, p, 64, 1, 0, p, 1, p, 0, p, None) == \
        g.B200_E_UNSUPPORTED
    assert lib.b200_mul_mat_tp_finish(None, 1, 1, p, None) == g.B200_E_INVALID
    assert lib.b200_mul_mat_tp_finish(p, 65, 1, p, None) == g.B200_E_UNSUPPORTED
    assert lib.b200_mul_mat_tp_workspace_size(12, 0, 16, 256) == 0
    # b200_mul_mat_id_group: no members, too many members
    assert lib.b200_mul_mat_id_group(0, 12, p, p, 256, 8, p, 1024, 1024, 1, p, 4, 16, 4, 8, p, p, p, p, 0, p,
                                     None) == g.B200_E_INVALID
    assert lib.b200_mul_mat_id_group(17, 12, p, p, 256, 8, p, 1024, 1024, 1, p, 4, 16, 4, 8, p, p, p, p, 0, p,
                                     None) == g.B200_E_UNSUPPORTED
    # b200_moe_ep_p2p_expert_group: no members
    assert lib.b200_moe_ep_p2p_expert_group(0, 12, p, p, 256, 4, 0, p, p, p, 2, 0, 4, 64, 0, p, p, p, p, 1, p, 0, p,
                                            None) == g.B200_E_INVALID


def test_buffer_type_and_handles_without_a_gpu():
    """The device buffer type answers its static queries anywhere; buffer, event and async calls
    on null or foreign handles fail with a status instead of touching memory."""
    lib = g.lib()
    assert lib.ggml_backend_b200_buffer_type_name() == b"B200"
    assert lib.ggml_backend_b200_buffer_type_alignment() == 256
    assert not lib.ggml_backend_b200_buffer_type_is_host()
    t = g.make_tensor(g.F32, [64, 3])
    assert lib.ggml_backend_b200_buffer_type_alloc_size(ctypes.byref(t)) == 64 * 3 * 4
    q = g.make_tensor(g.Q4_K, [512, 2])
    assert lib.ggml_backend_b200_buffer_type_alloc_size(ctypes.byref(q)) == 2 * 2 * 144
    assert not lib.ggml_backend_b200_buffer_alloc(None, 1024)
    assert lib.ggml_backend_b200_buffer_size(None) == 0 and not lib.ggml_backend_b200_buffer_base(None)
    buf = ctypes.create_string_buffer(64)
    assert lib.ggml_backend_b200_buffer_set(None, 0, buf, 16) == g.STATUS_FAILED
    assert lib.ggml_backend_b200_buffer_get(None, 0, buf, 16) == g.STATUS_FAILED
    assert lib.ggml_backend_b200_buffer_memset(None, 0, 0, 16) == g.STATUS_FAILED
    assert lib.ggml_backend_b200_buffer_copy(None, 0, None, 0, 16) == g.STATUS_FAILED
    assert lib.ggml_backend_b200_set_async(None, None, 0, buf, 16) == g.STATUS_FAILED
    assert lib.ggml_backend_b200_synchronize(None) == g.STATUS_FAILED
    assert not lib.ggml_backend_b200_event_new(None)
    assert lib.ggml_backend_b200_event_synchronize(None) == g.STATUS_FAILED
    lib.ggml_backend_b200_buffer_free(None)
    lib.ggml_backend_b200_event_free(None)
    flags = [ctypes.c_bool(True) for _ in range(4)]
    lib.ggml_backend_b200_device_caps(-1, *[ctypes.byref(f) for f in flags])
    assert not any(f.value for f in flags)
