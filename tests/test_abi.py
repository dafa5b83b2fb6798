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
    assert lib.ggml_backend_b200_op_from_name(b"ADD") == g.OP_OTHER
    assert g.weight_packed_size(g.Q4_K, 4096, 4096) == 4096 * 16 * 144
    assert g.weight_packed_size(g.Q4_K, 4096, 4000) == 0       # K % 256 != 0
