"""The MUL_MAT entry point that allocates nothing (b200_mul_mat_noalloc), on the GPU.

Callers that cannot call cudaMalloc -- a plugin inside a process whose allocator owns the
device, code that must not change the device memory map, a fixed memory budget -- get the same
MUL_MAT with its workspace in a fixed device array inside the library. This test calls it through
the C ABI twice in a row (the array keeps the previous call's contents, so the second call shows
nothing leaks between calls) and checks each result against b200_mul_mat, the entry point that
takes a caller-allocated workspace, within the MUL_MAT tolerance the other tests use. It also
checks the clear error for an op too large for the array and the internal error word.

The file is named to be collected last, so a run that stops at the first failure has already
run every other test; it passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _run_both(torch, g, wtype, N, K, M, seed):
    from ggml_b200 import quants
    rng = np.random.default_rng(seed)
    raw = quants.quantize(wtype, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    packed = torch.empty(g.weight_packed_size(wtype, N, K), dtype=torch.uint8, device="cuda")
    g.weight_pack(wtype, torch.from_numpy(raw.reshape(-1)).cuda(), N, K, packed)
    # the existing entry point, with a caller-allocated workspace
    ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ws = torch.empty(g.mul_mat_workspace_size(M, N, K, wtype), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    g.mul_mat(wtype, packed, N, K, a, M, ref, ws, err)
    # the no-alloc entry point: inputs and outputs only, the error word kept internally
    out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = g.lib().b200_mul_mat_noalloc(wtype, ctypes.c_void_p(packed.data_ptr()), N, K,
                                      ctypes.c_void_p(a.data_ptr()), K, M, ctypes.c_void_p(out.data_ptr()), N,
                                      None, stream)
    assert rc == 0
    host_err = ctypes.c_int(-1)
    assert g.lib().b200_mul_mat_noalloc_error(stream, ctypes.byref(host_err)) == 0
    torch.cuda.synchronize()
    assert host_err.value == 0 and int(err.item()) == 0
    return out.cpu().numpy(), ref.cpu().numpy()


def test_noalloc_matches_mul_mat_twice(cuda):
    import torch
    import ggml_b200 as g
    # calls in a row with different shapes and formats; the first and the last share output tiles
    # between CTAs under stream-K (partials and their flags, the part of the array that carries
    # state from one call to the next), so the last call runs on flags the first one left behind
    cases = ((g.Q4_K, 14336, 4096, 512, 1), (g.F16, 768, 2048, 96, 2), (g.Q4_K, 14336, 4096, 512, 3))
    plan = g.mul_mat_plan(512, 14336, 4096, g.Q4_K)
    tiles = (14336 // 128) * (512 // plan["token_tile"])
    # shared tiles, and more tiles than half the grid, so not the cluster split (which keeps no flags)
    assert plan["splits"] > 1 and 2 * tiles > plan["grid"]
    for wtype, N, K, M, seed in cases:
        got, want = _run_both(torch, g, wtype, N, K, M, seed)
        assert np.all(np.isfinite(got))
        assert rel_err(got, want) <= TOL


def test_noalloc_rejects_oversized_ops(cuda):
    import torch
    import ggml_b200 as g
    cap = g.lib().b200_mul_mat_noalloc_max_workspace()
    M, N, K = 8192, 4096, 14336                  # 8192 x 14336 fp16 activations alone exceed the array
    assert g.mul_mat_workspace_size(M, N, K, g.Q4_K) > cap
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = ctypes.c_void_p(dummy.data_ptr())
    rc = g.lib().b200_mul_mat_noalloc(g.Q4_K, p, N, K, p, K, M, p, N, None, stream)
    assert rc == g.B200_E_TOO_LARGE
