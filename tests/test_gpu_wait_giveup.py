"""The give-up path of a cross-GPU wait, on one GPU, without a fault.

The reference turns a failing device route into an error status instead of a hang (its breaker and
fault policy, ggml-rocket.cpp:263-307). Here every kernel that waits for another GPU's flag is
bounded: after b200_peer_wait_limit_ns of %globaltimer it records B200_DEV_WAIT_PEER in the caller's
error word and returns. This test makes such a wait run out on purpose -- a flag array that no rank
will ever publish to, with the limit lowered to a few milliseconds -- for the N-sharded MUL_MAT's
finish and the expert-parallel finish, then checks the error word, that the wait ended within a
bound, that the Python wrapper of the N-sharded op raises, and that the context still computes a
MUL_MAT correctly afterwards.
"""
import time

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu

LIMIT_NS = 5_000_000   # 5 ms


@pytest.fixture
def short_limit(cuda):
    import ggml_b200 as g
    L = g.lib()
    old = L.b200_peer_wait_limit_ns()
    L.b200_set_peer_wait_limit_ns(LIMIT_NS)
    assert L.b200_peer_wait_limit_ns() == LIMIT_NS
    yield L
    L.b200_set_peer_wait_limit_ns(0)            # back to the default
    assert L.b200_peer_wait_limit_ns() == old


@pytest.mark.parametrize("entry", ["b200_mul_mat_tp_finish", "b200_moe_ep_p2p_finish"])
def test_peer_wait_gives_up(short_limit, entry):
    import torch
    import ggml_b200 as g
    L = short_limit
    G = 2
    flags = torch.zeros((2 * G, 4), dtype=torch.int32, device="cuda")   # nobody will publish epoch 3
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = getattr(L, entry)(g._ptr(flags), G, 3, g._ptr(err), g._stream(stream))
    assert rc == 0                                # the launch itself is fine; the wait fails on the GPU
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert int(err.item()) == 7                   # B200_DEV_WAIT_PEER
    assert waited < 1.0                           # ended by the 5 ms limit, not the 2 s default
    # the context is still usable: a MUL_MAT right after computes the right thing
    rng = np.random.default_rng(5)
    N, K, M = 256, 512, 64
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    a = rng.standard_normal((M, K)).astype(np.float32)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ws = torch.empty(max(256, g.mul_mat_workspace_size(M, N, K, g.F16)), dtype=torch.uint8, device="cuda")
    err2 = torch.zeros(1, dtype=torch.int32, device="cuda")
    g.mul_mat(g.F16, torch.from_numpy(w.view(np.uint8).reshape(-1)).cuda(), N, K, torch.from_numpy(a).cuda(), M,
              out, ws, err2)
    torch.cuda.synchronize()
    assert int(err2.item()) == 0
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    assert rel_err(out.cpu().numpy(), ref) <= 1e-2


def test_sharded_mul_mat_wrapper_raises(short_limit):
    """ggml_b200.tp's one-rank op whose finish waits on a second, absent rank: the wait gives up and
    the wrapper's error check turns the device word into an exception."""
    import torch
    import ggml_b200 as g
    L = short_limit
    flags = torch.zeros((2, 4), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # rank 0 of 2 signals itself only; slot 1 stays empty
    assert L.b200_mul_mat_tp_finish(g._ptr(flags), 2, 9, g._ptr(err), None) == 0
    torch.cuda.synchronize()
    with pytest.raises(g.B200Error):
        g.check_device(err, "mul_mat_tp_finish")
