"""The device buffer type, async transfers and events on the GPU.

The reference hands out the host CPU buffer type and reports no async or event support
(ggml-rocket.cpp:7310-7328); a ggml device with its own memory offers them, and these tests drive
them as a ggml host would: tensors allocated in b200 buffers (on_device = 1) computed in place by
graph_compute, async set/get through pinned host memory ordered by events, and the weight cache
dropping packed copies whose device bytes were rewritten or freed."""
import ctypes

import numpy as np
import pytest

import ggml_b200 as g
import oracle
from conftest import rel_err
from ggml_b200 import quants

pytestmark = pytest.mark.gpu


def test_buffer_round_trip_memset_copy_and_bounds(cuda):
    lib = g.lib()
    be = g.Backend()
    a = g.DeviceBuffer(be, 1 << 20)
    b = g.DeviceBuffer(be, 1 << 20)
    assert a.base % lib.ggml_backend_b200_buffer_type_alignment() == 0
    assert lib.ggml_backend_b200_buffer_size(a.h) == 1 << 20
    x = np.arange(4096, dtype=np.float32)
    assert a.set(1024, x) == g.STATUS_SUCCESS
    y = np.zeros_like(x)
    assert a.get(1024, y) == g.STATUS_SUCCESS and np.array_equal(x, y)
    assert lib.ggml_backend_b200_buffer_copy(a.h, 1024, b.h, 0, x.nbytes) == g.STATUS_SUCCESS
    z = np.zeros_like(x)
    assert b.get(0, z) == g.STATUS_SUCCESS and np.array_equal(x, z)
    assert lib.ggml_backend_b200_buffer_memset(b.h, 16, 0, 32) == g.STATUS_SUCCESS
    assert b.get(0, z) == g.STATUS_SUCCESS
    assert np.array_equal(z[4:12], np.zeros(8, np.float32)) and np.array_equal(z[12:], x[12:])
    assert lib.ggml_backend_b200_buffer_clear(b.h, 0xFF) == g.STATUS_SUCCESS
    w = np.zeros(16, np.uint8)
    assert b.get((1 << 20) - 16, w) == g.STATUS_SUCCESS and np.all(w == 0xFF)
    # ranges past the end fail and leave the buffer alone
    assert a.set((1 << 20) - 8, x[:4]) == g.STATUS_FAILED
    assert a.get(1 << 20, np.zeros(1, np.uint8)) == g.STATUS_FAILED
    assert lib.ggml_backend_b200_buffer_copy(a.h, 0, b.h, (1 << 20) - 4, 8) == g.STATUS_FAILED
    a.free()
    b.free()
    be.close()


def test_async_transfers_events_and_pinned_memory(cuda):
    lib = g.lib()
    be = g.Backend()
    n = 1 << 22
    buf = g.DeviceBuffer(be, 2 * n)
    host_in = lib.ggml_backend_b200_host_alloc(n)
    host_out = lib.ggml_backend_b200_host_alloc(n)
    assert host_in and host_out
    src = np.frombuffer((ctypes.c_uint8 * n).from_address(host_in), dtype=np.uint8)
    dst = np.frombuffer((ctypes.c_uint8 * n).from_address(host_out), dtype=np.uint8)
    src[:] = np.random.default_rng(3).integers(0, 256, n, dtype=np.uint8)
    dst[:] = 0
    ev = lib.ggml_backend_b200_event_new(be.h)
    assert ev
    assert lib.ggml_backend_b200_set_async(be.h, buf.h, 0, host_in, n) == g.STATUS_SUCCESS
    assert lib.ggml_backend_b200_copy_async(be.h, buf.h, 0, buf.h, n, n) == g.STATUS_SUCCESS
    assert lib.ggml_backend_b200_event_record(be.h, ev) == g.STATUS_SUCCESS
    assert lib.ggml_backend_b200_event_wait(be.h, ev) == g.STATUS_SUCCESS
    assert lib.ggml_backend_b200_get_async(be.h, buf.h, n, host_out, n) == g.STATUS_SUCCESS
    assert lib.ggml_backend_b200_synchronize(be.h) == g.STATUS_SUCCESS
    assert lib.ggml_backend_b200_event_synchronize(ev) == g.STATUS_SUCCESS
    assert np.array_equal(src, dst)
    # a buffer of another backend is refused by this one's async calls
    other = g.Backend()
    assert lib.ggml_backend_b200_set_async(other.h, buf.h, 0, host_in, 16) == g.STATUS_FAILED
    caps = [ctypes.c_bool(False) for _ in range(4)]
    lib.ggml_backend_b200_device_caps(0, *[ctypes.byref(c) for c in caps])
    assert all(c.value for c in caps)
    lib.ggml_backend_b200_event_free(ev)
    lib.ggml_backend_b200_host_free(host_in)
    lib.ggml_backend_b200_host_free(host_out)
    buf.free()
    other.close()
    be.close()


def test_graph_compute_on_device_buffers_and_cache_invalidation(cuda):
    """Weights, activations and the output all live in a b200 buffer: graph_compute reads and
    writes them in place. Rewriting the weight's bytes through the buffer API drops the packed
    copy, so the next graph uses the new weight; freeing the buffer drops it too."""
    lib = g.lib()
    be = g.Backend()
    rng = np.random.default_rng(5)
    K, N, M = 1024, 512, 96
    raw1 = quants.quantize(g.Q4_K, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    raw2 = quants.quantize(g.Q4_K, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    a = rng.standard_normal((M, K)).astype(np.float32)
    w_off, x_off, y_off = 0, 1 << 20, 2 << 20
    buf = g.DeviceBuffer(be, 3 << 20)
    assert raw1.nbytes <= x_off and a.nbytes <= y_off - x_off
    assert buf.set(w_off, raw1) == g.STATUS_SUCCESS and buf.set(x_off, a) == g.STATUS_SUCCESS
    w = buf.tensor(w_off, g.Q4_K, [K, N], name="blk.0.ffn_up.weight")
    x = buf.tensor(x_off, g.F32, [K, M], name="x")
    y = buf.tensor(y_off, g.F32, [N, M], op=g.OP_MUL_MAT, srcs=[w, x], name="y")
    assert g.supports_op(y)
    out = np.zeros((M, N), np.float32)

    def run():
        assert be.graph_compute([y]) == g.STATUS_SUCCESS
        assert buf.get(y_off, out) == g.STATUS_SUCCESS
        return out.copy()

    assert rel_err(run(), oracle.mul_mat(g.Q4_K, raw1, N, K, a)) <= 1e-2
    assert be.weight_cache()[1] == 1
    assert rel_err(run(), oracle.mul_mat(g.Q4_K, raw1, N, K, a)) <= 1e-2   # served from the cache
    assert be.weight_cache()[1] == 1
    assert buf.set(w_off, raw2) == g.STATUS_SUCCESS                        # new bytes, same place
    assert be.weight_cache()[1] == 0
    assert rel_err(run(), oracle.mul_mat(g.Q4_K, raw2, N, K, a)) <= 1e-2
    assert be.weight_cache()[1] == 1
    assert be.cpu_fallbacks() == 0 and be.device_errors() == 0
    buf.free()
    assert be.weight_cache()[1] == 0
    be.close()
