"""Vectorised numpy encoders for the ggml block formats (Q8_0, Q4_K, Q6_K).

Used to synthesise quantized weights for the bench and the tests from seeded f32 data.
Q8_0 follows ggml's reference rounding (d = amax/127, q = roundf(x/d)); the Q4_K and Q6_K
encoders are plain min/max and symmetric encoders (any valid block is a valid GEMM input,
since every consumer decodes the same bytes). They produce exactly the bytes of the CPU
oracle's encoders, which the CPU tests check.
"""
import numpy as np


def _roundf(x):
    """C roundf (half away from zero), exact in float32."""
    x = np.asarray(x, dtype=np.float32)
    t = np.trunc(x)
    frac = np.abs(x - t)
    return (t + np.where(frac >= np.float32(0.5), np.sign(x), 0)).astype(np.float32)


def _f16(x):
    return np.asarray(x, dtype=np.float32).astype(np.float16)


def quantize_q8_0(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, K = x.shape
    v = x.reshape(R, K // 32, 32)
    amax = np.abs(v).max(-1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = _roundf(v * idv[..., None]).astype(np.int8)
    out = np.empty((R, K // 32, 34), dtype=np.uint8)
    out[..., 0:2] = _f16(d).view(np.uint8).reshape(R, K // 32, 2)
    out[..., 2:] = q.view(np.uint8)
    return out.reshape(R, -1)


def quantize_q4_k(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, K = x.shape
    nb = K // 256
    v = x.reshape(R, nb, 8, 32)
    lo = np.minimum(v.min(-1), np.float32(0.0))
    hi = np.maximum(v.max(-1), lo)
    scl = ((hi - lo) / np.float32(15.0)).astype(np.float32)
    mns = (-lo).astype(np.float32)
    dh = _f16(scl.max(-1) / np.float32(63.0))
    mh = _f16((mns.max(-1) + np.float32(0.0)) / np.float32(63.0))   # -0.0 -> +0.0, as the C max does
    d = dh.astype(np.float32)[..., None]
    dmin = mh.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d > 0, np.clip(_roundf(scl / np.where(d > 0, d, 1)), 0, 63), 0).astype(np.uint8)
        mq = np.where(dmin > 0, np.clip(_roundf(mns / np.where(dmin > 0, dmin, 1)), 0, 63), 0).astype(np.uint8)
        d1 = (d * sc.astype(np.float32))[..., None]
        m1 = (dmin * mq.astype(np.float32))[..., None]
        q = np.where(d1 > 0, np.clip(_roundf((v + m1) / np.where(d1 > 0, d1, 1)), 0, 15), 0).astype(np.uint8)
    out = np.zeros((R, nb, 144), dtype=np.uint8)
    out[..., 0:2] = dh.view(np.uint8).reshape(R, nb, 2)
    out[..., 2:4] = mh.view(np.uint8).reshape(R, nb, 2)
    s = out[..., 4:16]
    s[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = mq[..., 0:4] | ((mq[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((mq[..., 4:8] & 0x0F) << 4)
    qq = q.reshape(R, nb, 4, 2, 32)
    out[..., 16:] = (qq[..., 0, :] | (qq[..., 1, :] << 4)).reshape(R, nb, 128)
    return out.reshape(R, -1)


def quantize_q6_k(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    R, K = x.shape
    nb = K // 256
    v = x.reshape(R, nb, 16, 16)
    scl = (np.abs(v).max(-1) / np.float32(31.0)).astype(np.float32)
    dh = _f16(scl.max(-1) / np.float32(127.0))
    d = dh.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(d > 0, np.clip(_roundf(scl / np.where(d > 0, d, 1)), -128, 127), 0).astype(np.int8)
        ds = (d * sc.astype(np.float32))[..., None]
        q = (np.clip(np.where(ds != 0, _roundf(v / np.where(ds != 0, ds, 1)), 0), -32, 31) + 32).astype(np.uint8)
    q = q.reshape(R, nb, 2, 4, 32)          # [half][group of 32][l]
    out = np.zeros((R, nb, 210), dtype=np.uint8)
    ql = (q[..., 0:2, :] & 0x0F) | ((q[..., 2:4, :] & 0x0F) << 4)           # [half][2][32]
    out[..., 0:128] = ql.reshape(R, nb, 128)
    qh = (q[..., 0, :] >> 4) | ((q[..., 1, :] >> 4) << 2) | ((q[..., 2, :] >> 4) << 4) | ((q[..., 3, :] >> 4) << 6)
    out[..., 128:192] = qh.reshape(R, nb, 64)
    out[..., 192:208] = sc.view(np.uint8).reshape(R, nb, 16)
    out[..., 208:210] = dh.view(np.uint8).reshape(R, nb, 2)
    return out.reshape(R, -1)


def quantize(t, x):
    if t == 8:
        return quantize_q8_0(x)
    if t == 12:
        return quantize_q4_k(x)
    if t == 14:
        return quantize_q6_k(x)
    if t == 1:
        return np.ascontiguousarray(x, dtype=np.float32).astype(np.float16).view(np.uint8).reshape(x.shape[0], -1)
    raise ValueError(f"no encoder for type {t}")
