"""Vectorised numpy restatement of the KIVI quantizer
(crates/kvforge-cpu/src/quantize.rs:47-231).

TEST INFRASTRUCTURE ONLY: a second, independent check of the C oracle's
quantize / dequantize arithmetic (it shares no code with it).
"""
import numpy as np

INT4, INT8 = 0, 1
PER_CHANNEL, PER_TOKEN = 0, 1


def _levels(dt):
    return np.float32(15.0 if dt == INT4 else 255.0)  # quantize.rs:28-34


def _canon(a):
    a = a.copy()
    a[a == 0] = np.float32(0.0)
    return a


def _minmax(x, axis):
    xc = _canon(x)
    with np.errstate(invalid="ignore"):
        mn = np.nanmin(np.where(np.isnan(xc), np.inf, xc), axis=axis)
        mx = np.nanmax(np.where(np.isnan(xc), -np.inf, xc), axis=axis)
    return mn.astype(np.float32), mx.astype(np.float32)


def quantize(x, dt, axis):
    x = np.asarray(x, np.float32)
    H, T, D = x.shape
    lv = _levels(dt)
    red = 1 if axis == PER_CHANNEL else 2  # quantize.rs:79-98 (over t) / 112-127 (over c)
    mn, mx = _minmax(x, red)
    rng = (mx - mn).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        scale = np.where(rng < np.float32(1e-10), np.float32(1.0), (rng / lv).astype(np.float32)).astype(np.float32)
        mn_b = np.expand_dims(mn, red)
        sc_b = np.expand_dims(scale, red)
        y = ((x - mn_b).astype(np.float32) / sc_b).astype(np.float32)
        # round half away from zero (Rust f32::round)
        # floor(|y| + 0.5) taken in f64, where adding 0.5 to an f32 value is exact
        y64 = y.astype(np.float64)
        r = (np.sign(y64) * np.floor(np.abs(y64) + 0.5)).astype(np.float32)
        r = np.where(np.isnan(r), np.float32(0), np.clip(r, np.float32(0), lv))
    q = r.astype(np.uint8).reshape(-1)
    if dt == INT4:  # quantize.rs:136-150
        if q.size % 2:
            q = np.concatenate([q, np.zeros(1, np.uint8)])
        packed = (q[0::2] & 0x0F) | ((q[1::2] & 0x0F) << 4)
    else:
        packed = q
    return packed.astype(np.uint8), scale.reshape(-1), mn.reshape(-1)


def dequantize(packed, scales, mins, dt, axis, shape):
    H, T, D = shape
    n = H * T * D
    packed = np.asarray(packed, np.uint8)
    if dt == INT4:
        q = np.empty(packed.size * 2, np.uint8)
        q[0::2] = packed & 0x0F
        q[1::2] = (packed >> 4) & 0x0F
        q = q[:n]
    else:
        q = packed
    q = q.reshape(H, T, D).astype(np.float32)
    if axis == PER_CHANNEL:
        sc = scales.reshape(H, 1, D)
        mn = mins.reshape(H, 1, D)
    else:
        sc = scales.reshape(H, T, 1)
        mn = mins.reshape(H, T, 1)
    return ((q * sc).astype(np.float32) + mn).astype(np.float32)
