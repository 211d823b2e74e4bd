"""kvf_calibrate_noalloc: the calibration entry point for callers that cannot
allocate device memory (for example a serving engine that reserves all device
memory up front, or a path that cannot afford cudaMalloc's implicit device
synchronisation). Its scratch is a fixed file-scope device array, so it must
give exactly what the allocating kvf_calibrate gives, call after call, even
though every call reuses (and leaves behind) the same scratch contents.

This file is collected last on purpose: a failure here leaves every other test
already run."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _calibrate(lib, ctx, fn, x, H, T, D, stream):
    out = torch.full((H,), float("nan"), dtype=torch.float32, device="cuda")
    status = getattr(lib, fn)(ctx, _ptr(x), 1, H, T, D, 64, _ptr(out), stream)
    return status, out


def test_calibrate_noalloc_matches_allocating_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kvforge_b200 import _lib as L
    lib, ctx = L.lib(), L.context(0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(77)
    H, T, D = 8, 4096, 128
    x = (rng.standard_normal((H, T, D)) * np.linspace(0.5, 2.0, H)[:, None, None]).astype(np.float16)
    xt = torch.from_numpy(x).cuda()

    st, ref = _calibrate(lib, ctx, "kvf_calibrate", xt, H, T, D, stream)
    L.check(st)
    for _ in range(2):  # two calls in a row share the same scratch
        st, got = _calibrate(lib, ctx, "kvf_calibrate_noalloc", xt, H, T, D, stream)
        L.check(st)
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=1e-6, atol=1e-7)

    # a smaller call after a larger one: stale scratch from the previous call is never read
    xs = xt[:3, :100].contiguous()
    st, ref_s = _calibrate(lib, ctx, "kvf_calibrate", xs, 3, 100, D, stream)
    L.check(st)
    st, got_s = _calibrate(lib, ctx, "kvf_calibrate_noalloc", xs, 3, 100, D, stream)
    L.check(st)
    torch.cuda.synchronize()
    assert np.allclose(got_s.cpu().numpy(), ref_s.cpu().numpy(), rtol=1e-6, atol=1e-7)


def test_calibrate_noalloc_many_heads():
    """6000 heads: the finishing step keeps each head's variance in the
    static scratch itself, so the head count is bounded only by the slots."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kvforge_b200 import _lib as L
    lib, ctx = L.lib(), L.context(0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    rng = np.random.default_rng(78)
    H, T, D = 6000, 64, 8
    x = (rng.standard_normal((H, T, D)) * np.linspace(0.5, 2.0, H)[:, None, None]).astype(np.float16)
    xt = torch.from_numpy(x).cuda()
    st, ref = _calibrate(lib, ctx, "kvf_calibrate", xt, H, T, D, stream)
    L.check(st)
    for _ in range(2):
        st, got = _calibrate(lib, ctx, "kvf_calibrate_noalloc", xt, H, T, D, stream)
        L.check(st)
        torch.cuda.synchronize()
        assert np.allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=1e-6, atol=1e-7)


def test_calibrate_noalloc_rejects_sizes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kvforge_b200 import _lib as L
    lib, ctx = L.lib(), L.context(0)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    xt = torch.zeros((1, 64, 128), dtype=torch.float16, device="cuda")
    out = torch.zeros(16, dtype=torch.float32, device="cuda")
    # 16 heads x ceil(2^22 * 128 / 65536) = 16 x 8192 slots > 65536: rejected before any launch
    status = lib.kvf_calibrate_noalloc(ctx, _ptr(xt), 1, 16, 1 << 22, 128, 64, _ptr(out), stream)
    assert status == L.ERR_INVALID_CONFIG
    assert b"static scratch" in lib.kvf_last_error()
