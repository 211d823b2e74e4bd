"""GPU parity tests: every call goes through libkvforge_b200's C ABI and is
checked against the CPU oracle on the same seeded inputs.

Bars: quantized codes, scales, mins, dequantized values, projected
coefficients, rANS containers and compression ratios are bit-exact; the
default reconstruction (fused multiply-add on CUDA cores, or the tcgen05
split-tf32 GEMM engine for head_dim 128 and rank <= 16) is within relative
Frobenius error REC_TOL = 1e-5 of the reference's loop, ten times inside the
1e-4 that the f32 projection/reconstruction contract allows, and bit-exact in
the exact-reconstruction mode; calibration scores within 1e-6 relative."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

INT4, INT8 = 0, 1
PC, PT = 0, 1
# relative Frobenius error of the default (tensor-core / fused) reconstruction
REC_TOL = 1e-5


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    """f32 bit patterns with every NaN mapped to one value: IEEE 754 leaves NaN
    payloads unspecified (x86 yields 0xFFC00000 for 0 * inf, the GPU 0x7FFFFFFF),
    so NaN positions must match but their payloads are not compared."""
    a = np.ascontiguousarray(a, np.float32)
    b = a.view(np.uint32).copy()
    b[np.isnan(a)] = 0x7FC00000
    return b


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _x(shape, seed, f16=False, scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    if f16:
        x16 = x.astype(np.float16)
        return x16, x16.astype(np.float32)
    return x, x


# ---- quantization ---------------------------------------------------------------
# (even widths that are not multiples of four take the paired per-token kernel)
QSHAPES = [(4, 64, 32), (3, 17, 9), (1, 1, 1), (2, 128, 5), (2, 300, 128), (8, 1000, 128), (5, 7, 256),
           (3, 101, 58), (2, 33, 6), (1, 7, 2), (4, 50, 126),
           (2, 9, 13), (1, 3000, 24), (3, 65, 100)]


@pytest.mark.parametrize("shape", QSHAPES)
@pytest.mark.parametrize("dt", [INT4, INT8])
@pytest.mark.parametrize("ax", [PC, PT])
@pytest.mark.parametrize("f16", [False, True])
def test_quantize_parity(kvf, oracle, shape, dt, ax, f16):
    xin, x32 = _x(shape, hash((shape, dt, ax, f16)) % 2**31, f16, scale=3.0)
    q = kvf.GpuQuantizer()
    packed, params = q.quantize(dev(xin), dt, ax)
    p, s, m = oracle.quantize(x32, dt, ax)
    assert np.array_equal(host(packed), p)
    assert np.array_equal(bits(host(params.scales)), bits(s))
    assert np.array_equal(bits(host(params.mins)), bits(m))
    d = q.dequantize(packed, params)
    assert np.array_equal(bits(host(d)), bits(oracle.dequantize(p, s, m, dt, ax, shape)))


def test_quantize_golden(kvf, golden):
    q = kvf.GpuQuantizer()
    keys = sorted(k[:-2] for k in golden.files if k.startswith("q") and k.endswith("_x"))
    for key in keys:
        _, dt, ax = map(int, key[1:].split("_"))
        x = golden[key + "_x"]
        packed, params = q.quantize(dev(x), dt, ax)
        assert np.array_equal(host(packed), golden[key + "_packed"]), key
        assert np.array_equal(bits(host(params.scales)), bits(golden[key + "_scales"])), key
        assert np.array_equal(bits(host(params.mins)), bits(golden[key + "_mins"])), key
        d = q.dequantize(packed, params)
        assert np.array_equal(bits(host(d)), bits(golden[key + "_deq"])), key


@pytest.mark.parametrize("dt", [INT4, INT8])
def test_quantize_half_integer_quotients(kvf, oracle, dt):
    """Values whose (v - min) / scale falls within a few ulps of k + 0.5: the
    GPU divides by multiplying with the reciprocal and must fall back to the
    exact IEEE quotient exactly where rounding could differ."""
    rng = np.random.default_rng(99)
    levels = 15 if dt == INT4 else 255
    H, T, D = 4, 512, 64
    x = np.zeros((H, T, D), np.float32)
    for h in range(H):
        for t in range(T):
            M = np.float32(rng.uniform(0.01, 100.0))
            s = np.float32(M / np.float32(levels))
            k = rng.integers(0, levels, D - 2)
            base = ((k + 0.5) * s.astype(np.float64)).astype(np.float32)
            ulp = rng.integers(-3, 4, D - 2).astype(np.int32)
            vals = (base.view(np.int32) + ulp).view(np.float32)
            x[h, t, 0], x[h, t, 1] = 0.0, M
            x[h, t, 2:] = np.clip(vals, 0, M)
    q = kvf.GpuQuantizer()
    for ax in (PC, PT):
        packed, params = q.quantize(dev(x), dt, ax)
        p, s_, m = oracle.quantize(x, dt, ax)
        assert np.array_equal(host(packed), p)
        assert np.array_equal(bits(host(params.scales)), bits(s_))


def test_quantize_errors(kvf):
    q = kvf.GpuQuantizer()
    x = dev(np.zeros((2, 4, 4), np.float32))
    with pytest.raises(kvf.KvForgeError) as e:
        q.quantize(x, 2, PC)
    assert e.value.status == 3
    packed, params = q.quantize(x, INT8, PT)
    with pytest.raises(kvf.KvForgeError) as e:
        q.dequantize(packed[:-1], params)
    assert e.value.status == 3


# ---- calibration -----------------------------------------------------------------
@pytest.mark.parametrize("shape,f16", [((2, 128, 16), False), ((8, 4096, 128), True), ((3, 70, 7), False)])
def test_calibrate_parity(kvf, oracle, shape, f16):
    xin, x32 = _x(shape, 11, f16)
    x32 = x32 * np.linspace(0.1, 3.0, shape[0], dtype=np.float32)[:, None, None]
    xin = x32.astype(xin.dtype)
    s = host(kvf.GpuSensitivityCalibrator().calibrate(dev(xin)))
    so = oracle.calibrate(xin.astype(np.float32))
    assert np.allclose(s, so, rtol=1e-6, atol=1e-7)
    with pytest.raises(kvf.KvForgeError) as e:
        kvf.GpuSensitivityCalibrator().calibrate(dev(xin[:, :32]))
    assert e.value.status == 2


def test_calibrate_many_heads(kvf, oracle):
    """More heads than one block's shared memory could hold as doubles
    (6000 x 8 B > 40 KB): the per-head variances live in the partial slots."""
    xin, x32 = _x((6000, 64, 8), 12, True)
    x32 = x32 * np.linspace(0.1, 3.0, 6000, dtype=np.float32)[:, None, None]
    xin = x32.astype(np.float16)
    s = host(kvf.GpuSensitivityCalibrator().calibrate(dev(xin)))
    so = oracle.calibrate(xin.astype(np.float32))
    assert np.allclose(s, so, rtol=1e-6, atol=1e-7)


# ---- projection ------------------------------------------------------------------
def _basis(oracle, x32, thr, max_rank=None):
    bf, sv = oracle.compute_basis(x32, threads=4)
    return oracle.select_basis(bf, sv, x32.shape[1], thr, max_rank)


@pytest.mark.parametrize("shape,thr,f16", [((2, 300, 16), 0.9, False), ((4, 1000, 128), 0.75, True),
                                           ((3, 257, 128), 0.999, False), ((2, 100, 13), 0.9, True),
                                           ((1, 5000, 64), 0.5, False), ((2, 600, 128), 0.9999, True)])
def test_project_parity(kvf, oracle, shape, thr, f16):
    xin, x32 = _x(shape, 21, f16)
    bvt, ranks, R = _basis(oracle, x32, thr)
    basis = kvf.Basis.from_host(bvt, ranks)
    P = host(kvf.GpuProjector().project(dev(xin), basis))
    Po = oracle.project(x32, bvt, ranks, threads=4)
    assert np.array_equal(bits(P), bits(Po))


@pytest.mark.parametrize("R", [25, 32, 40, 58, 64])
@pytest.mark.parametrize("f16", [False, True])
def test_project_parity_several_passes(kvf, oracle, R, f16):
    """24 < R <= 64: the tensor-copy projection makes one pass per 32
    coefficients over every tile; ranks below R, and rank 1, included."""
    shape = (3, 700, 128)
    xin, x32 = _x(shape, 100 + R, f16)
    rng = np.random.default_rng(R)
    bvt = (rng.standard_normal((3, R, 128)) / np.sqrt(128)).astype(np.float32)
    ranks = np.array([R, max(1, R - 7), 1], np.uint64)
    basis = kvf.Basis.from_host(bvt, ranks)
    P = host(kvf.GpuProjector().project(dev(xin), basis))
    Po = oracle.project(x32, bvt, ranks, threads=4)
    assert np.array_equal(bits(P), bits(Po))


def test_pipeline_parity_high_rank(kvf, oracle):
    """A layer whose ranks exceed 32 (per-channel keys with calibration and
    per-token values, two projection passes per tile, tensor-core
    reconstruction by default): codes, bitstreams and ratio bit-exact,
    reconstruction within REC_TOL, and bit-exact in the exact mode."""
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    # a 0.2 noise floor over 128 channels spreads 75 % of the variance over about 46 directions
    k, v = synth.numpy_layer(2, 640, 128, seed=77, rank=24, noise=0.2, outlier=None, dtype="float16")
    c, co = _pipeline_case(kvf, oracle, k, v, "aggressive")
    Rk, Rv = c.tensor_info(0)["R"], c.tensor_info(1)["R"]
    assert 32 < Rk <= 64 and 32 < Rv <= 64, (Rk, Rv)
    kr, vr = oracle.decompress(co, threads=4)
    out = kvf.decompress(c)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    _exact(L, True)
    try:
        out = kvf.decompress(c)
    finally:
        _exact(L, False)
    assert np.array_equal(bits(out.keys()), bits(kr)) and np.array_equal(bits(out.values()), bits(vr))
    assert np.allclose(c.calibration_scores(), co["scores"], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("shape,thr", [((2, 300, 16), 0.9), ((4, 1000, 128), 0.99), ((2, 77, 13), 0.8)])
def test_reconstruct_parity(kvf, oracle, shape, thr):
    from kvforge_b200 import _lib as L
    _, x32 = _x(shape, 31)
    bvt, ranks, R = _basis(oracle, x32, thr)
    basis = kvf.Basis.from_host(bvt, ranks)
    Po = oracle.project(x32, bvt, ranks)
    ref = oracle.reconstruct(Po, bvt, ranks)
    pr = kvf.GpuProjector()
    out = host(pr.reconstruct(dev(Po), basis))
    assert rel(out, ref) < REC_TOL
    ctx = L.context(0)
    L.check(L.lib().kvf_set_exact_reconstruct(ctx, 1))
    try:
        out_exact = host(pr.reconstruct(dev(Po), basis))
    finally:
        L.check(L.lib().kvf_set_exact_reconstruct(ctx, 0))
    assert np.array_equal(bits(out_exact), bits(ref))


def _exact(L, on):
    L.check(L.lib().kvf_set_exact_reconstruct(L.context(0), 1 if on else 0))


@pytest.fixture
def tensor_cores():
    """Selects the tcgen05 reconstruction engine for one test."""
    from kvforge_b200 import _lib as L
    L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), L.RECON_TENSOR_CORE))
    yield
    L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), L.RECON_AUTO))


@pytest.mark.parametrize("H,T,R,ranks", [(1, 1, 1, [1]), (2, 127, 3, [3, 2]), (3, 128, 8, [8, 8, 5]),
                                         (2, 129, 9, [9, 1]), (2, 1000, 16, [16, 12]), (5, 300, 13, [13, 0, 7, 13, 4]),
                                         (2, 500, 17, [17, 9]), (3, 260, 32, [32, 31, 1]), (2, 300, 40, [40, 33]),
                                         (1, 257, 64, [64])])
def test_tensor_core_reconstruct_raw(kvf, oracle, tensor_cores, H, T, R, ranks):
    """head_dim 128, R <= 64: the tcgen05 path (partial tiles, ranks below R,
    rank 0, one and two A-operand stages) against the reference loop; the
    exact mode stays bit-exact."""
    from kvforge_b200 import _lib as L
    rng = np.random.default_rng(H * 1000 + T + R)
    D = 128
    bvt = rng.standard_normal((H, R, D)).astype(np.float32) / np.sqrt(D)
    rk = np.asarray(ranks, np.uint64)
    Po = (rng.standard_normal((H, T, R)) * 4).astype(np.float32)
    ref = oracle.reconstruct(Po, bvt, rk)
    basis = kvf.Basis.from_host(bvt, rk)
    pr = kvf.GpuProjector()
    out = host(pr.reconstruct(dev(Po), basis))
    assert rel(out, ref) < REC_TOL
    if H * T >= 128 and max(ranks) > 1:  # a different engine ran: its roundings differ somewhere
        L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), L.RECON_CUDA_CORE))
        out_fma = host(pr.reconstruct(dev(Po), basis))
        L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), L.RECON_TENSOR_CORE))
        assert not np.array_equal(bits(out), bits(out_fma))
    _exact(L, True)
    try:
        out_exact = host(pr.reconstruct(dev(Po), basis))
    finally:
        _exact(L, False)
    assert np.array_equal(bits(out_exact), bits(ref))


@pytest.mark.parametrize("dt", [INT8, INT4])
@pytest.mark.parametrize("shape,thr,maxr", [((2, 300, 128), 0.9, 12), ((3, 77, 128), 0.75, 12),
                                            ((2, 300, 128), 0.99, 40), ((2, 400, 128), 0.999, 64)])
def test_tensor_core_reconstruct_codes(kvf, oracle, tensor_cores, dt, shape, thr, maxr):
    """Projected INT8 and INT4 codes, keys per channel and values per token,
    decompressed on the tcgen05 path against the reference pipeline."""
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    H, T, D = shape
    k, v = synth.numpy_layer(H, T, D, seed=T + dt, rank=10, dtype="float16")
    cfg = kvf.config_from_preset("balanced")
    cfg.key_data_type = cfg.value_data_type = dt
    cfg.projection_variance_threshold = thr
    kb = kvf.Basis.compute(dev(k), thr, max_rank=maxr)
    vb = kvf.Basis.compute(dev(v), thr, max_rank=maxr)
    assert kb.R <= maxr and vb.R <= maxr
    c = kvf.CompressionPipeline().compress_with_config(kvf.KVCache(dev(k), dev(v), 0), cfg, kb, vb)
    kr = oracle.decompress_tensor(oracle.compress_tensor(k.astype(np.float32), dt, PC, kb.host()[:2]))
    vr = oracle.decompress_tensor(oracle.compress_tensor(v.astype(np.float32), dt, PT, vb.host()[:2]))
    out = kvf.decompress(c)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    _exact(L, True)
    try:
        out = kvf.decompress(c)
    finally:
        _exact(L, False)
    assert np.array_equal(bits(out.keys()), bits(kr)) and np.array_equal(bits(out.values()), bits(vr))


@pytest.mark.parametrize("shape,thr,f16", [((2, 400, 16), 0.9, False), ((4, 4096, 128), 0.75, True),
                                           ((3, 50, 128), 0.9, False)])
def test_basis_ranks(kvf, oracle, shape, thr, f16):
    xin, x32 = _x(shape, 41, f16)
    rng = np.random.default_rng(5)
    # low-rank structure so the threshold sits between well-separated values
    H, T, D = shape
    k = min(8, D)
    x32 = (np.einsum("htr,hrd->htd", rng.standard_normal((H, T, k)) * (0.7 ** np.arange(k)),
                     rng.standard_normal((H, k, D))) + 0.01 * rng.standard_normal(shape)).astype(np.float32)
    xin = x32.astype(np.float16) if f16 else x32
    x32 = xin.astype(np.float32)
    b = kvf.Basis.compute(dev(xin), thr)
    bvt, ranks, sv = b.host()
    _, ranks_o, R_o = _basis(oracle, x32, thr)
    assert np.array_equal(ranks, ranks_o)
    for h in range(H):
        s64 = np.linalg.svd(x32[h].astype(np.float64), compute_uv=False)
        n = min(T, D)
        assert np.allclose(sv[h, :n], s64[:n], rtol=1e-4, atol=1e-3 * s64[0])
        # the basis spans the same subspace as the SVD's leading right vectors
        _, _, vt = np.linalg.svd(x32[h].astype(np.float64), full_matrices=False)
        r = int(ranks[h])
        proj = vt[:r] @ bvt[h, :r].T.astype(np.float64)
        assert np.allclose(np.abs(np.linalg.det(proj)), 1.0, atol=1e-3)


# ---- rANS --------------------------------------------------------------------------
@pytest.mark.parametrize("n", [1, 31, 32, 33, 1000, 8191, 8192, 8193, 16385, 200000, 1 << 22])
def test_rans_parity(kvf, oracle, n):
    rng = np.random.default_rng(n)
    data = np.clip(np.round(rng.normal(120, 15, n)), 0, 255).astype(np.uint8)
    codec = kvf.GpuEntropyCodec()
    comp, state = codec.encode(dev(data))
    comp_o, freq_o = oracle.rans_encode(data)
    assert np.array_equal(host(state.frequencies).astype(np.uint32), freq_o)
    assert np.array_equal(host(comp), comp_o)
    # cross-decoding both ways
    assert np.array_equal(host(codec.decode(dev(comp_o), state)), data)
    assert np.array_equal(oracle.rans_decode(host(comp), freq_o, n), data)


def test_rans_golden_containers(kvf, golden):
    codec = kvf.GpuEntropyCodec()
    names = sorted(k[2:-5] for k in golden.files if k.startswith("r_") and k.endswith("_data"))
    for name in names:
        data = golden[f"r_{name}_data"]
        st = kvf.EntropyState(dev(golden[f"r_{name}_freq"].astype(np.int32)), data.size)
        out = host(codec.decode(dev(golden[f"r_{name}_comp"]), st))
        assert np.array_equal(out, data), name


def test_rans_special_inputs(kvf, oracle):
    codec = kvf.GpuEntropyCodec()
    for data in (np.full(70000, 7, np.uint8), np.arange(256, dtype=np.uint8), np.zeros(1, np.uint8),
                 np.tile(np.arange(256, dtype=np.uint8), 300)):
        comp, st = codec.encode(dev(data))
        comp_o, _ = oracle.rans_encode(data)
        assert np.array_equal(host(comp), comp_o)
        assert np.array_equal(host(codec.decode(comp, st)), data)
    empty, st = codec.encode(dev(np.zeros(0, np.uint8)))
    assert empty.numel() == 0 and st.original_len == 0
    raw, st = codec.encode(dev(np.arange(5, dtype=np.uint8)), enabled=False)
    assert np.array_equal(host(raw), np.arange(5)) and st.frequencies.numel() == 0


def test_rans_corrupt_is_reported(kvf, oracle):
    rng = np.random.default_rng(3)
    data = rng.integers(0, 60, 50000).astype(np.uint8)
    codec = kvf.GpuEntropyCodec()
    comp, st = codec.encode(dev(data))
    c = host(comp)
    with pytest.raises(kvf.KvForgeError) as e:
        codec.decode(dev(c[:-4]), st)
    assert e.value.status == 10
    with pytest.raises(kvf.KvForgeError) as e:
        codec.decode(dev(c[:-1]), st)
    assert e.value.status == 5
    bad = c.copy()
    bad[0] ^= 1
    with pytest.raises(kvf.KvForgeError) as e:
        codec.decode(dev(bad), st)
    assert e.value.status == 10
    # the context stays usable after a reported corruption
    assert np.array_equal(host(codec.decode(comp, st)), data)


@pytest.mark.parametrize("which", ["mbarrier", "lookback"])
def test_bounded_wait_timeout_is_reported(kvf, oracle, which):
    """A device wait on a barrier (or a look-back status word) that nothing
    completes gives up after its limit; the host reads KVF_ERR_DEVICE_TIMEOUT
    from the status word, and the same context then compresses bit-exactly."""
    from kvforge_b200 import _lib as L
    ctx = L.context(0)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    kind = L.WAIT_MBARRIER if which == "mbarrier" else L.WAIT_LOOKBACK
    L.check(L.lib().kvf_selftest_wait_timeout(ctx, kind, s))
    assert L.lib().kvf_sync(ctx, s) == L.ERR_DEVICE_TIMEOUT
    assert L.lib().kvf_sync(ctx, s) == 0  # reported once, then cleared
    rng = np.random.default_rng(4)
    data = rng.integers(0, 60, 70000).astype(np.uint8)
    codec = kvf.GpuEntropyCodec()
    comp, st = codec.encode(dev(data))
    assert np.array_equal(host(comp), oracle.rans_encode(data)[0])
    assert np.array_equal(host(codec.decode(comp, st)), data)


# ---- whole pipeline -----------------------------------------------------------------
def _pipeline_case(kvf, oracle, k, v, preset):
    import kvforge_b200.synth  # noqa: F401
    cfg = kvf.config_from_preset(preset)
    kb = vb = None
    bases = None
    if cfg.enable_projection:
        kb = kvf.Basis.compute(dev(k), cfg.projection_variance_threshold)
        vb = kvf.Basis.compute(dev(v), cfg.projection_variance_threshold)
        kh, vh = kb.host(), vb.host()
        bases = ((kh[0], kh[1]), (vh[0], vh[1]))
    c = kvf.CompressionPipeline().compress(kvf.KVCache(dev(k), dev(v), 3), preset, kb, vb)
    co = oracle.compress(k.astype(np.float32), v.astype(np.float32), preset, 3, bases, threads=4)
    for which, name in ((0, "key"), (1, "value")):
        parts = c.tensor_parts(which)
        ot = co[name]
        assert np.array_equal(host(parts["data"]), ot["data"]), (preset, name)
        assert np.array_equal(bits(host(parts["scales"])), bits(ot["scales"])), (preset, name)
        assert np.array_equal(bits(host(parts["mins"])), bits(ot["mins"])), (preset, name)
        if ot["entropy"] is not None and ot["entropy"][1] > 0:
            assert np.array_equal(host(parts["freq"]).astype(np.uint32), ot["entropy"][0])
    assert c.compressed_size_bytes() == oracle.compressed_size_bytes(co)
    assert c.original_size_bytes() == co["original_size_bytes"]
    assert c.ratio() == oracle.ratio(co)
    return c, co


@pytest.mark.parametrize("preset", ["conservative", "balanced", "aggressive", "adaptive"])
@pytest.mark.parametrize("shape,f16", [((4, 128, 32), False), ((3, 257, 128), True), ((2, 1000, 64), False)])
def test_pipeline_parity(kvf, oracle, preset, shape, f16):
    from kvforge_b200 import synth
    from kvforge_b200 import _lib as L
    H, T, D = shape
    k, v = synth.numpy_layer(H, T, D, seed=hash((preset, shape)) % 1000, rank=min(12, D),
                             dtype="float16" if f16 else "float32")
    c, co = _pipeline_case(kvf, oracle, k, v, preset)
    kr, vr = oracle.decompress(co, threads=4)
    out = kvf.decompress(c)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    ctx = L.context(0)
    L.check(L.lib().kvf_set_exact_reconstruct(ctx, 1))
    try:
        out = kvf.decompress(c)
    finally:
        L.check(L.lib().kvf_set_exact_reconstruct(ctx, 0))
    assert np.array_equal(bits(out.keys()), bits(kr)) and np.array_equal(bits(out.values()), bits(vr))
    if preset == "aggressive" and T >= 64:
        assert np.allclose(c.calibration_scores(), co["scores"], rtol=1e-6, atol=1e-7)


def test_pipeline_reference_bounds(kvf):
    """tests/roundtrip.rs and tests/compression_ratio.rs semantics on the GPU path."""
    rng = np.random.default_rng(12)
    k = rng.uniform(-1, 1, (4, 128, 32)).astype(np.float32)
    v = rng.uniform(-1, 1, (4, 128, 32)).astype(np.float32)
    for preset, bound in (("conservative", 5e-4), ("balanced", 5e-2), ("aggressive", 0.5)):
        out = kvf.decompress(kvf.compress(kvf.KVCache(k, v, 0), preset))
        assert out.layer_idx == 0
        assert float(((out.keys() - k) ** 2).mean()) < bound and float(((out.values() - v) ** 2).mean()) < bound
    k = rng.uniform(-1, 1, (8, 1024, 128)).astype(np.float32)
    v = rng.uniform(-1, 1, (8, 1024, 128)).astype(np.float32)
    r = {p: kvf.compress(kvf.KVCache(k, v, 0), p).ratio() for p in ("conservative", "balanced", "aggressive")}
    assert 3.0 < r["conservative"] < 6.0 and r["balanced"] > r["conservative"] and r["aggressive"] > r["balanced"]


def test_serialize_roundtrip(kvf):
    from kvforge_b200 import synth
    k, v = synth.numpy_layer(2, 300, 64, seed=5, rank=8, dtype="float16")
    for preset in ("conservative", "balanced", "aggressive"):
        c = kvf.compress(kvf.KVCache(k, v, 9), preset)
        blob = c.to_bytes()
        c2 = kvf.CompressedKV.from_bytes(blob)
        assert c2.layer_idx == 9 and c2.shape == (2, 300, 64)
        assert c2.compressed_size_bytes() == c.compressed_size_bytes() and c2.ratio() == c.ratio()
        a, b = kvf.decompress(c), kvf.decompress(c2)
        assert np.array_equal(a.keys(), b.keys()) and np.array_equal(a.values(), b.values())
        assert c2.to_bytes() == blob
    with pytest.raises(kvf.KvForgeError) as e:
        kvf.CompressedKV.from_bytes(blob[:-7])
    assert e.value.status == 6


@pytest.mark.parametrize("preset", ["conservative", "balanced", "aggressive", "adaptive"])
def test_serialize_is_reference_wire_format(kvf, oracle, preset):
    """to_bytes is the reference's CompressedKV.to_bytes (bincode 1.x of
    types.rs:36-148): byte-identical to the oracle's encoding of the same
    layer, and bytes the oracle writes load and decompress on the GPU."""
    from kvforge_b200 import synth
    k, v = synth.numpy_layer(3, 257, 64, seed=21, rank=8, dtype="float16")
    c, co = _pipeline_case(kvf, oracle, k, v, preset)
    blob = c.to_bytes()
    co["layer_idx"] = c.layer_idx
    assert blob == oracle.to_bincode(co)
    c2 = kvf.CompressedKV.from_bytes(oracle.to_bincode(co))
    kr, vr = oracle.decompress(co, threads=4)
    out = kvf.decompress(c2)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    assert c2.ratio() == oracle.ratio(co)
    bad = bytearray(blob)
    key_data_len = int(np.frombuffer(blob[32:40], "<u8")[0])
    nsc = int(np.frombuffer(blob[40 + key_data_len:48 + key_data_len], "<u8")[0])
    tag = 48 + key_data_len + 4 * nsc + 8 + 4 * nsc + 8 + 32  # key_data.projection_state tag
    assert blob[tag] in (0, 1)
    bad[tag] = 2
    with pytest.raises(kvf.KvForgeError) as e:
        kvf.CompressedKV.from_bytes(bytes(bad))
    assert e.value.status == 6


def test_deserialize_rejects_lengths_beyond_the_buffer(kvf):
    """A few-byte layer whose header claims a huge basis (H = 65535, R = D =
    1024: 275 GB of basis_vt) is a serialisation error, not a host allocation
    of that size; so is a rank list longer than the bytes that remain."""
    import struct
    H, T, D, R = 65535, 1, 1024, 1024
    u64 = lambda *v: struct.pack("<" + "Q" * len(v), *v)
    head = u64(0, H, T, D)
    tensor = (u64(0)            # quantized_data: empty
              + u64(0) + u64(0)  # scales, mins: empty
              + struct.pack("<II", INT4, PC) + u64(3, H, T, R)
              + b"\x01" + u64(H * R * D))  # projection_state: Some, basis_vt length
    with pytest.raises(kvf.KvForgeError) as e:
        kvf.CompressedKV.from_bytes(head + tensor + b"\x00" * 64)
    assert e.value.status == 6
    H, D, R = 2, 4, 1
    head = u64(0, H, T, D)
    tensor = (u64(0) + u64(0) + u64(0) + struct.pack("<II", INT4, PC) + u64(3, H, T, R)
              + b"\x01" + u64(H * R * D) + b"\x00" * (4 * H * R * D)
              + u64(H))  # ranks: H entries claimed, none present
    with pytest.raises(kvf.KvForgeError) as e:
        kvf.CompressedKV.from_bytes(head + tensor)
    assert e.value.status == 6


def test_compress_decompress_free_across_streams(kvf):
    """Compress on stream A, decompress on stream B with no host
    synchronisation in between, free at once, and let stream A compress other
    layers that may take the freed buffers from the pool: B's output is
    bit-identical to a same-stream decompression of the same layer."""
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    lib, ctx = L.lib(), L.context(0)
    cfg = kvf.config_from_preset("aggressive")
    k, v = synth.workload_layer("llama3_8b_32k", 3, backend="torch")
    k, v = k[:, :8192].contiguous(), v[:, :8192].contiguous()
    H, T, D = k.shape
    kb = kvf.Basis.compute(k, cfg.projection_variance_threshold)
    vb = kvf.Basis.compute(v, cfg.projection_variance_threshold)
    ref = kvf.CompressionPipeline().compress(kvf.KVCache(k, v, 0), "aggressive", kb, vb)
    ref_out = kvf.decompress(ref)
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    outs = []
    for rep in range(3):
        ko = torch.empty((H, T, D), dtype=torch.float32, device="cuda")
        vo = torch.empty_like(ko)
        torch.cuda.synchronize()
        h = C.c_void_p()
        L.check(lib.kvf_compress_layer(ctx, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()), L.IN_F16, H, T, D,
                                       rep, C.byref(cfg), kb.handle, vb.handle, C.byref(h),
                                       C.c_void_p(sa.cuda_stream)))
        L.check(lib.kvf_decompress_layer(ctx, h, C.c_void_p(ko.data_ptr()), C.c_void_p(vo.data_ptr()),
                                         C.c_void_p(sb.cuda_stream)))
        L.check(lib.kvf_compressed_free(h))
        for j in range(2):  # new objects on A reuse the pool's blocks once the free is ordered
            h2 = C.c_void_p()
            L.check(lib.kvf_compress_layer(ctx, C.c_void_p(v.data_ptr()), C.c_void_p(k.data_ptr()), L.IN_F16, H, T,
                                           D, j, C.byref(cfg), vb.handle, kb.handle, C.byref(h2),
                                           C.c_void_p(sa.cuda_stream)))
            L.check(lib.kvf_compressed_free(h2))
        outs.append((ko, vo))
    torch.cuda.synchronize()
    L.check(lib.kvf_sync(ctx, None))
    for ko, vo in outs:
        assert np.array_equal(ko.cpu().numpy(), ref_out.keys())
        assert np.array_equal(vo.cpu().numpy(), ref_out.values())


def test_host_buffer_entry_points(kvf):
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    k, v = synth.numpy_layer(2, 256, 128, seed=8, rank=8, dtype="float16")
    cfg = kvf.config_from_preset("aggressive")
    h = C.c_void_p()
    L.check(L.lib().kvf_compress_layer_host(L.context(0), k.ctypes.data_as(C.c_void_p), v.ctypes.data_as(C.c_void_p),
                                            1, 2, 256, 128, 4, C.byref(cfg), None, None, C.byref(h), None))
    c = kvf.CompressedKV(h, 0)
    ko = np.zeros((2, 256, 128), np.float32)
    vo = np.zeros((2, 256, 128), np.float32)
    L.check(L.lib().kvf_decompress_layer_host(L.context(0), h, ko.ctypes.data_as(C.c_void_p),
                                              vo.ctypes.data_as(C.c_void_p), None))
    ref = kvf.decompress(c)
    assert np.array_equal(ko, ref.keys()) and np.array_equal(vo, ref.values())
    assert c.layer_idx == 4


def test_full_size_llama_layer(kvf, oracle):
    """One Llama-3-8B-shaped layer at full size ([8, 32768, 128] fp16,
    Aggressive): codes, bitstreams and ratio bit-exact against the oracle;
    reconstruction within REC_TOL of the oracle's."""
    from kvforge_b200 import synth
    k, v = synth.workload_layer("llama3_8b_32k", 0, backend="torch")
    kh, vh = host(k), host(v)
    c, co = _pipeline_case(kvf, oracle, kh, vh, "aggressive")
    out = kvf.decompress(c)
    kr, vr = oracle.decompress(co, threads=8)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    assert c.ratio() > 10
    from kvforge_b200 import _lib as L
    L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), L.RECON_TENSOR_CORE))
    try:
        out = kvf.decompress(c)
    finally:
        L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), L.RECON_AUTO))
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
