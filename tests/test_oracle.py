"""CPU tests of the oracle: the reference's own known answers and bounds, and
the golden fixtures made by independent restatements (tests/golden/make_golden.py).
Mirrors the reference tests in crates/kvforge-cpu/src/*.rs and crates/kvforge-cpu/tests/."""
import numpy as np
import pytest

from oracle import quant_numpy as QN

INT4, INT8 = 0, 1
PC, PT = 0, 1


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---- reference known-answer tests -------------------------------------------
def test_pack_int4_kat(oracle):  # quantize.rs:246-258
    assert oracle.pack_int4(3, 12) == 0xC3
    assert oracle.unpack_int4(0xC3) == (3, 12)
    assert oracle.pack_int4(0, 0) == 0x00
    assert oracle.pack_int4(15, 15) == 0xFF
    assert oracle.unpack_int4(0xFF) == (15, 15)


def test_select_rank_kat(oracle):  # projection.rs:242-253
    sv = [10.0, 5.0, 2.0, 1.0, 0.5]
    assert oracle.select_rank(sv, 0.95) == 2
    assert oracle.select_rank(sv, 0.95, 2) == 2
    assert oracle.select_rank(sv, 0.5) == 1
    assert oracle.select_rank([], 0.9) == 0
    assert oracle.select_rank([0.0, 0.0], 0.9) == 1


def test_histogram_kat(oracle, golden):  # entropy.rs:192-199
    f = oracle.histogram(golden["kat_hist_data"])
    assert list(f[:4]) == list(golden["kat_hist_expect"])


# ---- golden fixtures ----------------------------------------------------------
def _quant_keys(golden):
    return sorted(k[:-2] for k in golden.files if k.startswith("q") and k.endswith("_x"))


def test_quantize_golden(oracle, golden):
    keys = _quant_keys(golden)
    assert len(keys) == 20
    for key in keys:
        si, dt, ax = map(int, key[1:].split("_"))
        x = golden[key + "_x"]
        p, s, m = oracle.quantize(x, dt, ax)
        assert np.array_equal(p, golden[key + "_packed"]), key
        assert np.array_equal(bits(s), bits(golden[key + "_scales"])), key
        assert np.array_equal(bits(m), bits(golden[key + "_mins"])), key
        d = oracle.dequantize(p, s, m, dt, ax, x.shape)
        assert np.array_equal(bits(d), bits(golden[key + "_deq"])), key


def test_rans_golden(oracle, golden):
    names = sorted(k[2:-5] for k in golden.files if k.startswith("r_") and k.endswith("_data"))
    assert len(names) == 6
    for name in names:
        data = golden[f"r_{name}_data"]
        chunk = int(golden[f"r_{name}_chunk"][0])
        comp, freq = oracle.rans_encode(data, chunk)
        assert np.array_equal(comp, golden[f"r_{name}_comp"]), name
        assert np.array_equal(freq, golden[f"r_{name}_freq"]), name
        dec = oracle.rans_decode(golden[f"r_{name}_comp"], freq, data.size)
        assert np.array_equal(dec, data), name


def test_ranks_golden(oracle, golden):
    x = golden["p_x"]
    bf, sv = oracle.compute_basis(x)
    for thr in (50, 75, 90, 99):
        _, ranks, R = oracle.select_basis(bf, sv, x.shape[1], thr / 100)
        assert np.array_equal(ranks, golden[f"p_ranks_{thr}"]), thr
        assert R == int(golden[f"p_ranks_{thr}"].max())


# ---- quantizer: numpy restatement vs C, reference bounds ------------------------
@pytest.mark.parametrize("shape", [(4, 64, 32), (3, 17, 9), (1, 1, 1), (2, 128, 5)])
@pytest.mark.parametrize("dt", [INT4, INT8])
@pytest.mark.parametrize("ax", [PC, PT])
def test_quantize_numpy_vs_c(oracle, shape, dt, ax):
    rng = np.random.default_rng(hash((shape, dt, ax)) % 2**32)
    x = (rng.standard_normal(shape) * rng.uniform(0.01, 10)).astype(np.float32)
    p, s, m = oracle.quantize(x, dt, ax)
    p2, s2, m2 = QN.quantize(x, dt, ax)
    assert np.array_equal(p, p2)
    assert np.array_equal(bits(s), bits(s2)) and np.array_equal(bits(m), bits(m2))
    d = oracle.dequantize(p, s, m, dt, ax, shape)
    assert np.array_equal(bits(d), bits(QN.dequantize(p, s, m, dt, ax, shape)))


@pytest.mark.parametrize("dt,ax,bound", [(INT8, PC, 1e-3), (INT4, PC, 1e-2), (INT8, PT, 1e-3), (INT4, PT, 1e-2)])
def test_quantize_roundtrip_mse(oracle, dt, ax, bound):  # quantize.rs:260-311
    x = np.random.default_rng(1).uniform(-1, 1, (4, 64, 32)).astype(np.float32)
    p, s, m = oracle.quantize(x, dt, ax)
    d = oracle.dequantize(p, s, m, dt, ax, x.shape)
    assert float(((d - x) ** 2).mean()) < bound


def test_kivi_param_counts(oracle):  # quantize.rs:313-340
    rng = np.random.default_rng(2)
    k = rng.uniform(-1, 1, (2, 16, 8)).astype(np.float32)
    _, ks, _ = oracle.quantize(k, INT4, PC)
    _, vs, _ = oracle.quantize(k, INT4, PT)
    assert ks.size == 2 * 8 and vs.size == 2 * 16


def test_int4_raw_ratio(oracle):  # quantize.rs:342-355
    x = np.random.default_rng(3).uniform(-1, 1, (4, 128, 64)).astype(np.float32)
    p, _, _ = oracle.quantize(x, INT4, PC)
    assert x.size * 4 / p.size > 7.0


def test_quantize_errors(oracle):
    x = np.zeros((2, 4, 4), np.float32)
    with pytest.raises(oracle.OracleError) as e:
        oracle.quantize(x, 2, PC)  # F32, quantize.rs:52-56
    assert e.value.status == 3
    p, s, m = oracle.quantize(x, INT8, PC)
    with pytest.raises(oracle.OracleError):
        oracle.dequantize(p[:-1], s, m, INT8, PC, x.shape)  # quantize.rs:191-197
    p4, s4, m4 = oracle.quantize(np.zeros((1, 1, 3), np.float32), INT4, PT)
    assert p4.size == 2
    with pytest.raises(oracle.OracleError):
        oracle.dequantize(p4[:1], s4, m4, INT4, PT, (1, 1, 3))
    # extra INT4 bytes are truncated away, as the reference does
    out = oracle.dequantize(np.concatenate([p4, [0xFF]]).astype(np.uint8), s4, m4, INT4, PT, (1, 1, 3))
    assert out.shape == (1, 1, 3)


def test_quantize_special_values(oracle):
    x = np.array([[[0.0, -0.0, 1.0, np.nan], [np.inf, -1.0, 2.0, 3.0]]], np.float32)
    for dt in (INT4, INT8):
        for ax in (PC, PT):
            p, s, m = oracle.quantize(x, dt, ax)
            p2, s2, m2 = QN.quantize(x, dt, ax)
            assert np.array_equal(p, p2)
            assert np.array_equal(bits(s), bits(s2)) and np.array_equal(bits(m), bits(m2))


# ---- calibration (calibration.rs:82-150) -------------------------------------------
def test_calibrate(oracle):
    rng = np.random.default_rng(4)
    keys = np.zeros((2, 128, 16), np.float32)
    keys[0] = rng.uniform(-0.1, 0.1, (128, 16))
    keys[1] = rng.uniform(-10, 10, (128, 16))
    s = oracle.calibrate(keys)
    assert s.shape == (2,) and s[1] > s[0] and np.all((s >= 0) & (s <= 1))
    with pytest.raises(oracle.OracleError) as e:
        oracle.calibrate(np.zeros((2, 32, 16), np.float32))
    assert e.value.status == 2
    u = oracle.calibrate(rng.uniform(-1, 1, (4, 128, 16)).astype(np.float32))
    assert u.max() - u.min() < 0.3
    z = oracle.calibrate(np.zeros((3, 64, 4), np.float32))
    assert np.all(z == 0.5)


# ---- projection (projection.rs:186-253) --------------------------------------------
def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_project_reconstruct(oracle):
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, (2, 32, 16)).astype(np.float32)
    bvt, ranks = oracle.basis_for(x, 0.99)
    P = oracle.project(x, bvt, ranks)
    xr = oracle.reconstruct(P, bvt, ranks)
    assert xr.shape == x.shape and float(((xr - x) ** 2).mean()) < 0.01
    bvt5, r5 = oracle.basis_for(x, 0.5)
    assert float(((oracle.reconstruct(oracle.project(x, bvt5, r5), bvt5, r5) - x) ** 2).mean()) < 1.0
    # cap (projection.rs:223-239)
    x1 = rng.uniform(-1, 1, (1, 64, 32)).astype(np.float32)
    bf, sv = oracle.compute_basis(x1)
    bvt8, r8, R8 = oracle.select_basis(bf, sv, 64, 0.80, 8)
    assert R8 <= 8 and r8[0] <= 8
    # projected coefficients agree with the fp64 SVD's U*S up to sign
    u, s, vt = np.linalg.svd(x[0].astype(np.float64), full_matrices=False)
    k = int(ranks[0])
    us = u[:, :k] * s[:k]
    sgn = np.sign(np.sum(us * P[0, :, :k], axis=0))
    assert _rel(P[0, :, :k].astype(np.float64), us * sgn) < 1e-4
    # padded columns are +0.0
    assert np.all(bits(P[1, :, int(ranks[1]):]) == 0)


def test_projection_fma_order(oracle):
    """The projection is one fmaf chain over c starting at +0.0."""
    rng = np.random.default_rng(6)
    x = rng.standard_normal((1, 5, 7)).astype(np.float32)
    bvt = rng.standard_normal((1, 3, 7)).astype(np.float32)
    P = oracle.project(x, bvt, np.array([3], np.uint64))
    from fractions import Fraction
    for t in range(5):
        for r in range(3):
            acc = np.float32(0.0)
            for c in range(7):
                exact = Fraction(float(x[0, t, c])) * Fraction(float(bvt[0, r, c])) + Fraction(float(acc))
                acc = _round_f32(exact)
            assert bits(np.float32(acc)) == bits(P[0, t, r])


def _round_f32(fr):
    """Correctly rounded Fraction -> float32 (round half to even)."""
    f64 = float(fr)
    c = np.float32(f64)
    # candidates around the f64 rounding; pick the nearest to the exact value
    cands = [np.nextafter(c, np.float32(-np.inf)), c, np.nextafter(c, np.float32(np.inf))]
    from fractions import Fraction
    best = min(cands, key=lambda v: (abs(Fraction(float(v)) - fr), int(np.float32(v).view(np.uint32)) & 1))
    return np.float32(best)


# ---- rANS container ---------------------------------------------------------------
@pytest.mark.parametrize("n", [1, 31, 32, 33, 1000, 8191, 8192, 8193, 16384, 16385, 40000])
def test_rans_roundtrip_sizes(oracle, n):
    rng = np.random.default_rng(n)
    data = np.clip(np.round(rng.normal(100, 20, n)), 0, 255).astype(np.uint8)
    comp, freq = oracle.rans_encode(data)
    assert comp.size % 4 == 0
    assert np.array_equal(oracle.rans_decode(comp, freq, n), data)


def test_rans_skewed_compresses(oracle):  # entropy.rs:130-166
    data = np.zeros(1000, np.uint8)
    data[100], data[200], data[300] = 1, 2, 255
    comp, freq = oracle.rans_encode(data)
    assert comp.size < data.size
    assert np.array_equal(oracle.rans_decode(comp, freq, data.size), data)
    full = np.arange(256, dtype=np.uint8)
    c2, f2 = oracle.rans_encode(full)
    assert np.array_equal(oracle.rans_decode(c2, f2, 256), full)


def test_rans_near_entropy(oracle):
    rng = np.random.default_rng(7)
    p = np.exp(-0.5 * ((np.arange(256) - 128) / 9.0) ** 2)
    p /= p.sum()
    data = rng.choice(256, size=200000, p=p).astype(np.uint8)
    comp, freq = oracle.rans_encode(data)
    ideal = oracle.entropy_bits(freq) / 8
    assert comp.size < ideal * 1.03 + 4096


def test_rans_corrupt(oracle):
    rng = np.random.default_rng(8)
    data = rng.integers(0, 40, 5000).astype(np.uint8)
    comp, freq = oracle.rans_encode(data, 1024)
    with pytest.raises(oracle.OracleError) as e:
        oracle.rans_decode(comp[:-4], freq, data.size)
    assert e.value.status == 10
    with pytest.raises(oracle.OracleError) as e:
        oracle.rans_decode(comp[:-1], freq, data.size)
    assert e.value.status == 5  # entropy.rs:94-98
    for pos in (0, 40, 200, comp.size - 2):
        bad = comp.copy()
        bad[pos] ^= 0x5A
        try:
            out = oracle.rans_decode(bad, freq, data.size)
            assert not np.array_equal(out, data) or pos >= 32  # payload flips may decode to garbage
        except oracle.OracleError as err:
            assert err.status in (5, 10)


# ---- pipeline (pipeline.rs:205-281, tests/roundtrip.rs, tests/compression_ratio.rs) ----
def _kv(shape, seed):
    rng = np.random.default_rng(seed)
    return rng.uniform(-1, 1, shape).astype(np.float32), rng.uniform(-1, 1, shape).astype(np.float32)


@pytest.mark.parametrize("preset,bound", [("conservative", 5e-4), ("balanced", 5e-2), ("aggressive", 0.5)])
def test_pipeline_roundtrip_mse(oracle, preset, bound):
    k, v = _kv((4, 128, 32), 9)
    c = oracle.compress(k, v, preset)
    kr, vr = oracle.decompress(c)
    assert kr.shape == k.shape and vr.shape == v.shape
    assert float(((kr - k) ** 2).mean()) < bound and float(((vr - v) ** 2).mean()) < bound


def test_pipeline_ratios(oracle):
    k, v = _kv((8, 1024, 128), 10)
    r = {p: oracle.ratio(oracle.compress(k, v, p, threads=4)) for p in ("conservative", "balanced", "aggressive")}
    assert 3.0 < r["conservative"] < 6.0
    assert r["balanced"] > 4.0 and r["aggressive"] > 4.0
    assert r["balanced"] > r["conservative"] and r["aggressive"] > r["balanced"]


def test_conservative_ratio_formula(oracle):
    """types.rs accounting: [32,2048,128] INT8 -> 67108864 / 17334272."""
    H, T, D = 32, 2048, 128
    comp = (H * T * D + 2 * 4 * H * D) + (H * T * D + 2 * 4 * H * T)  # keys per-channel + values per-token
    assert comp == 17334272 and abs(2 * H * T * D * 4 / comp - 3.8715) < 1e-4
    k, v = _kv((2, 16, 8), 11)
    c = oracle.compress(k, v, "conservative")
    assert oracle.compressed_size_bytes(c) == (2 * 16 * 8 + 2 * 4 * 2 * 8) + (2 * 16 * 8 + 2 * 4 * 2 * 16)


def test_bincode_known_answer(oracle):
    """The oracle's CompressedKV.to_bytes against bytes written out by hand from
    bincode 1.x's default encoding (little-endian, u64 lengths and usize, u8
    Option tags, u32 enum variants) of types.rs:36-148."""
    import struct
    key = dict(data=np.array([3, 250], np.uint8), scales=np.array([0.5], np.float32),
               mins=np.array([-1.0], np.float32), data_type=1, axis=0, qshape=(1, 2, 1),
               proj=(np.array([[[1.0]]], np.float32), np.array([1], np.uint64)), entropy=None)
    val = dict(data=np.array([1, 2], np.uint8), scales=np.array([0.25, 2.0], np.float32),
               mins=np.array([0.0, 1.5], np.float32), data_type=1, axis=1, qshape=(1, 2, 1), proj=None,
               entropy=(np.zeros(0, np.uint32), 2))
    ckv = dict(layer_idx=7, shape=(1, 2, 1), key=key, value=val, original_size_bytes=16)
    want = (struct.pack("<QQQQ", 7, 1, 2, 1)
            # key_data: quantized_data, scales, mins, DataType::INT8, QuantAxis::PerChannel, shape
            + struct.pack("<Q", 2) + bytes([3, 250]) + struct.pack("<Qf", 1, 0.5) + struct.pack("<Qf", 1, -1.0)
            + struct.pack("<II", 1, 0) + struct.pack("<QQQQ", 3, 1, 2, 1)
            # Some(ProjectionState { basis_vt, ranks, num_heads, head_dim, projected_shape }), None
            + b"\x01" + struct.pack("<Qf", 1, 1.0) + struct.pack("<QQ", 1, 1) + struct.pack("<QQ", 1, 1)
            + struct.pack("<QQQQ", 3, 1, 2, 1) + b"\x00"
            # value_data: ..., QuantAxis::PerToken, None, Some(EntropyState { [], 2 })
            + struct.pack("<Q", 2) + bytes([1, 2]) + struct.pack("<Qff", 2, 0.25, 2.0)
            + struct.pack("<Qff", 2, 0.0, 1.5) + struct.pack("<II", 1, 1) + struct.pack("<QQQQ", 3, 1, 2, 1)
            + b"\x00" + b"\x01" + struct.pack("<Q", 0) + struct.pack("<Q", 2)
            + struct.pack("<Q", 16))
    assert oracle.to_bincode(ckv) == want
    back = oracle.from_bincode(want)
    assert oracle.to_bincode(back) == want and back["layer_idx"] == 7


def test_bincode_roundtrip_of_compressed_layers(oracle):
    rng = np.random.default_rng(4)
    k = rng.standard_normal((2, 40, 16)).astype(np.float32)
    v = rng.standard_normal((2, 40, 16)).astype(np.float32)
    for preset in ("conservative", "balanced", "aggressive"):
        co = oracle.compress(k, v, preset, 3)
        b = oracle.to_bincode(co)
        back = oracle.from_bincode(b)
        assert oracle.to_bincode(back) == b
        assert oracle.compressed_size_bytes(back) == oracle.compressed_size_bytes(co)
        kr, vr = oracle.decompress(co)
        kb, vb = oracle.decompress(back)
        assert np.array_equal(kr, kb) and np.array_equal(vr, vb)
