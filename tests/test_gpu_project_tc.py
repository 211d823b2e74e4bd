"""The tensor-core projection engine against the CUDA-core chain and the oracle.

kvf_fused_project_quantize with per-token quantization runs on tcgen05 by
default (f16 input, head_dim 128, R <= 64) and on CUDA cores with
kvf_set_projection_engine(CUDA_CORE). Both must give the oracle's codes,
scales and mins bit for bit: the oracle projects with one fmaf chain per
coefficient (crates/kvforge-cpu/src/projection.rs:61-140 as restated in
oracle/kvforge_oracle.c) and quantizes per token (quantize.rs:102-130).

Cases: ranks 1 to 64 with odd and even R, heads of lower rank than R, token
counts that are not multiples of the 128-token tile, INT4 and INT8, rows of
zeros, rows whose coefficients are all nearly equal (every coefficient is a
candidate for the row's minimum and maximum), rows at the f16 maximum,
subnormal rows, and rows with inf / NaN (every coefficient recomputed)."""
import ctypes as C

import numpy as np
import pytest
import torch

from test_gpu_parity import bits, dev, host

pytestmark = pytest.mark.gpu

INT4, INT8 = 0, 1
PT = 1


def _run(kvf, x16, bvt, ranks, R, dt, engine):
    from kvforge_b200 import _lib as L
    lib, ctx = L.lib(), L.context(0)
    H, T, D = x16.shape
    basis = kvf.Basis.from_host(bvt, ranks)
    n = H * T * R
    plen = (n + 1) // 2 if dt == INT4 else n
    packed = torch.zeros(plen, dtype=torch.uint8, device="cuda")
    sc = torch.zeros(H * T, dtype=torch.float32, device="cuda")
    mn = torch.zeros(H * T, dtype=torch.float32, device="cuda")
    xd = dev(x16)
    L.check(lib.kvf_set_projection_engine(ctx, engine))
    try:
        L.check(lib.kvf_fused_project_quantize(ctx, C.c_void_p(xd.data_ptr()), L.IN_F16, H, T, D,
                                               C.c_void_p(basis.device_vt()), C.c_void_p(basis.device_ranks()), R,
                                               dt, PT, C.c_void_p(packed.data_ptr()), C.c_void_p(sc.data_ptr()),
                                               C.c_void_p(mn.data_ptr()), None))
        L.check(lib.kvf_sync(ctx, None))
    finally:
        L.check(lib.kvf_set_projection_engine(ctx, L.PROJ_AUTO))
    return host(packed), host(sc), host(mn)


def _basis(rng, H, R, D, ranks):
    bvt = np.zeros((H, R, D), np.float32)
    for h in range(H):
        q = np.linalg.qr(rng.standard_normal((D, R)))[0].T.astype(np.float32)
        bvt[h, : ranks[h]] = q[: ranks[h]]
    return bvt


def _check(kvf, oracle, x16, bvt, ranks, R, dt):
    from kvforge_b200 import _lib as L
    x32 = x16.astype(np.float32)
    P = oracle.project(x32, bvt, ranks, threads=8)
    p, s, m = oracle.quantize(P, dt, PT)
    for engine in (L.PROJ_TENSOR_CORE, L.PROJ_CUDA_CORE):
        gp, gs, gm = _run(kvf, x16, bvt, ranks, R, dt, engine)
        assert np.array_equal(gp, p), engine
        assert np.array_equal(bits(gs), bits(s)), engine
        assert np.array_equal(bits(gm), bits(m)), engine


@pytest.mark.parametrize("R", [1, 3, 8, 9, 12, 16, 17, 24, 32, 33, 48, 58, 64])
@pytest.mark.parametrize("dt", [INT4, INT8])
@pytest.mark.parametrize("T", [1000, 999])
def test_tensor_core_projection_codes(kvf, oracle, R, dt, T):
    """Odd R with even T packs INT4 pairs across rows inside the kernel; odd R
    with odd T writes unpacked codes for a separate packing pass."""
    rng = np.random.default_rng(1000 + R + 7 * dt + T)
    H, D = 3, 128
    ranks = np.array([R, max(1, R - 3), max(1, R // 2)], np.uint64)
    bvt = _basis(rng, H, R, D, ranks)
    # low-rank rows in the basis's span plus noise, so coefficients spread widely
    coef = rng.standard_normal((H, T, R)).astype(np.float32) * (0.9 ** np.arange(R, dtype=np.float32))
    x = np.einsum("htr,hrd->htd", coef, bvt) + 0.05 * rng.standard_normal((H, T, D))
    _check(kvf, oracle, x.astype(np.float16), bvt, ranks, R, dt)


def test_tensor_core_projection_edge_rows(kvf, oracle):
    rng = np.random.default_rng(77)
    H, T, D, R = 2, 384, 128, 12
    ranks = np.array([R, R], np.uint64)
    bvt = _basis(rng, H, R, D, ranks)
    x = rng.standard_normal((H, T, D)).astype(np.float32)
    x[0, 0] = 0.0                                   # zero row: range 0, scale 1
    x[0, 1] = 1.0                                   # constant row
    x[0, 2] = np.float32(65504.0)                   # f16 maximum
    x[0, 3] = -65504.0
    x[0, 4] = np.float32(6e-8)                      # f16 subnormals
    x[0, 5, 7] = np.inf                             # non-finite rows: every coefficient exact
    x[0, 6, 3] = np.nan
    x[0, 7, 0] = -np.inf
    x[0, 8] = rng.standard_normal(D) * 30000.0
    # rows whose coefficients nearly tie: x along the sum of the basis rows
    s = bvt[1].sum(axis=0)
    for t in range(16, 64):
        x[1, t] = s * np.float32(rng.uniform(0.1, 10.0)) + 1e-4 * rng.standard_normal(D)
    x16 = np.clip(x, -65504, 65504).astype(np.float16)
    x16[0, 5, 7], x16[0, 6, 3], x16[0, 7, 0] = np.inf, np.nan, -np.inf
    for dt in (INT4, INT8):
        _check(kvf, oracle, x16, bvt, ranks, R, dt)


def test_tensor_core_projection_large_layer(kvf, oracle):
    """A Llama-3-8B-shaped value tensor ([8, 32768, 128] f16, the benchmark's
    generator) at the basis the pipeline calibrates: over 2 M token rows, so
    the rare exact recomputations (ties for a row's minimum or maximum, codes
    near a rounding boundary) all occur many times."""
    from kvforge_b200 import synth
    _, v = synth.workload_layer("llama3_8b_32k", 0, backend="torch")
    cfg = kvf.config_from_preset("aggressive")
    vb = kvf.Basis.compute(v, cfg.projection_variance_threshold)
    bvt, ranks, _ = vb.host()
    _check(kvf, oracle, host(v), bvt, ranks, bvt.shape[1], INT4)


@pytest.mark.parametrize("R", [3, 12, 17, 33, 58])
def test_tensor_core_projection_approx_engine(kvf, oracle, R):
    """KVF_PROJ_TENSOR_CORE_APPROX quantizes the tensor-core coefficients
    directly. Tolerances (against the oracle's quantization of its own exact
    coefficients): at most 0.5 % of codes differ and none by more than one
    level; a row's scale and min within 1e-5 of the norm of the row's input
    (divided by the levels for the scale) -- a tensor-core coefficient's error
    scales with sum |x_c v_c| <= ||x||, not with the coefficient -- and the
    dequantized rows within relative Frobenius error 2e-2 (the tensor-core
    bar) of the oracle's."""
    from kvforge_b200 import _lib as L
    rng = np.random.default_rng(2000 + R)
    H, T, D = 3, 1000, 128
    ranks = np.array([R, max(1, R - 3), max(1, R // 2)], np.uint64)
    bvt = _basis(rng, H, R, D, ranks)
    coef = rng.standard_normal((H, T, R)).astype(np.float32) * (0.9 ** np.arange(R, dtype=np.float32))
    x16 = (np.einsum("htr,hrd->htd", coef, bvt) + 0.05 * rng.standard_normal((H, T, D))).astype(np.float16)
    P = oracle.project(x16.astype(np.float32), bvt, ranks, threads=8)
    for dt in (INT4, INT8):
        p, s, m = oracle.quantize(P, dt, PT)
        gp, gs, gm = _run(kvf, x16, bvt, ranks, R, dt, L.PROJ_TENSOR_CORE_APPROX)
        if dt == INT4 and R % 2 == 0:
            a = np.stack([gp & 0xF, gp >> 4], -1).reshape(-1).astype(np.int16)
            b = np.stack([p & 0xF, p >> 4], -1).reshape(-1).astype(np.int16)
        else:
            if dt == INT4:  # odd R: unpack over the flat index
                a = np.stack([gp & 0xF, gp >> 4], -1).reshape(-1)[: H * T * R].astype(np.int16)
                b = np.stack([p & 0xF, p >> 4], -1).reshape(-1)[: H * T * R].astype(np.int16)
            else:
                a, b = gp.astype(np.int16), p.astype(np.int16)
        d = np.abs(a - b)
        assert d.max() <= 1 and (d > 0).mean() < 5e-3, (d.max(), (d > 0).mean())
        levels = 15.0 if dt == INT4 else 255.0
        xn = np.linalg.norm(x16.astype(np.float64).reshape(H * T, D), axis=1)
        es = np.abs(gs.astype(np.float64) - s) / (xn / levels + 1e-30)
        em = np.abs(gm.astype(np.float64) - m) / (xn + 1e-30)
        assert es.max() < 1e-5 and em.max() < 1e-5, (es.max(), em.max())
        deq_g = a.reshape(H * T, R) * gs[:, None] + gm[:, None]
        deq_o = b.reshape(H * T, R) * s[:, None] + m[:, None]
        assert np.linalg.norm(deq_g - deq_o) / np.linalg.norm(deq_o) < 2e-2
