"""GPU tests of fused dequantize + decode attention: one query row per head
against the compressed cache, softmax(scale * K_h q_h) V_h, computed on the
codes (KernelLauncher::fused_dequant_attention, kernel_launcher.rs:43-57; an
empty stub in the reference, kernels/fused_dequant_attention.cu:1-53).

The oracle evaluates the same formula in fp64 on the oracle's own
dequantized and reconstructed K and V (the reference's loops). The kernel
works in the basis's coordinates and sums in f32, so the bar is a relative
Frobenius error below ATTN_TOL = 1e-4 of the output (on a full Llama-3-8B
layer the error against fp64 attention is 2.3e-7)."""
import ctypes as C

import numpy as np
import pytest
import torch

from test_gpu_parity import dev, host, rel

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-4
INT4, INT8 = 0, 1
PC, PT = 0, 1


def _query(H, D, seed):
    return np.random.default_rng(seed).standard_normal((H, D)).astype(np.float32)


def _compressed(kvf, oracle, k, v, preset):
    cfg = kvf.config_from_preset(preset)
    kb = vb = bases = None
    if cfg.enable_projection:
        kb = kvf.Basis.compute(dev(k), cfg.projection_variance_threshold)
        vb = kvf.Basis.compute(dev(v), cfg.projection_variance_threshold)
        kh, vh = kb.host(), vb.host()
        bases = ((kh[0], kh[1]), (vh[0], vh[1]))
    c = kvf.CompressionPipeline().compress(kvf.KVCache(dev(k), dev(v), 0), preset, kb, vb)
    co = oracle.compress(k.astype(np.float32), v.astype(np.float32), preset, 0, bases, threads=4)
    return c, co


@pytest.mark.parametrize("preset", ["conservative", "balanced", "aggressive", "adaptive"])
@pytest.mark.parametrize("shape,f16", [((4, 128, 32), False), ((3, 257, 128), True), ((2, 1, 64), False),
                                       ((2, 1000, 64), True), ((1, 129, 128), False)])
@pytest.mark.parametrize("scale", [None, 1.0])
def test_compressed_attention_parity(kvf, oracle, preset, shape, f16, scale):
    from kvforge_b200 import synth
    H, T, D = shape
    k, v = synth.numpy_layer(H, T, D, seed=hash((preset, shape)) % 997, rank=min(12, D),
                             dtype="float16" if f16 else "float32")
    c, co = _compressed(kvf, oracle, k, v, preset)
    kr, vr = oracle.decompress(co, threads=4)
    q = _query(H, D, T)
    sc = scale if scale is not None else 1.0 / np.sqrt(D)
    ref = oracle.decode_attention(kr, vr, q, sc)
    out = host(c.attention(dev(q), scale))
    assert out.shape == (H, D)
    assert rel(out, ref) < ATTN_TOL, (preset, shape, rel(out, ref))


def _raw_call(kvf, kc, vc, q, ks, km, vs, vm, kdt, vdt, H, T, D, Rk, Rv, kb=None, vb=None, scale=0.125):
    from kvforge_b200 import _lib as L
    out = torch.empty((H, D), dtype=torch.float32, device="cuda")
    p = lambda t: C.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    L.check(L.lib().kvf_fused_dequant_attention(
        L.context(0), p(kc), p(vc), p(q), p(ks), p(km), p(vs), p(vm), kdt, vdt, H, T, D, Rk, Rv,
        p(kb[0]) if kb else None, p(kb[1]) if kb else None, p(vb[0]) if vb else None, p(vb[1]) if vb else None,
        scale, p(out), C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    return host(out)


@pytest.mark.parametrize("kdt,vdt", [(INT8, INT4), (INT4, INT8), (INT4, INT4), (INT8, INT8)])
@pytest.mark.parametrize("projected", [False, True])
def test_fused_attention_on_codes(kvf, oracle, kdt, vdt, projected):
    """The stage entry point on codes and parameters made by the oracle's
    quantizer, with and without a basis (ranks below R in some heads)."""
    from kvforge_b200 import synth
    H, T, D = 3, 300, 64
    k, v = synth.numpy_layer(H, T, D, seed=11, rank=10)
    q = _query(H, D, 5)
    kb = vb = None
    if projected:
        bases = []
        for x in (k, v):
            bvt, rk = oracle.basis_for(x, 0.9)
            rk[0] = max(1, int(rk[0]) - 2)  # a head whose rank is below the width
            bvt[0, int(rk[0]):] = 0.0
            bases.append((bvt, rk))
        (kbv, krk), (vbv, vrk) = bases
        kx, vx = oracle.project(k, kbv, krk), oracle.project(v, vbv, vrk)
        kb = (dev(kbv), dev(krk.astype(np.int64)))  # same bits as the u64 ranks
        vb = (dev(vbv), dev(vrk.astype(np.int64)))
    else:
        kx, vx = k, v
    Rk, Rv = kx.shape[2], vx.shape[2]
    kp, ks, km = oracle.quantize(kx, kdt, PC)
    vp, vs, vm = oracle.quantize(vx, vdt, PT)
    kd = oracle.dequantize(kp, ks, km, kdt, PC, kx.shape)
    vd = oracle.dequantize(vp, vs, vm, vdt, PT, vx.shape)
    if projected:
        kd = oracle.reconstruct(kd, kbv, krk)
        vd = oracle.reconstruct(vd, vbv, vrk)
    ref = oracle.decode_attention(kd, vd, q, 0.125)
    out = _raw_call(kvf, dev(kp), dev(vp), dev(q), dev(ks), dev(km), dev(vs), dev(vm), kdt, vdt, H, T, D, Rk, Rv,
                    kb, vb)
    assert rel(out, ref) < ATTN_TOL


def test_attention_empty_sequence_writes_zeros(kvf):
    H, D = 2, 32
    q = torch.ones((H, D), device="cuda")
    out = _raw_call(kvf, None, None, q, None, None, None, None, INT8, INT4, H, 0, D, D, D)
    assert np.array_equal(out, np.zeros((H, D), np.float32))


def test_attention_rejects_bad_arguments(kvf):
    from kvforge_b200 import _lib as L
    H, T, D = 2, 16, 32
    b = torch.zeros(H * T * D, dtype=torch.uint8, device="cuda")
    f = torch.zeros(H * T * D, dtype=torch.float32, device="cuda")
    with pytest.raises(kvf.KvForgeError):  # F32 is not a code type
        _raw_call(kvf, b, b, f, f, f, f, f, 2, INT4, H, T, D, D, D)
    with pytest.raises(kvf.KvForgeError):  # without a basis the width is head_dim
        _raw_call(kvf, b, b, f, f, f, f, f, INT8, INT4, H, T, D, 8, D)
    assert L.lib().kvf_compressed_attention(L.context(0), None, None, 1.0, None, None) != 0


def test_attention_full_size_llama_layer(kvf):
    """Llama-3-8B layer [8, 32768, 128] fp16, Aggressive preset: attention on
    the codes equals attention on the decompressed layer (exact reconstruction)."""
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    k, v = synth.workload_layer("llama3_8b_32k", 0, backend="torch", device="cuda")
    cfg = kvf.config_from_preset("aggressive")
    kb = kvf.Basis.compute(k, cfg.projection_variance_threshold)
    vb = kvf.Basis.compute(v, cfg.projection_variance_threshold)
    c = kvf.CompressionPipeline().compress(kvf.KVCache(k, v, 0), "aggressive", kb, vb)
    q = torch.randn((8, 128), generator=torch.Generator(device="cuda").manual_seed(3), device="cuda")
    out = host(c.attention(q))
    ctx = L.context(0)
    L.check(L.lib().kvf_set_exact_reconstruct(ctx, 1))
    try:
        d = kvf.decompress(c)
    finally:
        L.check(L.lib().kvf_set_exact_reconstruct(ctx, 0))
    kd, vd = d.keys_tensor.double(), d.values_tensor.double()
    s = torch.einsum("htd,hd->ht", kd, q.double()) / np.sqrt(128)
    ref = torch.einsum("ht,htd->hd", torch.softmax(s, dim=1), vd).cpu().numpy()
    assert rel(out, ref) < ATTN_TOL
