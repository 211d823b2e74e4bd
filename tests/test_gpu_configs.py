"""Parity at the benchmark workloads' stated shapes, through the C ABI.

- Conservative, one layer of keys and values f32 [32, 2048, 128] i.i.d.
  N(0, 1), seed 0 (the shape of the reference's README example,
  crates/kvforge-cpu/examples/basic_compress.rs);
- Balanced, f32 [32, 4096, 128], rank-32 signal (singular values 0.9^i) plus
  0.1 N(0, 1) noise, four key channels per head x10, seed 1;
- Aggressive, f16 [32, 8192, 128], the same generator, seed 2;
- the Llama-3-70B streaming layer: an f16 [8, 16384, 128] prefix compressed
  once (Balanced), then 64-token appends, with the prefix's basis and with a
  fresh basis per chunk (the reference's semantics, pipeline.rs:100-163).

Codes, scales, mins, rANS containers, sizes and ratio are bit-exact against
the CPU oracle on the same seeded inputs (numpy generator); reconstruction is
within REC_TOL of the oracle's, and bit-exact in the exact mode.
"""
import numpy as np
import pytest

from test_gpu_parity import REC_TOL, _pipeline_case, bits, dev, host, rel
from test_gpu_stream import _check_chunk

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["conservative_32x2048", "balanced_32x4096", "aggressive_32x8192"])
def test_workload_at_stated_shape(kvf, oracle, name):
    from kvforge_b200 import _lib as L
    from kvforge_b200 import synth
    w = synth.WORKLOADS[name]
    k, v = synth.workload_layer(name, 0, backend="numpy")
    assert k.shape == (w["H"], w["T"], w["D"]) and k.dtype == np.dtype(w["dtype"])
    c, co = _pipeline_case(kvf, oracle, k, v, w["preset"])
    kr, vr = oracle.decompress(co, threads=8)
    out = kvf.decompress(c)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    ctx = L.context(0)
    L.check(L.lib().kvf_set_exact_reconstruct(ctx, 1))
    try:
        out = kvf.decompress(c)
    finally:
        L.check(L.lib().kvf_set_exact_reconstruct(ctx, 0))
    assert np.array_equal(bits(out.keys()), bits(kr)) and np.array_equal(bits(out.values()), bits(vr))
    if name == "conservative_32x2048":
        # 2 x 8,388,608 INT8 codes + keys' 2 x 4096 and values' 2 x 65536 f32 parameters (types.rs:66-78)
        assert c.original_size_bytes() == 67108864 and c.compressed_size_bytes() == 17334272


@pytest.mark.parametrize("reuse", [True, False])
def test_llama3_70b_stream_layer(kvf, oracle, reuse):
    from kvforge_b200 import synth
    w = synth.WORKLOADS["llama3_70b_stream"]
    H, P, D, A = w["H"], w["T"], w["D"], w["append"]
    n_app = 3
    k, v = synth.workload_layer("llama3_70b_stream", 0, backend="numpy", T=P + n_app * A)
    sc = kvf.StreamingCompressor(w["preset"], reuse_basis=reuse)
    cp = sc.prefill(kvf.KVCache(dev(k[:, :P]), dev(v[:, :P]), 0))
    if reuse:
        kb, vb = sc.bases(0)
    else:
        kb, vb = cp.basis(0), cp.basis(1)
    kh, vh = kb.host(), vb.host()
    _check_chunk(kvf, oracle, cp, k[:, :P], v[:, :P], w["preset"], 0, ((kh[0], kh[1]), (vh[0], vh[1])))
    for i in range(n_app):
        t0 = P + i * A
        kc, vc = k[:, t0:t0 + A], v[:, t0:t0 + A]
        c = sc.append(kvf.KVCache(dev(kc), dev(vc), 0))
        if not reuse:
            kh, vh = c.basis(0).host(), c.basis(1).host()
        _check_chunk(kvf, oracle, c, kc, vc, w["preset"], 0, ((kh[0], kh[1]), (vh[0], vh[1])))
        out = sc.decompress(c)
        assert rel(out.keys(), kc.astype(np.float32)) < 0.5
