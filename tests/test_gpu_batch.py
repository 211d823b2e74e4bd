"""Many layers in one call (kvf_compress_layers) against the per-layer path.

The batched entry point must give, for every layer, what kvf_compress_layer
gives for that layer alone: the serialized objects (codes, scales, mins,
bases, sizes) are compared byte for byte, and the decompressed chunks bit for
bit against kvf_decompress_layer on the CUDA-core reconstruction engine (and
in the exact mode, which the oracle matches bit for bit). Cases: the
streaming append of a Llama-3-70B-shaped cache (8 heads, 64-token chunks,
Balanced, each layer on its own prefix basis), no projection (Conservative),
f16 and f32 inputs, single tokens, odd widths (one head), INT8 codes with
projection, more layers than one launch takes, and configurations the batched
kernel does not take (entropy coding, long chunks), which run the per-layer
path inside the same call."""
import ctypes as C

import numpy as np
import pytest
import torch

from test_gpu_parity import bits, dev, host
from test_gpu_stream import _check_chunk

pytestmark = pytest.mark.gpu


def _layers(H, T, D, n, seed, f16=True):
    from kvforge_b200 import synth
    out = []
    for i in range(n):
        k, v = synth.numpy_layer(H, T, D, seed=seed + i, rank=24, dtype="float16" if f16 else "float32")
        out.append((k, v))
    return out


def _recon_engine(L, engine):
    L.check(L.lib().kvf_set_reconstruct_engine(L.context(0), engine))


def _exact(L, on):
    L.check(L.lib().kvf_set_exact_reconstruct(L.context(0), 1 if on else 0))


def _compare(kvf, cfg, chunks, kbs, vbs, layer_ids=None):
    """Batched call vs one kvf_compress_layer per layer: serialized bytes and
    decompressed chunks (CUDA-core engine, fused and exact)."""
    from kvforge_b200 import _lib as L
    pipe = kvf.CompressionPipeline()
    ids = layer_ids or list(range(len(chunks)))
    kvs = [kvf.KVCache(dev(k), dev(v), i) for (k, v), i in zip(chunks, ids)]
    _recon_engine(L, L.RECON_CUDA_CORE)
    try:
        for exact in (False, True):
            _exact(L, exact)
            cs, outs = pipe.compress_layers(kvs, cfg, kbs, vbs, decompress=True)
            assert len(cs) == len(kvs)
            for i, kv in enumerate(kvs):
                ref = pipe.compress_with_config(kv, cfg, kbs[i] if kbs else None, vbs[i] if vbs else None)
                assert cs[i].layer_idx == ids[i]
                assert cs[i].to_bytes() == ref.to_bytes(), i
                assert cs[i].compressed_size_bytes() == ref.compressed_size_bytes()
                r = pipe.decompress(ref)
                assert np.array_equal(bits(outs[i].keys()), bits(r.keys())), (i, exact)
                assert np.array_equal(bits(outs[i].values()), bits(r.values())), (i, exact)
                # the batched object decompresses like any other
                r2 = pipe.decompress(cs[i])
                assert np.array_equal(bits(r2.keys()), bits(r.keys())), (i, exact)
    finally:
        _exact(L, False)
        _recon_engine(L, L.RECON_AUTO)
    return cs


def _prefix_bases(kvf, H, P, D, n, seed, f16=True, preset="balanced"):
    pipe = kvf.CompressionPipeline()
    cfg = kvf.config_from_preset(preset)
    kbs, vbs, hosts = [], [], []
    for i, (k, v) in enumerate(_layers(H, P, D, n, seed, f16)):
        c = pipe.compress_with_config(kvf.KVCache(dev(k), dev(v), i), cfg)
        kbs.append(c.basis(0))
        vbs.append(c.basis(1))
    return kbs, vbs


@pytest.mark.parametrize("T", [64, 1, 17, 128])
def test_batched_streaming_append_balanced(kvf, T):
    H, D, n = 8, 128, 6
    kbs, vbs = _prefix_bases(kvf, H, 512, D, n, seed=300)
    _compare(kvf, kvf.config_from_preset("balanced"), _layers(H, T, D, n, seed=400 + T), kbs, vbs,
             layer_ids=[10 + i for i in range(n)])


@pytest.mark.parametrize("f16", [True, False])
@pytest.mark.parametrize("T", [64, 3])
def test_batched_without_projection(kvf, f16, T):
    _compare(kvf, kvf.config_from_preset("conservative"), _layers(4, T, 128, 5, seed=500 + T, f16=f16), None, None)


def test_batched_f32_odd_width_one_head(kvf):
    """One head with an odd T * R: INT4 pairs run across rows."""
    kbs, vbs = _prefix_bases(kvf, 1, 256, 64, 3, seed=600, f16=False)
    chunks = _layers(1, 33, 64, 3, seed=700, f16=False)
    _compare(kvf, kvf.config_from_preset("balanced"), chunks, kbs, vbs)


def test_batched_int8_projection(kvf):
    from kvforge_b200 import _lib as L
    cfg = kvf.config_from_preset("balanced")
    cfg.key_data_type = L.INT8
    cfg.value_data_type = L.INT8
    kbs, vbs = _prefix_bases(kvf, 2, 256, 128, 4, seed=800)
    _compare(kvf, cfg, _layers(2, 40, 128, 4, seed=900), kbs, vbs)


def test_batched_many_layers(kvf):
    """More layers than one launch takes (groups of 128)."""
    _compare(kvf, kvf.config_from_preset("conservative"), _layers(2, 4, 32, 130, seed=1000), None, None)


@pytest.mark.parametrize("case", ["entropy", "long_chunk", "fresh_basis"])
def test_batched_falls_back_to_per_layer(kvf, case):
    H, D = 4, 128
    if case == "entropy":
        kbs, vbs = _prefix_bases(kvf, H, 512, D, 3, seed=1100, preset="aggressive")
        _compare(kvf, kvf.config_from_preset("aggressive"), _layers(H, 64, D, 3, seed=1200), kbs, vbs)
    elif case == "long_chunk":
        kbs, vbs = _prefix_bases(kvf, H, 512, D, 2, seed=1300)
        _compare(kvf, kvf.config_from_preset("balanced"), _layers(H, 300, D, 2, seed=1400), kbs, vbs)
    else:  # no bases given: each chunk gets its own (the reference's semantics)
        from kvforge_b200 import _lib as L
        pipe = kvf.CompressionPipeline()
        chunks = _layers(H, 96, D, 2, seed=1500)
        cs = pipe.compress_layers([kvf.KVCache(dev(k), dev(v), i) for i, (k, v) in enumerate(chunks)], "balanced")
        for i, (k, v) in enumerate(chunks):
            ref = pipe.compress(kvf.KVCache(dev(k), dev(v), i), "balanced")
            assert cs[i].to_bytes() == ref.to_bytes()


def test_batched_streaming_append_against_oracle(kvf, oracle):
    """Batched appends of a Llama-3-70B-shaped layer stack (8 heads, 64-token
    chunks, Balanced, each layer's own prefix basis) through
    StreamingCompressor.append_layers, against the oracle's compress of each
    chunk with the same basis: codes, scales, mins, sizes and ratio bit for
    bit."""
    H, P, D, A, n = 8, 512, 128, 64, 4
    sc = kvf.StreamingCompressor("balanced", reuse_basis=True)
    data = _layers(H, P + A, D, n, seed=1600)
    for i, (k, v) in enumerate(data):
        sc.prefill(kvf.KVCache(dev(k[:, :P]), dev(v[:, :P]), i))
    cs, outs = sc.append_layers([kvf.KVCache(dev(k[:, P:]), dev(v[:, P:]), i) for i, (k, v) in enumerate(data)],
                                decompress=True)
    for i, (k, v) in enumerate(data):
        kb, vb = sc.bases(i)
        kh, vh = kb.host(), vb.host()
        _check_chunk(kvf, oracle, cs[i], k[:, P:], v[:, P:], "balanced", i, ((kh[0], kh[1]), (vh[0], vh[1])))
        assert outs[i].keys().shape == (H, A, D)


def test_batched_objects_free_in_any_order(kvf):
    """The objects of one call share one device block: freeing some leaves the
    others intact, on any stream."""
    from kvforge_b200 import _lib as L
    H, T, D, n = 4, 32, 128, 5
    kbs, vbs = _prefix_bases(kvf, H, 256, D, n, seed=1700)
    pipe = kvf.CompressionPipeline()
    chunks = _layers(H, T, D, n, seed=1800)
    kvs = [kvf.KVCache(dev(k), dev(v), i) for i, (k, v) in enumerate(chunks)]
    cs = pipe.compress_layers(kvs, "balanced", kbs, vbs)
    want = [c.to_bytes() for c in cs]
    ref = [pipe.decompress(c) for c in cs]
    for i in (3, 0, 4):
        L.check(L.lib().kvf_compressed_free(cs[i].handle))
        cs[i]._h = None
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in (1, 2):
            assert cs[i].to_bytes() == want[i]
            out = pipe.decompress(cs[i])
            assert np.array_equal(bits(out.values()), bits(ref[i].values()))
    torch.cuda.synchronize()


def test_batched_argument_errors(kvf):
    from kvforge_b200 import _lib as L
    lib, ctx = L.lib(), L.context(0)
    cfg = kvf.config_from_preset("balanced")
    out = (C.c_void_p * 1)()
    x = torch.zeros((1, 4, 8), dtype=torch.float16, device="cuda")
    P = (C.c_void_p * 1)(x.data_ptr())
    # keys_out without values_out
    assert lib.kvf_compress_layers(ctx, 1, P, P, L.IN_F16, 1, 4, 8, None, C.byref(cfg), None, None, out,
                                   P, None, None) == L.ERR_INVALID_CONFIG
    assert lib.kvf_compress_layers(ctx, 1, P, P, 7, 1, 4, 8, None, C.byref(cfg), None, None, out, None, None,
                                   None) == L.ERR_INVALID_CONFIG
    # zero layers: nothing to do
    assert lib.kvf_compress_layers(ctx, 0, None, None, L.IN_F16, 1, 4, 8, None, C.byref(cfg), None, None, out,
                                   None, None, None) == L.OK
