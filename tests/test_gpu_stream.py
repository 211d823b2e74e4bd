"""GPU tests of streaming append (StreamingCompressor): a layer's prefix is
compressed once, then chunks of new tokens are compressed one at a time.

The reference compresses every chunk as its own KVCache with a fresh SVD
(crates/kvforge-cpu/src/pipeline.rs:100-163): reuse_basis=False. With
reuse_basis=True each chunk is projected onto the basis calibrated on the
prefix. Either way a chunk is a complete CompressedKV, so the oracle's
compress with the same basis must give the same codes, parameters, rANS
container and sizes bit for bit."""
import numpy as np
import pytest
import torch

from test_gpu_parity import REC_TOL, bits, dev, host, rel

pytestmark = pytest.mark.gpu


def _stream_layer(H, T, D, seed):
    from kvforge_b200 import synth
    return synth.numpy_layer(H, T, D, seed=seed, rank=24, dtype="float16")


def _check_chunk(kvf, oracle, c, k, v, preset, layer_idx, bases):
    co = oracle.compress(k.astype(np.float32), v.astype(np.float32), preset, layer_idx, bases, threads=4)
    for which, name in ((0, "key"), (1, "value")):
        parts = c.tensor_parts(which)
        ot = co[name]
        assert np.array_equal(host(parts["data"]), ot["data"]), name
        assert np.array_equal(bits(host(parts["scales"])), bits(ot["scales"])), name
        assert np.array_equal(bits(host(parts["mins"])), bits(ot["mins"])), name
        if ot["entropy"] is not None and ot["entropy"][1] > 0:
            assert np.array_equal(host(parts["freq"]).astype(np.uint32), ot["entropy"][0]), name
    assert c.compressed_size_bytes() == oracle.compressed_size_bytes(co)
    assert c.ratio() == oracle.ratio(co)
    kr, vr = oracle.decompress(co, threads=4)
    out = kvf.decompress(c)
    assert rel(out.keys(), kr) < REC_TOL and rel(out.values(), vr) < REC_TOL
    return co


def _basis_bytes(bases, D):
    return sum(int(vt.shape[0]) * int(vt.shape[1]) * D * 4 + int(vt.shape[0]) * 8 for vt, _ in bases)


@pytest.mark.parametrize("preset", ["balanced", "aggressive"])
def test_append_reuses_prefix_basis(kvf, oracle, preset):
    H, P, D = 4, 512, 128
    sizes = [64, 1, 63, 65, 130]
    k, v = _stream_layer(H, P + sum(sizes), D, seed=71)
    sc = kvf.StreamingCompressor(preset, reuse_basis=True)
    cp = sc.prefill(kvf.KVCache(dev(k[:, :P]), dev(v[:, :P]), 5))
    kb, vb = sc.bases(5)
    kh, vh = kb.host(), vb.host()
    # the kept bases are the prefix's own projection state, shared
    for which, (bvt, rk, _) in ((0, kh), (1, vh)):
        parts = cp.tensor_parts(which)
        assert np.array_equal(bits(host(parts["basis_vt"])), bits(bvt))
        assert np.array_equal(host(parts["ranks"]), rk)
    bases = ((kh[0], kh[1]), (vh[0], vh[1]))
    _check_chunk(kvf, oracle, cp, k[:, :P], v[:, :P], preset, 5, bases)
    t0 = P
    for n in sizes:
        kc, vc = k[:, t0:t0 + n], v[:, t0:t0 + n]
        t0 += n
        c = sc.append(kvf.KVCache(dev(kc), dev(vc), 5))
        assert c.shape == (H, n, D)
        _check_chunk(kvf, oracle, c, kc, vc, preset, 5, bases)
        assert c.basis_size_bytes() == _basis_bytes(bases, D)
        assert sc.amortized_size_bytes(c) == c.compressed_size_bytes() - c.basis_size_bytes()
        # the chunk carries the prefix's basis object itself
        assert c.basis(0).device_vt() == kb.device_vt() and c.basis(1).device_vt() == vb.device_vt()


def test_append_reference_mode_fresh_basis(kvf, oracle):
    """reuse_basis=False: every 64-token chunk gets its own basis, as the
    reference does; ranks follow select_rank on the chunk's own spectrum."""
    H, P, D = 4, 256, 128
    k, v = _stream_layer(H, P + 128, D, seed=72)
    sc = kvf.StreamingCompressor("balanced", reuse_basis=False)
    sc.prefill(kvf.KVCache(dev(k[:, :P]), dev(v[:, :P]), 0))
    assert sc.bases(0) is None
    thr = kvf.config_from_preset("balanced").projection_variance_threshold
    for t0 in (P, P + 64):
        kc, vc = k[:, t0:t0 + 64], v[:, t0:t0 + 64]
        c = sc.append(kvf.KVCache(dev(kc), dev(vc), 0))
        kh, vh = c.basis(0).host(), c.basis(1).host()
        for x, bh in ((kc, kh), (vc, vh)):
            _, rk = oracle.basis_for(x.astype(np.float32), thr, threads=4)
            assert np.array_equal(bh[1], rk)
        _check_chunk(kvf, oracle, c, kc, vc, "balanced", 0, ((kh[0], kh[1]), (vh[0], vh[1])))
        assert sc.amortized_size_bytes(c) == c.compressed_size_bytes()


def test_append_without_projection(kvf, oracle):
    H, D = 2, 64
    k, v = _stream_layer(H, 256 + 64, D, seed=73)
    sc = kvf.StreamingCompressor("conservative", reuse_basis=True)
    sc.prefill(kvf.KVCache(dev(k[:, :256]), dev(v[:, :256]), 1))
    assert sc.bases(1) is None
    c = sc.append(kvf.KVCache(dev(k[:, 256:]), dev(v[:, 256:]), 1))
    assert c.basis(0) is None and c.basis(1) is None and c.basis_size_bytes() == 0
    _check_chunk(kvf, oracle, c, k[:, 256:], v[:, 256:], "conservative", 1, None)


def test_append_before_prefill_is_rejected(kvf):
    sc = kvf.StreamingCompressor("balanced", reuse_basis=True)
    x = torch.zeros((2, 64, 128), device="cuda")
    with pytest.raises(kvf.KvForgeError):
        sc.append(kvf.KVCache(x, x, 9))


def test_append_shares_basis_across_many_chunks(kvf):
    """The prefix's basis outlives the prefix object and is reused by many
    chunks; the amortized ratio of a 64-token chunk beats the fresh-basis one."""
    H, P, D = 8, 2048, 128
    k, v = _stream_layer(H, P + 16 * 64, D, seed=74)
    reuse = kvf.StreamingCompressor("balanced", reuse_basis=True)
    fresh = kvf.StreamingCompressor("balanced", reuse_basis=False)
    cp = reuse.prefill(kvf.KVCache(dev(k[:, :P]), dev(v[:, :P]), 2))
    e_prefix = rel(reuse.decompress(cp).keys(), k[:, :P].astype(np.float32))
    del cp
    am, fr, errs = [], [], []
    for i in range(16):
        t0 = P + 64 * i
        kv = kvf.KVCache(dev(k[:, t0:t0 + 64]), dev(v[:, t0:t0 + 64]), 2)
        c = reuse.append(kv)
        am.append(c.original_size_bytes() / reuse.amortized_size_bytes(c))
        out = reuse.decompress(c)
        errs.append(rel(out.keys(), k[:, t0:t0 + 64].astype(np.float32)))
        f = fresh.append(kv)
        fr.append(f.ratio())
    assert min(am) > max(fr)
    # the data is stationary: chunks projected onto the prefix basis lose about
    # what the prefix itself loses
    assert max(errs) < 1.5 * e_prefix + 1e-3
