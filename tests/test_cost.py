"""Cost model: the reference's CostModel arithmetic through the C ABI
(kvf_cost_estimate / kvf_cost_select are host code, so these run without a
GPU), checked with the reference's own table and the cases of its tests
(crates/kvforge-cpu/tests/cost_model.rs); then the GPU-measured table."""
import numpy as np
import pytest

CONSERVATIVE, BALANCED, AGGRESSIVE = 0, 1, 2
TIERS = range(6)

# CpuCostModel::new (crates/kvforge-cpu/src/cost.rs:26-50): the table the
# reference's tests run against
REFERENCE_ROWS = [
    dict(preset=CONSERVATIVE, compression_ratio=4.0, compress_us_per_byte=0.0005,
         decompress_us_per_byte=0.0003, quality=0.95),
    dict(preset=BALANCED, compression_ratio=12.0, compress_us_per_byte=0.002,
         decompress_us_per_byte=0.001, quality=0.80),
    dict(preset=AGGRESSIVE, compression_ratio=20.0, compress_us_per_byte=0.004,
         decompress_us_per_byte=0.002, quality=0.60),
]


@pytest.fixture(scope="module")
def K():
    import kvforge_b200
    return kvforge_b200


def test_bandwidth_tiers(K):
    assert [K.BandwidthTier.bytes_per_us(t) for t in TIERS] == [25000.0, 12500.0, 10000.0, 2500.0, 1000.0, 100.0]
    with pytest.raises(ValueError):
        K.BandwidthTier.bytes_per_us(6)


def test_reference_table_estimates(K):
    m = K.GpuCostModel(REFERENCE_ROWS)
    for p in (CONSERVATIVE, BALANCED, AGGRESSIVE):
        for t in TIERS:
            e = m.estimate(1_000_000, p, t)
            assert e.compress_us > 0 and e.transfer_us > 0 and e.decompress_us > 0
            assert abs(e.total_us - (e.compress_us + e.transfer_us + e.decompress_us)) < 1e-6
    e = m.estimate(1_000_000, CONSERVATIVE, K.BandwidthTier.ETHERNET_10G)
    assert e.compression_ratio == 4.0 and e.compress_us == 500.0 and e.transfer_us == 250.0
    assert m.estimate(1_000_000, "adaptive", 0).preset == CONSERVATIVE  # absent preset: first row


def test_reference_table_decisions(K):
    m = K.GpuCostModel(REFERENCE_ROWS)
    c = m.estimate(10_000_000, CONSERVATIVE, K.BandwidthTier.ETHERNET_10G)
    a = m.estimate(10_000_000, AGGRESSIVE, K.BandwidthTier.ETHERNET_10G)
    assert a.transfer_us < c.transfer_us
    assert m.select_codec(1_000_000, K.BandwidthTier.LOCAL)[0].preset == CONSERVATIVE
    assert all(e.preset == CONSERVATIVE for e in m.select_codec(1_000_000, K.BandwidthTier.WAN, 0.9))
    for t in (K.BandwidthTier.LOCAL, K.BandwidthTier.WAN, K.BandwidthTier.ETHERNET_10G):
        est = m.select_codec(5_000_000, t)
        assert len(est) == 3 and all(x.total_us <= y.total_us for x, y in zip(est, est[1:]))
    # cost.rs unit tests: on WAN all presets are ranked and Aggressive moves
    # fewer bytes; on the local bus Conservative wins
    wan = m.select_codec(10_000_000, K.BandwidthTier.WAN)
    by = {e.preset: e for e in wan}
    assert len(wan) == 3 and by[AGGRESSIVE].transfer_us < by[CONSERVATIVE].transfer_us
    assert m.select_codec(10_000_000, K.BandwidthTier.LOCAL)[0].preset == CONSERVATIVE
    # with the CPU table's costs the codec costs more than any transfer it saves:
    # Conservative is chosen on every tier
    assert all(m.select_preset(10_000_000, t) == "conservative" for t in TIERS)
    with pytest.raises(K.KvForgeError):
        m.select_preset(1_000_000, K.BandwidthTier.WAN, 0.99)


@pytest.mark.gpu
def test_measured_table(K):
    """Rows measured on the GPU: ratio equal to compressing the sample, costs
    positive, quality ordered by how lossy the preset is; with GPU costs the
    transfer term dominates on every tier, so the highest ratio allowed by the
    quality floor wins."""
    import torch
    from kvforge_b200 import synth
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    k, v = synth.workload_layer("llama3_8b_32k", 0, backend="torch", device="cuda", T=4096)
    kv = K.KVCache(k, v, 0)
    m = K.GpuCostModel.measure(kv, reps=3)
    rows = {r["preset"]: r for r in m.rows()}
    assert set(rows) == {"conservative", "balanced", "aggressive"}
    for name, r in rows.items():
        assert r["compress_us_per_byte"] > 0 and r["decompress_us_per_byte"] > 0
        assert 0.0 < r["quality"] <= 1.0
        assert r["compression_ratio"] == K.compress(kv, name).ratio()
    assert rows["conservative"]["quality"] > rows["balanced"]["quality"] > rows["aggressive"]["quality"]
    best = max(rows, key=lambda n: rows[n]["compression_ratio"])
    for t in TIERS:
        assert m.select_preset(kv.size_bytes(), t) == best
    floor = rows["conservative"]["quality"] - 1e-9
    c, preset = K.compress_adaptive(kv, m, K.BandwidthTier.WAN, floor)
    assert preset == "conservative" and c.ratio() == rows["conservative"]["compression_ratio"]
