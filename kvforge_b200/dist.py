"""Layer sharding across the GPUs of one node, and the statistics gather.

Each compressed layer is independent (crates/kvforge-core/src/types.rs:37-43),
so the codec path shards by layer with no collective. The only communication
is an all-gather of a few dozen bytes of per-rank statistics (compressed bytes,
squared error, reference energy, times), over NCCL on GPUs or gloo on CPUs.
"""
from __future__ import annotations

STAT_KEYS = ("layers", "input_bytes", "compressed_bytes", "original_bytes", "err2_k", "ref2_k", "err2_v",
             "ref2_v", "ms", "compress_ms", "decompress_ms", "ent_kvr2", "ent_single", "ent_shannon")
TIME_KEYS = ("ms", "compress_ms", "decompress_ms")


def layer_shard(num_layers: int, world_size: int, rank: int) -> range:
    """Contiguous block of layers for `rank`; the first num_layers % world_size
    ranks take one extra layer."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("bad world_size / rank")
    base, extra = divmod(num_layers, world_size)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_stats(stats: dict, device=None, group=None) -> list:
    """All-gather one float64 vector of STAT_KEYS per rank -> list of dicts
    (rank order). Works on any initialised process group (nccl or gloo)."""
    import torch
    import torch.distributed as dist

    vec = torch.tensor([float(stats.get(k, 0.0)) for k in STAT_KEYS], dtype=torch.float64,
                       device=device if device is not None else "cpu")
    if not (dist.is_available() and dist.is_initialized()):
        return [dict(zip(STAT_KEYS, vec.tolist()))]
    out = [torch.empty_like(vec) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, vec, group=group)
    return [dict(zip(STAT_KEYS, t.cpu().tolist())) for t in out]


def reduce_stats(per_rank: list) -> dict:
    """Sums over ranks; times are the max (the slowest rank bounds the job)."""
    tot = {k: 0.0 for k in STAT_KEYS}
    for s in per_rank:
        for k in STAT_KEYS:
            tot[k] = max(tot[k], s[k]) if k in TIME_KEYS else tot[k] + s[k]
    return tot
