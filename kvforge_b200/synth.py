"""Seeded synthetic KV caches with the shapes and value distributions of the
benchmark workloads (no real KV traces ship with the reference; its own tests
use U(-1, 1) noise only).

Low-rank generator, per head and per tensor:
    X = U(T x r) . diag(0.9^i) . V(r x D) + noise * N(0, 1)
with U ~ N(0, 1), V the orthonormal rows of a QR of an N(0, 1) matrix; keys
additionally get 4 distinct channels per head scaled by `outlier` (a fixed
factor, or U[lo, hi] per channel). Two back ends draw from different RNGs:
numpy (exact, for tests and fixtures) and torch on the GPU (fast, for the
multi-GB benchmark workload).
"""
from __future__ import annotations

import numpy as np

WORKLOADS = {
    # name: (preset, H, T, D, dtype, generator args)
    "conservative_32x2048": dict(preset="conservative", H=32, T=2048, D=128, dtype="float32", gen="iid", seed=0),
    "balanced_32x4096": dict(preset="balanced", H=32, T=4096, D=128, dtype="float32", gen="lowrank", rank=32,
                             noise=0.1, outlier=10.0, seed=1),
    "aggressive_32x8192": dict(preset="aggressive", H=32, T=8192, D=128, dtype="float16", gen="lowrank", rank=32,
                               noise=0.1, outlier=10.0, seed=2),
    "llama3_8b_32k": dict(preset="aggressive", H=8, T=32768, D=128, dtype="float16", gen="lowrank", rank=24,
                          noise=0.1, outlier=(8.0, 16.0), seed=100, layers=32),
    "llama3_70b_stream": dict(preset="balanced", H=8, T=16384, D=128, dtype="float16", gen="lowrank", rank=24,
                              noise=0.1, outlier=(8.0, 16.0), seed=7, layers=80, append=64, appends=256),
}


def _np_tensor(rng, H, T, D, rank, noise, outlier):
    x = np.empty((H, T, D), np.float32)
    s = 0.9 ** np.arange(rank)
    for h in range(H):
        U = rng.standard_normal((T, rank))
        V = np.linalg.qr(rng.standard_normal((D, rank)))[0].T
        x[h] = ((U * s) @ V + noise * rng.standard_normal((T, D))).astype(np.float32)
        if outlier is not None:
            ch = rng.choice(D, size=min(4, D), replace=False)
            f = np.full(len(ch), outlier) if np.isscalar(outlier) else rng.uniform(outlier[0], outlier[1], len(ch))
            x[h][:, ch] *= f.astype(np.float32)
    return x


def numpy_layer(H, T, D, seed, gen="lowrank", rank=24, noise=0.1, outlier=(8.0, 16.0), dtype="float32"):
    """-> (keys, values) numpy arrays of `dtype`."""
    rng = np.random.default_rng(seed)
    if gen == "iid":
        k = rng.standard_normal((H, T, D)).astype(np.float32)
        v = rng.standard_normal((H, T, D)).astype(np.float32)
    else:
        k = _np_tensor(rng, H, T, D, rank, noise, outlier)
        v = _np_tensor(rng, H, T, D, rank, noise, None)
    return k.astype(dtype), v.astype(dtype)


def torch_layer(H, T, D, seed, gen="lowrank", rank=24, noise=0.1, outlier=(8.0, 16.0), dtype="float16",
                device="cuda"):
    """-> (keys, values) torch tensors on `device`, drawn with a seeded torch generator."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    tdt = getattr(torch, dtype)

    def one(with_outliers):
        if gen == "iid":
            return torch.randn((H, T, D), generator=g, device=device, dtype=torch.float32).to(tdt)
        U = torch.randn((H, T, rank), generator=g, device=device)
        V = torch.linalg.qr(torch.randn((H, D, rank), generator=g, device=device))[0].transpose(1, 2)
        s = 0.9 ** torch.arange(rank, device=device, dtype=torch.float32)
        x = torch.bmm(U * s, V)
        x += noise * torch.randn((H, T, D), generator=g, device=device)
        if with_outliers and outlier is not None:
            ch = torch.argsort(torch.rand((H, D), generator=g, device=device), dim=1)[:, :4]
            if isinstance(outlier, (int, float)):
                f = torch.full((H, 4), float(outlier), device=device)
            else:
                f = outlier[0] + (outlier[1] - outlier[0]) * torch.rand((H, 4), generator=g, device=device)
            scale = torch.ones((H, D), device=device)
            scale.scatter_(1, ch, f)
            x *= scale[:, None, :]
        return x.to(tdt).contiguous()

    return one(True), one(False)


def workload_layer(name: str, layer: int = 0, backend: str = "numpy", device="cuda", T: int | None = None,
                   H: int | None = None):
    """One layer of a named workload (seed = base seed + layer)."""
    w = WORKLOADS[name]
    args = dict(gen=w["gen"], rank=w.get("rank", 24), noise=w.get("noise", 0.1), outlier=w.get("outlier"),
                dtype=w["dtype"])
    HH, TT = H or w["H"], T or w["T"]
    if backend == "numpy":
        return numpy_layer(HH, TT, w["D"], w["seed"] + layer, **args)
    return torch_layer(HH, TT, w["D"], w["seed"] + layer, device=device, **args)
