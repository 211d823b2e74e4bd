"""kvforge_b200 -- B200-native KVForge KV-cache codec.

Python face of libkvforge_b200.so, mirroring the reference Python API
(crates/kvforge-python/kvforge/__init__.py:3-17): KVCache, CompressedKV,
CompressionPipeline, compress, decompress -- plus stage-level classes that
mirror the kvforge-core traits (crates/kvforge-core/src/codec.rs:27-137).

Tensors may be numpy arrays or torch tensors, float32 or float16, on the host
or on the GPU; the codec itself always runs on the GPU through the C ABI.
PyTorch supplies device memory and the current stream only.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib as L
from ._lib import KvForgeError

__all__ = [
    "KVCache", "CompressedKV", "CompressionPipeline", "StreamingCompressor", "GpuCostModel", "BandwidthTier",
    "CostEstimate", "compress_adaptive", "compress", "decompress", "KvForgeError",
    "Basis", "QuantParams", "EntropyState", "GpuQuantizer", "GpuProjector", "GpuSensitivityCalibrator",
    "GpuEntropyCodec", "config_from_preset", "parse_preset", "INT4", "INT8", "F32", "PER_CHANNEL", "PER_TOKEN",
]

INT4, INT8, F32 = L.INT4, L.INT8, L.F32
PER_CHANNEL, PER_TOKEN = L.PER_CHANNEL, L.PER_TOKEN

_PRESETS = {"conservative": L.CONSERVATIVE, "balanced": L.BALANCED, "aggressive": L.AGGRESSIVE,
            "adaptive": L.ADAPTIVE}


def parse_preset(preset) -> int:
    """Case-insensitive preset name (crates/kvforge-python/src/py_pipeline.rs:16-27)."""
    if isinstance(preset, int):
        return preset
    p = _PRESETS.get(str(preset).lower())
    if p is None:
        raise ValueError(f"Unknown preset '{preset}'. Choose from: conservative, balanced, aggressive, adaptive")
    return p


def config_from_preset(preset) -> L.PipelineConfig:
    """PipelineConfig::from_preset (crates/kvforge-core/src/pipeline.rs:30-71)."""
    cfg = L.PipelineConfig()
    L.check(L.lib().kvf_pipeline_config_from_preset(parse_preset(preset), C.byref(cfg)))
    return cfg


def _device_index(device) -> int:
    if device is None:
        return torch.cuda.current_device() if torch.cuda.is_available() else 0
    if isinstance(device, torch.device):
        return device.index or 0
    if isinstance(device, str):
        return torch.device(device).index or 0
    return int(device)


def _stream(dev: int) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _as_device(x, dev: int) -> torch.Tensor:
    """Contiguous float32/float16 tensor on cuda:dev (other dtypes are rejected)."""
    if isinstance(x, np.ndarray):
        if x.dtype not in (np.float32, np.float16):
            raise TypeError(f"expected float32 or float16 data, got {x.dtype}")
        x = torch.from_numpy(np.ascontiguousarray(x))
    if not isinstance(x, torch.Tensor):
        raise TypeError("expected a numpy array or a torch tensor")
    if x.dtype not in (torch.float32, torch.float16):
        raise TypeError(f"expected float32 or float16 data, got {x.dtype}")
    return x.to(device=f"cuda:{dev}").contiguous()


def _dtype_code(t: torch.Tensor) -> int:
    return L.IN_F16 if t.dtype == torch.float16 else L.IN_F32


def _ptr(t: Optional[torch.Tensor]) -> C.c_void_p:
    return C.c_void_p(t.data_ptr() if t is not None else 0)


class _CudaView:
    """Zero-copy view of library-owned device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def _view(ptr: int, shape, typestr: str, dev: int) -> torch.Tensor:
    if int(np.prod(shape)) == 0 or not ptr:
        dt = {"<f4": torch.float32, "|u1": torch.uint8, "<u4": torch.int32, "<u8": torch.int64}[typestr]
        return torch.empty(shape, dtype=dt, device=f"cuda:{dev}")
    return torch.as_tensor(_CudaView(ptr, shape, typestr), device=f"cuda:{dev}")


# ---------------------------------------------------------------------------
# KVCache / CompressedKV (crates/kvforge-python/src/py_types.rs)
# ---------------------------------------------------------------------------
class KVCache:
    """One layer's KV cache, keys and values of shape [num_heads, seq_len, head_dim]."""

    def __init__(self, keys, values, layer_idx: int = 0):
        ks, vs = tuple(keys.shape), tuple(values.shape)
        if ks != vs:
            raise ValueError("keys and values must have the same shape")  # py_types.rs:29-33
        if len(ks) != 3:
            raise ValueError("keys and values must be 3-D [num_heads, seq_len, head_dim]")
        self._keys = keys
        self._values = values
        self._layer_idx = int(layer_idx)

    @property
    def layer_idx(self) -> int:
        return self._layer_idx

    @property
    def shape(self):
        return tuple(int(s) for s in self._keys.shape)

    @staticmethod
    def _np(x) -> np.ndarray:
        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu", torch.float32).numpy()
        return np.asarray(x, dtype=np.float32)

    def keys(self) -> np.ndarray:
        return self._np(self._keys)

    def values(self) -> np.ndarray:
        return self._np(self._values)

    @property
    def keys_tensor(self):
        return self._keys

    @property
    def values_tensor(self):
        return self._values

    def size_bytes(self) -> int:
        """Size as f32 (crates/kvforge-core/src/types.rs:30-32)."""
        H, T, D = self.shape
        return 2 * H * T * D * 4

    def __repr__(self):
        H, T, D = self.shape
        return f"KVCache(num_heads={H}, seq_len={T}, head_dim={D}, layer_idx={self._layer_idx})"


class CompressedKV:
    """Device-resident compressed layer (crates/kvforge-core/src/types.rs:36-56)."""

    def __init__(self, handle: C.c_void_p, device: int):
        self._h = handle
        self._dev = device

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and L is not None and L._lib is not None:  # module globals are gone at interpreter exit
            L.lib().kvf_compressed_free(h)
            self._h = None

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    @property
    def device(self) -> int:
        return self._dev

    def ratio(self) -> float:
        r = C.c_double()
        L.check(L.lib().kvf_compression_ratio(self._h, C.byref(r)))
        return r.value

    def compressed_size_bytes(self) -> int:
        n = C.c_size_t()
        L.check(L.lib().kvf_compressed_size_bytes(self._h, C.byref(n)))
        return n.value

    def original_size_bytes(self) -> int:
        n = C.c_size_t()
        L.check(L.lib().kvf_original_size_bytes(self._h, C.byref(n)))
        return n.value

    @property
    def shape(self):
        H, T, D = C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.check(L.lib().kvf_compressed_shape(self._h, C.byref(H), C.byref(T), C.byref(D), None))
        return H.value, T.value, D.value

    @property
    def layer_idx(self) -> int:
        li = C.c_size_t()
        L.check(L.lib().kvf_compressed_shape(self._h, None, None, None, C.byref(li)))
        return li.value

    def tensor_info(self, which: int) -> dict:
        """which: 0 keys, 1 values -> {R, packed_len, data_len, entropy}."""
        R, pl, dl, he = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_int32()
        L.check(L.lib().kvf_compressed_tensor_info(self._h, which, C.byref(R), C.byref(pl), C.byref(dl),
                                                  C.byref(he)))
        return {"R": R.value, "packed_len": pl.value, "data_len": dl.value, "entropy": bool(he.value)}

    def tensor_parts(self, which: int) -> dict:
        """Device tensors (zero-copy views) of one tensor's compressed state:
        data, scales, mins, freq (or None), basis_vt and ranks (or None)."""
        info = self.tensor_info(which)
        ptrs = [C.c_void_p() for _ in range(6)]
        L.check(L.lib().kvf_compressed_tensor_views(self._h, which, *[C.byref(p) for p in ptrs]))
        data, scales, mins, freq, bvt, ranks = [p.value or 0 for p in ptrs]
        H, T, D = self.shape
        R = info["R"]
        q = R if R else D
        axis = PER_CHANNEL if which == 0 else PER_TOKEN
        npar = H * q if axis == PER_CHANNEL else H * T
        out = {
            "data": _view(data, (info["data_len"],), "|u1", self._dev),
            "scales": _view(scales, (npar,), "<f4", self._dev),
            "mins": _view(mins, (npar,), "<f4", self._dev),
            "freq": _view(freq, (256,), "<u4", self._dev) if freq else None,
            "basis_vt": _view(bvt, (H, R, D), "<f4", self._dev) if bvt else None,
            "ranks": _view(ranks, (H,), "<u8", self._dev) if ranks else None,
            "packed_len": info["packed_len"],
            "R": R,
        }
        return out

    def attention(self, query, scale: Optional[float] = None) -> torch.Tensor:
        """Decode attention of one query row per head on the compressed layer:
        softmax(scale * K_h q_h) V_h for every head h, computed on the codes
        (KernelLauncher::fused_dequant_attention, kernel_launcher.rs:43-57).
        query [H, D] or [H, 1, D]; scale defaults to 1/sqrt(D). -> f32 [H, D] on
        the device, stream-ordered on the current stream."""
        H, T, D = self.shape
        q = _as_device(query, self._dev).to(torch.float32).reshape(H, D).contiguous()
        out = torch.empty((H, D), dtype=torch.float32, device=f"cuda:{self._dev}")
        sc = float(scale) if scale is not None else 1.0 / float(np.sqrt(D))
        L.check(L.lib().kvf_compressed_attention(L.context(self._dev), self._h, _ptr(q), sc, _ptr(out),
                                                 _stream(self._dev)))
        out._query = q  # keep the query alive until the stream has consumed it
        return out

    def basis(self, which: int) -> Optional["Basis"]:
        """The projection basis of one tensor (0 keys, 1 values) as a Basis that
        shares it (no copy), or None when that tensor was not projected."""
        h = C.c_void_p()
        L.check(L.lib().kvf_compressed_basis(self._h, which, C.byref(h)))
        return Basis(h, self._dev) if h.value else None

    def basis_size_bytes(self) -> int:
        """Bytes of projection state (ProjectionState::size_bytes,
        crates/kvforge-core/src/types.rs:131-135) inside compressed_size_bytes()."""
        n = C.c_size_t()
        L.check(L.lib().kvf_compressed_basis_bytes(self._h, C.byref(n)))
        return n.value

    def calibration_scores(self) -> Optional[np.ndarray]:
        """Per-head key sensitivity scores, or None (calibration off or T < 64)."""
        p = L.lib().kvf_compressed_calibration(self._h)
        if not p:
            return None
        torch.cuda.current_stream(self._dev).synchronize()
        return _view(p, (self.shape[0],), "<f4", self._dev).cpu().numpy()

    def to_bytes(self) -> bytes:
        n = C.c_size_t()
        L.check(L.lib().kvf_compressed_serialize(self._h, None, 0, C.byref(n)))
        buf = (C.c_uint8 * n.value)()
        L.check(L.lib().kvf_compressed_serialize(self._h, buf, n.value, C.byref(n)))
        return bytes(buf)

    @staticmethod
    def from_bytes(data: bytes, device=None) -> "CompressedKV":
        dev = _device_index(device)
        h = C.c_void_p()
        buf = (C.c_uint8 * len(data)).from_buffer_copy(data)
        L.check(L.lib().kvf_compressed_deserialize(L.context(dev), buf, len(data), C.byref(h), _stream(dev)))
        return CompressedKV(h, dev)

    def __repr__(self):
        return (f"CompressedKV(ratio={self.ratio():.1f}x, compressed_bytes={self.compressed_size_bytes()}, "
                f"original_bytes={self.original_size_bytes()})")


# ---------------------------------------------------------------------------
# Projection basis (the calibrated basis)
# ---------------------------------------------------------------------------
class Basis:
    """Per-head projection basis: basis_vt [H, R, D] (rows >= ranks[h] zero) and ranks [H]."""

    def __init__(self, handle: C.c_void_p, device: int):
        self._h = handle
        self._dev = device

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and L is not None and L._lib is not None:  # module globals are gone at interpreter exit
            L.lib().kvf_basis_free(h)
            self._h = None

    @property
    def handle(self):
        return self._h

    @staticmethod
    def compute(data, variance_threshold: float, max_rank: Optional[int] = None, device=None) -> "Basis":
        """Gram matrix on the GPU + fp64 eigen-solve on the host (projection.rs:77-92)."""
        dev = _device_index(device)
        x = _as_device(data, dev)
        H, T, D = x.shape
        h = C.c_void_p()
        L.check(L.lib().kvf_basis_compute(L.context(dev), _ptr(x), _dtype_code(x), H, T, D,
                                          float(variance_threshold), int(max_rank or 0), C.byref(h), _stream(dev)))
        return Basis(h, dev)

    @staticmethod
    def from_host(basis_vt: np.ndarray, ranks, device=None) -> "Basis":
        dev = _device_index(device)
        bvt = np.ascontiguousarray(basis_vt, np.float32)
        rk = np.ascontiguousarray(ranks, np.uint64)
        H, R, D = bvt.shape
        h = C.c_void_p()
        L.check(L.lib().kvf_basis_from_host(L.context(dev), H, R, D, bvt.ctypes.data_as(C.c_void_p),
                                            rk.ctypes.data_as(C.c_void_p), C.byref(h)))
        return Basis(h, dev)

    @property
    def dims(self):
        H, R, D = C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.check(L.lib().kvf_basis_info(self._h, C.byref(H), C.byref(R), C.byref(D)))
        return H.value, R.value, D.value

    @property
    def R(self) -> int:
        return self.dims[1]

    def host(self):
        """-> (basis_vt [H,R,D] f32, ranks [H] u64, singular values [H,D] f32)."""
        H, R, D = self.dims
        bvt = np.zeros((H, R, D), np.float32)
        rk = np.zeros(H, np.uint64)
        sv = np.zeros((H, D), np.float32)
        L.check(L.lib().kvf_basis_download(self._h, bvt.ctypes.data_as(C.c_void_p), rk.ctypes.data_as(C.c_void_p),
                                           sv.ctypes.data_as(C.c_void_p)))
        return bvt, rk, sv

    @property
    def ranks(self) -> np.ndarray:
        return self.host()[1]

    def device_vt(self) -> int:
        return L.lib().kvf_basis_device_vt(self._h) or 0

    def device_ranks(self) -> int:
        return L.lib().kvf_basis_device_ranks(self._h) or 0


# ---------------------------------------------------------------------------
# Pipeline (crates/kvforge-python/src/py_pipeline.rs, cpu/src/pipeline.rs:99-186)
# ---------------------------------------------------------------------------
class CompressionPipeline:
    """GPU compression pipeline. compress() takes a KVCache and a preset name."""

    def __init__(self, device=None):
        self._dev = _device_index(device)

    def compress(self, kv: KVCache, preset="balanced", key_basis: Optional[Basis] = None,
                 value_basis: Optional[Basis] = None) -> CompressedKV:
        cfg = config_from_preset(preset)
        return self.compress_with_config(kv, cfg, key_basis, value_basis)

    def compress_with_config(self, kv: KVCache, cfg: L.PipelineConfig, key_basis: Optional[Basis] = None,
                             value_basis: Optional[Basis] = None) -> CompressedKV:
        dev = self._dev
        k = _as_device(kv.keys_tensor, dev)
        v = _as_device(kv.values_tensor, dev)
        if k.dtype != v.dtype:
            v = v.to(k.dtype)
        H, T, D = k.shape
        h = C.c_void_p()
        L.check(L.lib().kvf_compress_layer(L.context(dev), _ptr(k), _ptr(v), _dtype_code(k), H, T, D, kv.layer_idx,
                                           C.byref(cfg), key_basis.handle if key_basis else None,
                                           value_basis.handle if value_basis else None, C.byref(h), _stream(dev)))
        c = CompressedKV(h, dev)
        c._inputs = (k, v)  # keep the inputs alive until the stream has consumed them
        return c

    def compress_layers(self, kvs, cfg, key_bases=None, value_bases=None, decompress: bool = False):
        """Compress the chunks of many layers (same [H, T, D] and input dtype)
        in one call, kvf_compress_layers: short chunks take one kernel launch
        for all layers. cfg is a preset name or a PipelineConfig; key_bases /
        value_bases are lists of Basis (one per layer) or None. Returns the
        list of CompressedKV, bit for bit what compress_with_config gives per
        layer; with decompress=True also the list of decompressed KVCache (f32,
        the CUDA-core reconstruction), without a host synchronisation."""
        if isinstance(cfg, (str, int)):
            cfg = config_from_preset(cfg)
        dev = self._dev
        kvs = list(kvs)
        n = len(kvs)
        ks, vs = [], []
        for kv in kvs:
            k = _as_device(kv.keys_tensor, dev)
            v = _as_device(kv.values_tensor, dev)
            if k.dtype != v.dtype:
                v = v.to(k.dtype)
            ks.append(k)
            vs.append(v)
        if n == 0:
            return ([], []) if decompress else []
        H, T, D = ks[0].shape
        for k, v in zip(ks, vs):
            if tuple(k.shape) != (H, T, D) or tuple(v.shape) != (H, T, D) or k.dtype != ks[0].dtype:
                raise KvForgeError(L.ERR_SHAPE_MISMATCH, "compress_layers: every layer needs the same shape and dtype")
        P = C.c_void_p * n
        kp = P(*[k.data_ptr() for k in ks])
        vp = P(*[v.data_ptr() for v in vs])
        idx = (C.c_size_t * n)(*[kv.layer_idx for kv in kvs])
        kb = P(*[b.handle.value if b is not None else None for b in key_bases]) if key_bases else None
        vb = P(*[b.handle.value if b is not None else None for b in value_bases]) if value_bases else None
        outs = P()
        ko = vo = None
        kop = vop = None
        if decompress:
            ko = [torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}") for _ in range(n)]
            vo = [torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}") for _ in range(n)]
            kop = P(*[t.data_ptr() for t in ko])
            vop = P(*[t.data_ptr() for t in vo])
        L.check(L.lib().kvf_compress_layers(L.context(dev), n, kp, vp, _dtype_code(ks[0]), H, T, D, idx, C.byref(cfg),
                                            kb, vb, outs, kop, vop, _stream(dev)))
        cs = []
        for i in range(n):
            c = CompressedKV(C.c_void_p(outs[i]), dev)
            c._inputs = (ks[i], vs[i])
            cs.append(c)
        if not decompress:
            return cs
        return cs, [KVCache(ko[i], vo[i], kvs[i].layer_idx) for i in range(n)]

    def decompress(self, compressed: CompressedKV) -> KVCache:
        dev = compressed.device
        H, T, D = compressed.shape
        ko = torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")
        vo = torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")
        L.check(L.lib().kvf_decompress_layer(L.context(dev), compressed.handle, _ptr(ko), _ptr(vo), _stream(dev)))
        L.check(L.lib().kvf_sync(L.context(dev), _stream(dev)))
        return KVCache(ko, vo, compressed.layer_idx)


class StreamingCompressor:
    """Append-mode compression of a growing KV cache, one layer at a time.

    The reference has no append API: every chunk is compressed as its own
    KVCache, with a fresh SVD over the chunk's tokens for projection presets
    (crates/kvforge-cpu/src/pipeline.rs:100-163). That is this class with
    reuse_basis=False. With reuse_basis=True (the extension) prefill() keeps the
    bases calibrated on each layer's prefix and append() projects every later
    chunk of that layer onto them: no eigen-solve and no host synchronisation
    per chunk, and the chunk is still a complete CompressedKV in the
    reference's format (it carries the prefix's basis). A store that keeps one
    basis per layer charges an appended chunk amortized_size_bytes(): its
    compressed size without the basis bytes. Without projection both modes
    are the same."""

    def __init__(self, preset="balanced", reuse_basis: bool = True, device=None):
        self._pipe = CompressionPipeline(device)
        self._cfg = config_from_preset(preset)
        self._reuse = bool(reuse_basis)
        self._bases = {}

    @property
    def reuse_basis(self) -> bool:
        return self._reuse

    def prefill(self, kv: KVCache) -> CompressedKV:
        """Compress a layer's prefix; with basis reuse, keep its bases for that layer."""
        c = self._pipe.compress_with_config(kv, self._cfg)
        if self._reuse and self._cfg.enable_projection:
            self._bases[kv.layer_idx] = (c.basis(0), c.basis(1))
        return c

    def append(self, kv: KVCache) -> CompressedKV:
        """Compress one appended chunk of a layer (any number of tokens >= 1)."""
        kb = vb = None
        if self._reuse and self._cfg.enable_projection:
            if kv.layer_idx not in self._bases:
                raise KvForgeError(L.ERR_INVALID_CONFIG, f"layer {kv.layer_idx}: append before prefill")
            kb, vb = self._bases[kv.layer_idx]
        return self._pipe.compress_with_config(kv, self._cfg, kb, vb)

    def append_layers(self, kvs, decompress: bool = False):
        """Compress one appended chunk of each of many layers (same shape) in
        one call (CompressionPipeline.compress_layers); with basis reuse each
        layer projects onto its own prefix's bases."""
        kvs = list(kvs)
        kb = vb = None
        if self._reuse and self._cfg.enable_projection:
            for kv in kvs:
                if kv.layer_idx not in self._bases:
                    raise KvForgeError(L.ERR_INVALID_CONFIG, f"layer {kv.layer_idx}: append before prefill")
            kb = [self._bases[kv.layer_idx][0] for kv in kvs]
            vb = [self._bases[kv.layer_idx][1] for kv in kvs]
        return self._pipe.compress_layers(kvs, self._cfg, kb, vb, decompress)

    def bases(self, layer_idx: int):
        """(key Basis, value Basis) kept for a layer, or None."""
        return self._bases.get(layer_idx)

    def amortized_size_bytes(self, c: CompressedKV) -> int:
        """Compressed size of an appended chunk when its bases are the layer's
        shared ones (stored once, with the prefix); the full size otherwise."""
        return c.compressed_size_bytes() - (c.basis_size_bytes() if self._reuse else 0)

    def decompress(self, c: CompressedKV) -> KVCache:
        return self._pipe.decompress(c)


# ---------------------------------------------------------------------------
# Cost model (CostModel, crates/kvforge-core/src/cost.rs) with measured GPU costs
# ---------------------------------------------------------------------------
class BandwidthTier:
    """BandwidthTier (crates/kvforge-core/src/cost.rs), in declaration order."""
    LOCAL, RDMA, ETHERNET_100G, ETHERNET_25G, ETHERNET_10G, WAN = range(6)

    @staticmethod
    def bytes_per_us(tier: int) -> float:
        v = L.lib().kvf_bandwidth_bytes_per_us(int(tier))
        if v < 0:
            raise ValueError(f"unknown bandwidth tier {tier}")
        return v


@dataclass
class CostEstimate:
    preset: int
    compress_us: float
    transfer_us: float
    decompress_us: float
    total_us: float
    compression_ratio: float


_PRESET_NAMES = {v: k for k, v in _PRESETS.items()}


class GpuCostModel:
    """CostModel whose table is measured on this GPU.

    The reference's CpuCostModel (crates/kvforge-cpu/src/cost.rs:9-115) holds a
    fixed table of ratio, microseconds per byte and quality per preset and ranks
    presets by compress + transfer + decompress time on a bandwidth tier. Here
    measure() times the GPU pipeline on a sample layer (bases calibrated once,
    outside the timing), takes the sample's ratio and scores quality as
    1 - the larger relative Frobenius error of keys and values. estimate() and
    select_codec() are the reference's arithmetic (through the C ABI); any
    table, the reference's own included, can be given to the constructor.
    select_preset() picks the preset the Adaptive preset stands for
    (crates/kvforge-core/src/pipeline.rs:14-15)."""

    def __init__(self, rows):
        self._rows = (L.PresetCost * len(rows))()
        for i, r in enumerate(rows):
            if isinstance(r, L.PresetCost):
                self._rows[i] = r
            else:
                self._rows[i] = L.PresetCost(int(r["preset"]), float(r["compression_ratio"]),
                                             float(r["compress_us_per_byte"]), float(r["decompress_us_per_byte"]),
                                             float(r["quality"]))

    @staticmethod
    def measure(kv: KVCache, reps: int = 5, device=None) -> "GpuCostModel":
        dev = _device_index(device)
        k = _as_device(kv.keys_tensor, dev)
        v = _as_device(kv.values_tensor, dev)
        if k.dtype != v.dtype:
            v = v.to(k.dtype)
        H, T, D = k.shape
        rows = (L.PresetCost * 3)()
        L.check(L.lib().kvf_cost_measure(L.context(dev), _ptr(k), _ptr(v), _dtype_code(k), H, T, D, int(reps),
                                         rows, _stream(dev)))
        return GpuCostModel(list(rows))

    def rows(self) -> list:
        return [dict(preset=_PRESET_NAMES[r.preset], compression_ratio=r.compression_ratio,
                     compress_us_per_byte=r.compress_us_per_byte, decompress_us_per_byte=r.decompress_us_per_byte,
                     quality=r.quality) for r in self._rows]

    @staticmethod
    def _bw(bandwidth) -> float:
        return float(bandwidth) if isinstance(bandwidth, float) else BandwidthTier.bytes_per_us(bandwidth)

    def estimate(self, original_bytes: int, preset, bandwidth) -> CostEstimate:
        """bandwidth: a BandwidthTier value, or bytes per microsecond as a float."""
        e = L.CostEstimate()
        L.check(L.lib().kvf_cost_estimate(self._rows, len(self._rows), int(original_bytes), parse_preset(preset),
                                          self._bw(bandwidth), C.byref(e)))
        return CostEstimate(e.preset, e.compress_us, e.transfer_us, e.decompress_us, e.total_us, e.compression_ratio)

    def select_codec(self, original_bytes: int, bandwidth, min_quality: Optional[float] = None) -> list:
        out = (L.CostEstimate * len(self._rows))()
        n = C.c_size_t()
        L.check(L.lib().kvf_cost_select(self._rows, len(self._rows), int(original_bytes), self._bw(bandwidth),
                                        float(min_quality or 0.0), out, C.byref(n)))
        return [CostEstimate(e.preset, e.compress_us, e.transfer_us, e.decompress_us, e.total_us,
                             e.compression_ratio) for e in out[: n.value]]

    def select_preset(self, original_bytes: int, bandwidth, min_quality: Optional[float] = None) -> str:
        est = self.select_codec(original_bytes, bandwidth, min_quality)
        if not est:
            raise KvForgeError(L.ERR_INVALID_CONFIG, "no preset meets the quality floor")
        return _PRESET_NAMES[est[0].preset]


def compress_adaptive(kv: KVCache, model: GpuCostModel, bandwidth, min_quality: Optional[float] = None,
                      device=None):
    """Compress with the preset the cost model ranks fastest end to end for
    this layer's size on `bandwidth`. -> (CompressedKV, preset name)."""
    preset = model.select_preset(kv.size_bytes(), bandwidth, min_quality)
    return CompressionPipeline(device).compress(kv, preset), preset


def compress(kv: KVCache, preset="balanced") -> CompressedKV:
    """Module-level compress (crates/kvforge-python/src/py_pipeline.rs:65-70)."""
    return CompressionPipeline().compress(kv, preset)


def decompress(compressed: CompressedKV) -> KVCache:
    """Module-level decompress (crates/kvforge-python/src/py_pipeline.rs:73-77)."""
    return CompressionPipeline(compressed.device).decompress(compressed)


# ---------------------------------------------------------------------------
# Stage-level API, mirroring the kvforge-core traits
# ---------------------------------------------------------------------------
@dataclass
class QuantParams:
    """QuantParams (crates/kvforge-core/src/types.rs:81-95)."""
    scales: torch.Tensor
    mins: torch.Tensor
    data_type: int
    axis: int
    shape: tuple

    def size_bytes(self) -> int:
        return (self.scales.numel() + self.mins.numel()) * 4


@dataclass
class EntropyState:
    """EntropyState (crates/kvforge-core/src/types.rs:138-148)."""
    frequencies: torch.Tensor  # uint32 counts [256], or empty when coding was skipped
    original_len: int

    def size_bytes(self) -> int:
        return self.frequencies.numel() * 4 + 8


class GpuQuantizer:
    """Quantizer trait (codec.rs:104-115) on the GPU."""

    def __init__(self, device=None):
        self._dev = _device_index(device)

    def quantize(self, data, data_type: int, axis: int):
        dev = self._dev
        x = _as_device(data, dev)
        H, T, D = x.shape
        n = H * T * D
        plen = (n + 1) // 2 if data_type == INT4 else n
        npar = H * D if axis == PER_CHANNEL else H * T
        packed = torch.empty(plen, dtype=torch.uint8, device=f"cuda:{dev}")
        scales = torch.empty(npar, dtype=torch.float32, device=f"cuda:{dev}")
        mins = torch.empty(npar, dtype=torch.float32, device=f"cuda:{dev}")
        L.check(L.lib().kvf_quantize(L.context(dev), _ptr(x), _dtype_code(x), H, T, D, data_type, axis,
                                     _ptr(packed), _ptr(scales), _ptr(mins), _stream(dev)))
        return packed, QuantParams(scales, mins, data_type, axis, (H, T, D))

    def dequantize(self, packed: torch.Tensor, params: QuantParams) -> torch.Tensor:
        dev = self._dev
        H, T, D = params.shape
        out = torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")
        p = packed.to(f"cuda:{dev}").contiguous()
        L.check(L.lib().kvf_dequantize(L.context(dev), _ptr(p), p.numel(), _ptr(params.scales), _ptr(params.mins),
                                       params.data_type, params.axis, H, T, D, _ptr(out), _stream(dev)))
        return out


class GpuProjector:
    """Projector trait (codec.rs:49-65) on the GPU, against a calibrated basis."""

    def __init__(self, device=None):
        self._dev = _device_index(device)

    def compute_basis(self, data, variance_threshold: float, max_rank: Optional[int] = None) -> Basis:
        return Basis.compute(data, variance_threshold, max_rank, self._dev)

    def project(self, data, basis: Basis) -> torch.Tensor:
        dev = self._dev
        x = _as_device(data, dev)
        H, T, D = x.shape
        R = basis.R
        out = torch.empty((H, T, R), dtype=torch.float32, device=f"cuda:{dev}")
        L.check(L.lib().kvf_project(L.context(dev), _ptr(x), _dtype_code(x), H, T, D,
                                    C.c_void_p(basis.device_vt()), C.c_void_p(basis.device_ranks()), R, _ptr(out),
                                    _stream(dev)))
        return out

    def reconstruct(self, projected, basis: Basis) -> torch.Tensor:
        dev = self._dev
        p = _as_device(projected, dev).float()
        H, T, R = p.shape
        D = basis.dims[2]
        out = torch.empty((H, T, D), dtype=torch.float32, device=f"cuda:{dev}")
        L.check(L.lib().kvf_reconstruct(L.context(dev), _ptr(p), H, T, R, D, C.c_void_p(basis.device_vt()),
                                        C.c_void_p(basis.device_ranks()), _ptr(out), _stream(dev)))
        return out


class GpuSensitivityCalibrator:
    """SensitivityCalibrator trait (codec.rs:26-29) on the GPU; takes the keys."""

    def __init__(self, device=None):
        self._dev = _device_index(device)

    def calibrate(self, keys, min_tokens: int = 64) -> torch.Tensor:
        dev = self._dev
        x = _as_device(keys.keys_tensor if isinstance(keys, KVCache) else keys, dev)
        H, T, D = x.shape
        out = torch.empty(H, dtype=torch.float32, device=f"cuda:{dev}")
        L.check(L.lib().kvf_calibrate(L.context(dev), _ptr(x), _dtype_code(x), H, T, D, min_tokens, _ptr(out),
                                      _stream(dev)))
        return out


class GpuEntropyCodec:
    """EntropyCodec trait (codec.rs:130-137) on the GPU, chunked rANS container."""

    def __init__(self, device=None):
        self._dev = _device_index(device)

    def encode(self, data: torch.Tensor, enabled: bool = True):
        dev = self._dev
        d = data.to(f"cuda:{dev}").contiguous().view(torch.uint8).reshape(-1)
        if not enabled or d.numel() == 0:  # entropy.rs:43-49
            return d.clone(), EntropyState(torch.empty(0, dtype=torch.int32, device=f"cuda:{dev}"), d.numel())
        cap = int(L.lib().kvf_rans_max_encoded_len(d.numel()))
        out = torch.empty(cap, dtype=torch.uint8, device=f"cuda:{dev}")
        freq = torch.empty(256, dtype=torch.int32, device=f"cuda:{dev}")
        n = C.c_size_t()
        L.check(L.lib().kvf_rans_encode(L.context(dev), _ptr(d), d.numel(), _ptr(out), cap, C.byref(n), _ptr(freq),
                                        _stream(dev)))
        return out[: n.value].clone(), EntropyState(freq, d.numel())

    def decode(self, data: torch.Tensor, state: EntropyState) -> torch.Tensor:
        dev = self._dev
        d = data.to(f"cuda:{dev}").contiguous().view(torch.uint8).reshape(-1)
        if state.frequencies.numel() == 0 or state.original_len == 0:  # entropy.rs:89-91
            return d.clone()
        out = torch.empty(state.original_len, dtype=torch.uint8, device=f"cuda:{dev}")
        f = state.frequencies.to(f"cuda:{dev}").contiguous()
        L.check(L.lib().kvf_rans_decode(L.context(dev), _ptr(d), d.numel(), _ptr(f), state.original_len, _ptr(out),
                                        _stream(dev)))
        return out
