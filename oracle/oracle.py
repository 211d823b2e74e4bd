"""ctypes front-end of the CPU oracle (oracle/kvforge_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU legs of bench.py, always as the checker. The product package never imports
this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

INT4, INT8, F32 = 0, 1, 2
PER_CHANNEL, PER_TOKEN = 0, 1
DEFAULT_CHUNK = 8192

_lib = None


def build(force: bool = False) -> str:
    src = os.path.join(_HERE, "kvforge_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE, "liboracle.so"])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sz, p, i32, f64 = C.c_size_t, C.c_void_p, C.c_int, C.c_double
        L.orc_pack_int4.restype = C.c_uint8
        L.orc_pack_int4.argtypes = [C.c_uint8, C.c_uint8]
        L.orc_unpack_int4.argtypes = [C.c_uint8, p, p]
        L.orc_quantize.argtypes = [p, sz, sz, sz, i32, i32, p, p, p]
        L.orc_dequantize.argtypes = [p, sz, p, p, i32, i32, sz, sz, sz, p]
        L.orc_calibrate.argtypes = [p, sz, sz, sz, sz, p]
        L.orc_select_rank.restype = sz
        L.orc_select_rank.argtypes = [p, sz, f64, sz]
        L.orc_compute_basis.argtypes = [p, sz, sz, sz, p, p, i32]
        L.orc_select_basis.restype = sz
        L.orc_select_basis.argtypes = [p, p, sz, sz, sz, f64, sz, p, p]
        L.orc_project.argtypes = [p, sz, sz, sz, p, p, sz, p, i32]
        L.orc_reconstruct.argtypes = [p, sz, sz, sz, sz, p, p, p, i32]
        L.orc_histogram.argtypes = [p, sz, p]
        L.orc_rans_normalize.argtypes = [p, p, p]
        L.orc_rans_max_encoded_len.restype = sz
        L.orc_rans_max_encoded_len.argtypes = [sz, C.c_uint32]
        L.orc_rans_encode.argtypes = [p, sz, C.c_uint32, p, sz, C.POINTER(C.c_size_t), p]
        L.orc_rans_decode.argtypes = [p, sz, p, sz, p]
        L.orc_entropy_bits.restype = f64
        L.orc_entropy_bits.argtypes = [p]
        _lib = L
    return _lib


class OracleError(RuntimeError):
    def __init__(self, status: int, what: str):
        super().__init__(f"oracle {what} failed with status {status}")
        self.status = status


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _chk(st: int, what: str):
    if st != 0:
        raise OracleError(st, what)


def pack_int4(a: int, b: int) -> int:
    return int(lib().orc_pack_int4(a, b))


def unpack_int4(byte: int):
    lo, hi = C.c_uint8(), C.c_uint8()
    lib().orc_unpack_int4(byte, C.byref(lo), C.byref(hi))
    return lo.value, hi.value


def packed_len(n: int, data_type: int) -> int:
    return (n + 1) // 2 if data_type == INT4 else n


def quantize(x: np.ndarray, data_type: int, axis: int):
    x = np.ascontiguousarray(x, dtype=np.float32)
    H, T, D = x.shape
    n = H * T * D
    packed = np.zeros(max(packed_len(n, data_type), 1), np.uint8)[: packed_len(n, data_type)]
    npar = H * D if axis == PER_CHANNEL else H * T
    scales = np.zeros(npar, np.float32)
    mins = np.zeros(npar, np.float32)
    _chk(lib().orc_quantize(_ptr(x), H, T, D, data_type, axis, _ptr(packed), _ptr(scales), _ptr(mins)), "quantize")
    return packed, scales, mins


def dequantize(packed: np.ndarray, scales, mins, data_type: int, axis: int, shape):
    H, T, D = shape
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.zeros((H, T, D), np.float32)
    sc = np.ascontiguousarray(scales, np.float32)
    mn = np.ascontiguousarray(mins, np.float32)
    _chk(lib().orc_dequantize(_ptr(packed), packed.size, _ptr(sc), _ptr(mn), data_type, axis, H, T, D, _ptr(out)),
         "dequantize")
    return out


def calibrate(keys: np.ndarray, min_tokens: int = 64):
    keys = np.ascontiguousarray(keys, dtype=np.float32)
    H, T, D = keys.shape
    scores = np.zeros(H, np.float32)
    _chk(lib().orc_calibrate(_ptr(keys), H, T, D, min_tokens, _ptr(scores)), "calibrate")
    return scores


def select_rank(sv, threshold: float, max_rank=None) -> int:
    sv = np.ascontiguousarray(sv, dtype=np.float32)
    return int(lib().orc_select_rank(_ptr(sv), sv.size, float(threshold), int(max_rank or 0)))


def compute_basis(x: np.ndarray, threads: int = 1):
    """Full per-head eigenbasis: (basis_full [H,D,D], sv [H,D])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    H, T, D = x.shape
    basis = np.zeros((H, D, D), np.float32)
    sv = np.zeros((H, D), np.float32)
    _chk(lib().orc_compute_basis(_ptr(x), H, T, D, _ptr(basis), _ptr(sv), threads), "compute_basis")
    return basis, sv


def select_basis(basis_full, sv, T: int, threshold: float, max_rank=None):
    """-> (basis_vt [H,R,D], ranks [H] uint64, R)."""
    basis_full = np.ascontiguousarray(basis_full, np.float32)
    sv = np.ascontiguousarray(sv, np.float32)
    H, D, _ = basis_full.shape
    ranks = np.zeros(H, np.uint64)
    R = int(lib().orc_select_basis(_ptr(basis_full), _ptr(sv), H, T, D, float(threshold), int(max_rank or 0),
                                   _ptr(ranks), None))
    bvt = np.zeros((H, R, D), np.float32)
    lib().orc_select_basis(_ptr(basis_full), _ptr(sv), H, T, D, float(threshold), int(max_rank or 0),
                           _ptr(ranks), _ptr(bvt))
    return bvt, ranks, R


def project(x: np.ndarray, basis_vt: np.ndarray, ranks: np.ndarray, threads: int = 1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    H, T, D = x.shape
    bvt = np.ascontiguousarray(basis_vt, np.float32)
    R = bvt.shape[1]
    rk = np.ascontiguousarray(ranks, np.uint64)
    out = np.zeros((H, T, R), np.float32)
    _chk(lib().orc_project(_ptr(x), H, T, D, _ptr(bvt), _ptr(rk), R, _ptr(out), threads), "project")
    return out


def reconstruct(p: np.ndarray, basis_vt: np.ndarray, ranks: np.ndarray, threads: int = 1):
    p = np.ascontiguousarray(p, np.float32)
    H, T, R = p.shape
    bvt = np.ascontiguousarray(basis_vt, np.float32)
    D = bvt.shape[2]
    rk = np.ascontiguousarray(ranks, np.uint64)
    out = np.zeros((H, T, D), np.float32)
    _chk(lib().orc_reconstruct(_ptr(p), H, T, R, D, _ptr(bvt), _ptr(rk), _ptr(out), threads), "reconstruct")
    return out


def histogram(data: np.ndarray):
    data = np.ascontiguousarray(data, np.uint8)
    f = np.zeros(256, np.uint32)
    lib().orc_histogram(_ptr(data), data.size, _ptr(f))
    return f


def rans_normalize(freq):
    freq = np.ascontiguousarray(freq, np.uint32)
    q = np.zeros(256, np.uint32)
    cum = np.zeros(256, np.uint32)
    _chk(lib().orc_rans_normalize(_ptr(freq), _ptr(q), _ptr(cum)), "rans_normalize")
    return q, cum


def rans_encode(data: np.ndarray, chunk: int = DEFAULT_CHUNK):
    """-> (container bytes, freq[256])."""
    data = np.ascontiguousarray(data, np.uint8)
    cap = int(lib().orc_rans_max_encoded_len(data.size, chunk))
    out = np.zeros(max(cap, 1), np.uint8)
    olen = C.c_size_t(0)
    freq = np.zeros(256, np.uint32)
    _chk(lib().orc_rans_encode(_ptr(data), data.size, chunk, _ptr(out), cap, C.byref(olen), _ptr(freq)),
         "rans_encode")
    return out[: olen.value].copy(), freq


def rans_decode(comp: np.ndarray, freq, original_len: int):
    comp = np.ascontiguousarray(comp, np.uint8)
    freq = np.ascontiguousarray(freq, np.uint32)
    out = np.zeros(max(original_len, 1), np.uint8)
    _chk(lib().orc_rans_decode(_ptr(comp), comp.size, _ptr(freq), original_len, _ptr(out)), "rans_decode")
    return out[:original_len]


def entropy_bits(freq) -> float:
    freq = np.ascontiguousarray(freq, np.uint32)
    return float(lib().orc_entropy_bits(_ptr(freq)))


# ---------------------------------------------------------------------------
# Pipeline (crates/kvforge-cpu/src/pipeline.rs:38-186, core/src/pipeline.rs:30-71)
# ---------------------------------------------------------------------------
PRESETS = {
    "conservative": dict(key=INT8, value=INT8, proj=False, thr=0.99, entropy=False, calib=False),
    "balanced": dict(key=INT4, value=INT4, proj=True, thr=0.90, entropy=False, calib=False),
    "aggressive": dict(key=INT4, value=INT4, proj=True, thr=0.75, entropy=True, calib=True),
    "adaptive": dict(key=INT4, value=INT4, proj=True, thr=0.90, entropy=True, calib=True),
}


def compress_tensor(x, data_type, axis, basis=None, entropy=False, threads=1):
    """pipeline.rs:38-72. basis = (basis_vt, ranks) when projecting.
    Returns a dict with the same fields as the reference CompressedTensor."""
    x = np.ascontiguousarray(x, np.float32)
    H, T, D = x.shape
    proj_state = None
    q_in = x
    if basis is not None:
        bvt, ranks = basis
        q_in = project(x, bvt, ranks, threads)
        proj_state = (np.ascontiguousarray(bvt, np.float32), np.ascontiguousarray(ranks, np.uint64))
    packed, scales, mins = quantize(q_in, data_type, axis)
    ent = None
    data = packed
    if entropy:
        if packed.size == 0:
            ent = (np.zeros(0, np.uint32), 0)
        else:
            data, freq = rans_encode(packed)
            ent = (freq, packed.size)
    return dict(data=data, scales=scales, mins=mins, data_type=data_type, axis=axis,
                qshape=q_in.shape, proj=proj_state, entropy=ent)


def decompress_tensor(ct, threads=1):
    """pipeline.rs:75-97."""
    data = ct["data"]
    if ct["entropy"] is not None and ct["entropy"][1] > 0:
        data = rans_decode(data, ct["entropy"][0], ct["entropy"][1])
    deq = dequantize(data, ct["scales"], ct["mins"], ct["data_type"], ct["axis"], ct["qshape"])
    if ct["proj"] is not None:
        return reconstruct(deq, ct["proj"][0], ct["proj"][1], threads)
    return deq


def tensor_size_bytes(ct) -> int:
    """types.rs:66-78, 91-95, 131-135, 144-148."""
    total = int(ct["data"].size) + (ct["scales"].size + ct["mins"].size) * 4
    if ct["proj"] is not None:
        total += ct["proj"][0].size * 4 + ct["proj"][1].size * 8
    if ct["entropy"] is not None:
        total += ct["entropy"][0].size * 4 + 8
    return total


def basis_for(x, threshold, max_rank=None, threads=1):
    basis_full, sv = compute_basis(x, threads)
    bvt, ranks, R = select_basis(basis_full, sv, x.shape[1], threshold, max_rank)
    return bvt, ranks


def compress(keys, values, preset="balanced", layer_idx=0, bases=None, threads=1):
    """CpuCompressionPipeline::compress (pipeline.rs:99-163). bases: optional
    ((k_basis_vt, k_ranks), (v_basis_vt, v_ranks)); computed here when absent."""
    p = PRESETS[preset.lower()]
    keys = np.ascontiguousarray(keys, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    if keys.shape != values.shape:
        raise ValueError("keys and values must have the same shape")
    original = (keys.size + values.size) * 4
    scores = None
    if p["calib"]:
        try:
            scores = calibrate(keys, 64)
        except OracleError:
            scores = None  # pipeline.rs:106-111 discards the result and the error
    kb = vb = None
    if p["proj"]:
        if bases is None:
            kb = basis_for(keys, p["thr"], None, threads)
            vb = basis_for(values, p["thr"], None, threads)
        else:
            kb, vb = bases
    k = compress_tensor(keys, p["key"], PER_CHANNEL, kb, p["entropy"], threads)
    v = compress_tensor(values, p["value"], PER_TOKEN, vb, p["entropy"], threads)
    return dict(layer_idx=layer_idx, shape=keys.shape, key=k, value=v, original_size_bytes=original,
                scores=scores)


def decompress(ckv, threads=1):
    return decompress_tensor(ckv["key"], threads), decompress_tensor(ckv["value"], threads)


def decode_attention(keys, values, query, scale):
    """Single-query attention per head, fp64: out[h] = softmax(scale * K_h q_h) V_h,
    on the dequantized (and reconstructed) K and V -- the computation the
    reference's fused_dequant_attention kernel describes and leaves unimplemented
    (crates/kvforge-cuda/kernels/fused_dequant_attention.cu:1-10, steps at :30-34).
    keys, values [H, T, D]; query [H, D] -> [H, D] float64 (zeros when T = 0)."""
    k = np.asarray(keys, np.float64)
    v = np.asarray(values, np.float64)
    q = np.asarray(query, np.float64)
    H, T, D = k.shape
    if T == 0:
        return np.zeros((H, D))
    s = scale * np.einsum("htd,hd->ht", k, q)
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=1, keepdims=True)
    return np.einsum("ht,htd->hd", p, v)


# ---------------------------------------------------------------------------
# Wire format: CompressedKV.to_bytes / from_bytes are bincode::serialize /
# deserialize (crates/kvforge-python/src/py_types.rs:98-110) with bincode 1.x
# (Cargo.toml:28) of the structs in crates/kvforge-core/src/types.rs:36-148.
# bincode 1.x's default encoding, as its specification states it:
# little-endian fixed-width integers, usize as u64, a sequence as a u64
# length then its elements, an Option as a u8 tag (0 None, 1 Some) then the
# value, a unit enum variant as its u32 index, struct fields in order.
# ---------------------------------------------------------------------------
def _bc_seq(parts, arr, dtype):
    a = np.ascontiguousarray(arr, dtype)
    parts.append(np.uint64(a.size).tobytes())
    parts.append(a.astype(np.dtype(dtype).newbyteorder("<"), copy=False).tobytes())


def _bc_tensor(parts, ct):
    H, T, cols = (int(x) for x in ct["qshape"])
    _bc_seq(parts, ct["data"], np.uint8)                      # quantized_data
    _bc_seq(parts, ct["scales"], np.float32)                  # QuantParams.scales
    _bc_seq(parts, ct["mins"], np.float32)                    # QuantParams.mins
    parts.append(np.array([ct["data_type"], ct["axis"]], "<u4").tobytes())  # DataType, QuantAxis
    _bc_seq(parts, [H, T, cols], np.uint64)                   # QuantParams.shape
    if ct["proj"] is None:
        parts.append(b"\x00")
    else:
        bvt, ranks = ct["proj"]
        D = int(np.asarray(bvt).shape[2])
        parts.append(b"\x01")
        _bc_seq(parts, np.asarray(bvt).reshape(-1), np.float32)  # ProjectionState.basis_vt
        _bc_seq(parts, ranks, np.uint64)                           # ranks
        parts.append(np.array([H, D], "<u8").tobytes())            # num_heads, head_dim
        _bc_seq(parts, [H, T, cols], np.uint64)                    # projected_shape
    if ct["entropy"] is None:
        parts.append(b"\x00")
    else:
        freq, original_len = ct["entropy"]
        parts.append(b"\x01")
        _bc_seq(parts, freq, np.uint32)                            # EntropyState.frequencies
        parts.append(np.uint64(original_len).tobytes())            # original_len


def to_bincode(ckv) -> bytes:
    """The reference's CompressedKV.to_bytes of an oracle compressed layer."""
    H, T, D = (int(x) for x in ckv["shape"])
    parts = [np.array([ckv["layer_idx"], H, T, D], "<u8").tobytes()]
    _bc_tensor(parts, ckv["key"])
    _bc_tensor(parts, ckv["value"])
    parts.append(np.uint64(ckv["original_size_bytes"]).tobytes())
    return b"".join(parts)


class _BcReader:
    def __init__(self, b: bytes):
        self.b, self.p = b, 0

    def take(self, n: int) -> bytes:
        if self.p + n > len(self.b):
            raise ValueError("truncated bincode")
        s = self.b[self.p:self.p + n]
        self.p += n
        return s

    def u(self, fmt: str) -> int:
        d = np.dtype(fmt)
        return int(np.frombuffer(self.take(d.itemsize), d)[0])

    def seq(self, dtype) -> np.ndarray:
        n = self.u("<u8")
        d = np.dtype(dtype).newbyteorder("<")
        return np.frombuffer(self.take(n * d.itemsize), d).astype(dtype)


def _bc_read_tensor(r: _BcReader):
    data = r.seq(np.uint8)
    scales, mins = r.seq(np.float32), r.seq(np.float32)
    dt, ax = r.u("<u4"), r.u("<u4")
    qshape = tuple(int(x) for x in r.seq(np.uint64))
    proj = None
    if r.u("<u1"):
        bvt = r.seq(np.float32)
        ranks = r.seq(np.uint64)
        H, D = r.u("<u8"), r.u("<u8")
        r.seq(np.uint64)  # projected_shape
        proj = (bvt.reshape(H, -1, D), ranks)
    ent = None
    if r.u("<u1"):
        freq = r.seq(np.uint32)
        ent = (freq, r.u("<u8"))
    return dict(data=data, scales=scales, mins=mins, data_type=dt, axis=ax, qshape=qshape, proj=proj, entropy=ent)


def from_bincode(b: bytes):
    """CompressedKV.from_bytes into an oracle compressed layer (no calibration scores)."""
    r = _BcReader(b)
    layer_idx, H, T, D = (r.u("<u8") for _ in range(4))
    k = _bc_read_tensor(r)
    v = _bc_read_tensor(r)
    orig = r.u("<u8")
    if r.p != len(b):
        raise ValueError("trailing bytes")
    return dict(layer_idx=layer_idx, shape=(H, T, D), key=k, value=v, original_size_bytes=orig, scores=None)


def compressed_size_bytes(ckv) -> int:
    return tensor_size_bytes(ckv["key"]) + tensor_size_bytes(ckv["value"])


def ratio(ckv) -> float:
    return ckv["original_size_bytes"] / compressed_size_bytes(ckv)
