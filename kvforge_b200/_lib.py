"""ctypes binding of libkvforge_b200.so (declarations in include/kvforge.h).

Loading fails loudly: there is no CPU fallback. A missing library raises
ImportError with the build command; a missing CUDA device surfaces as a
KvForgeError from kvf_init.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkvforge_b200.so")

OK = 0
ERR_SHAPE_MISMATCH = 1
ERR_INVALID_CONFIG = 2
ERR_QUANTIZATION = 3
ERR_PROJECTION = 4
ERR_ENTROPY = 5
ERR_SERIALIZATION = 6
ERR_CUDA = 7
ERR_PIPELINE = 8
ERR_DEVICE_TIMEOUT = 9
ERR_CORRUPT_STREAM = 10

STATUS_NAMES = {
    0: "Ok", 1: "ShapeMismatch", 2: "InvalidConfig", 3: "QuantizationError", 4: "ProjectionError",
    5: "EntropyError", 6: "SerializationError", 7: "CudaError", 8: "PipelineError",
    9: "DeviceTimeout", 10: "CorruptStream",
}

INT4, INT8, F32 = 0, 1, 2
PER_CHANNEL, PER_TOKEN = 0, 1
IN_F32, IN_F16 = 0, 1
CONSERVATIVE, BALANCED, AGGRESSIVE, ADAPTIVE = 0, 1, 2, 3
RECON_AUTO, RECON_CUDA_CORE, RECON_TENSOR_CORE = 0, 1, 2
PROJ_AUTO, PROJ_CUDA_CORE, PROJ_TENSOR_CORE, PROJ_TENSOR_CORE_APPROX = 0, 1, 2, 3
WAIT_MBARRIER, WAIT_LOOKBACK = 0, 1

# every symbol include/kvforge.h declares
EXPORTS = [
    "kvf_init", "kvf_destroy", "kvf_last_error", "kvf_abi_version", "kvf_set_exact_reconstruct",
    "kvf_set_reconstruct_engine", "kvf_selftest_wait_timeout", "kvf_sync",
    "kvf_pipeline_config_from_preset", "kvf_calibrate", "kvf_quantize", "kvf_dequantize", "kvf_project",
    "kvf_reconstruct", "kvf_fused_project_quantize", "kvf_rans_max_encoded_len", "kvf_rans_encode",
    "kvf_rans_decode", "kvf_entropy_decode_dequant", "kvf_fused_dequant_attention", "kvf_compressed_attention",
    "kvf_basis_compute", "kvf_basis_from_host",
    "kvf_basis_info", "kvf_basis_download", "kvf_basis_device_vt", "kvf_basis_device_ranks", "kvf_basis_free",
    "kvf_compress_layer", "kvf_decompress_layer", "kvf_compress_layer_host", "kvf_decompress_layer_host",
    "kvf_compressed_shape", "kvf_compressed_size_bytes", "kvf_original_size_bytes", "kvf_compression_ratio",
    "kvf_compressed_tensor_info", "kvf_compressed_tensor_views", "kvf_compressed_basis",
    "kvf_compressed_basis_bytes", "kvf_compressed_calibration", "kvf_compressed_serialize",
    "kvf_compressed_deserialize", "kvf_compressed_free",
    "kvf_bandwidth_bytes_per_us", "kvf_cost_measure", "kvf_cost_estimate", "kvf_cost_select",
    "kvf_launch_count", "kvf_stage_name", "kvf_profile_enable", "kvf_profile_read", "kvf_calibrate_noalloc",
    "kvf_set_projection_engine", "kvf_compress_layers", "kvf_compressed_free_many",
]

NUM_STAGES = 8
STAGES = ["calibrate", "project", "quantize", "entropy_encode", "entropy_decode", "reconstruct", "dequantize",
          "basis"]


class PipelineConfig(C.Structure):
    """kvf_pipeline_config (crates/kvforge-core/src/pipeline.rs:17-28)."""
    _fields_ = [
        ("preset", C.c_int32),
        ("key_data_type", C.c_int32),
        ("value_data_type", C.c_int32),
        ("enable_projection", C.c_int32),
        ("projection_variance_threshold", C.c_double),
        ("enable_entropy_coding", C.c_int32),
        ("enable_calibration", C.c_int32),
    ]


class PresetCost(C.Structure):
    """kvf_preset_cost: one row of the cost table (crates/kvforge-cpu/src/cost.rs:15-24)."""
    _fields_ = [
        ("preset", C.c_int32),
        ("compression_ratio", C.c_double),
        ("compress_us_per_byte", C.c_double),
        ("decompress_us_per_byte", C.c_double),
        ("quality", C.c_double),
    ]


class CostEstimate(C.Structure):
    """kvf_estimate: CostEstimate (crates/kvforge-core/src/cost.rs)."""
    _fields_ = [
        ("preset", C.c_int32),
        ("compress_us", C.c_double),
        ("transfer_us", C.c_double),
        ("decompress_us", C.c_double),
        ("total_us", C.c_double),
        ("compression_ratio", C.c_double),
    ]


class KvForgeError(RuntimeError):
    """A failing kvf_* call; .status mirrors the reference KvForgeError kind."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_lib = None
_lock = threading.Lock()


def _declare(L):
    p, sz, i32, f64, st = C.c_void_p, C.c_size_t, C.c_int32, C.c_double, C.c_int
    u64p = C.POINTER(C.c_uint64)
    szp = C.POINTER(C.c_size_t)
    sig = {
        "kvf_init": (st, [C.c_int, C.POINTER(p)]),
        "kvf_destroy": (st, [p]),
        "kvf_last_error": (C.c_char_p, []),
        "kvf_abi_version": (C.c_int, []),
        "kvf_set_exact_reconstruct": (st, [p, C.c_int]),
        "kvf_set_reconstruct_engine": (st, [p, C.c_int]),
        "kvf_set_projection_engine": (st, [p, C.c_int]),
        "kvf_compress_layers": (st, [p, sz, p, p, i32, sz, sz, sz, p, C.POINTER(PipelineConfig), p, p, p, p, p, p]),
        "kvf_compressed_free_many": (st, [p, sz]),
        "kvf_selftest_wait_timeout": (st, [p, C.c_int, p]),
        "kvf_sync": (st, [p, p]),
        "kvf_pipeline_config_from_preset": (st, [i32, C.POINTER(PipelineConfig)]),
        "kvf_calibrate": (st, [p, p, i32, sz, sz, sz, sz, p, p]),
        "kvf_quantize": (st, [p, p, i32, sz, sz, sz, i32, i32, p, p, p, p]),
        "kvf_dequantize": (st, [p, p, sz, p, p, i32, i32, sz, sz, sz, p, p]),
        "kvf_project": (st, [p, p, i32, sz, sz, sz, p, p, sz, p, p]),
        "kvf_reconstruct": (st, [p, p, sz, sz, sz, sz, p, p, p, p]),
        "kvf_fused_project_quantize": (st, [p, p, i32, sz, sz, sz, p, p, sz, i32, i32, p, p, p, p]),
        "kvf_rans_max_encoded_len": (sz, [sz]),
        "kvf_rans_encode": (st, [p, p, sz, p, sz, szp, p, p]),
        "kvf_rans_decode": (st, [p, p, sz, p, sz, p, p]),
        "kvf_entropy_decode_dequant": (st, [p, p, sz, p, p, p, i32, i32, sz, sz, sz, p, p]),
        "kvf_fused_dequant_attention": (st, [p, p, p, p, p, p, p, p, i32, i32, sz, sz, sz, sz, sz, p, p, p, p,
                                             C.c_float, p, p]),
        "kvf_compressed_attention": (st, [p, p, p, C.c_float, p, p]),
        "kvf_basis_compute": (st, [p, p, i32, sz, sz, sz, f64, sz, C.POINTER(p), p]),
        "kvf_basis_from_host": (st, [p, sz, sz, sz, p, p, C.POINTER(p)]),
        "kvf_basis_info": (st, [p, szp, szp, szp]),
        "kvf_basis_download": (st, [p, p, p, p]),
        "kvf_basis_device_vt": (p, [p]),
        "kvf_basis_device_ranks": (p, [p]),
        "kvf_basis_free": (st, [p]),
        "kvf_compress_layer": (st, [p, p, p, i32, sz, sz, sz, sz, C.POINTER(PipelineConfig), p, p, C.POINTER(p), p]),
        "kvf_decompress_layer": (st, [p, p, p, p, p]),
        "kvf_compress_layer_host": (st, [p, p, p, i32, sz, sz, sz, sz, C.POINTER(PipelineConfig), p, p,
                                         C.POINTER(p), p]),
        "kvf_decompress_layer_host": (st, [p, p, p, p, p]),
        "kvf_compressed_shape": (st, [p, szp, szp, szp, szp]),
        "kvf_compressed_size_bytes": (st, [p, szp]),
        "kvf_original_size_bytes": (st, [p, szp]),
        "kvf_compression_ratio": (st, [p, C.POINTER(C.c_double)]),
        "kvf_compressed_tensor_info": (st, [p, i32, szp, szp, szp, C.POINTER(C.c_int32)]),
        "kvf_compressed_tensor_views": (st, [p, i32, C.POINTER(p), C.POINTER(p), C.POINTER(p), C.POINTER(p),
                                             C.POINTER(p), C.POINTER(p)]),
        "kvf_compressed_basis": (st, [p, i32, C.POINTER(p)]),
        "kvf_compressed_basis_bytes": (st, [p, szp]),
        "kvf_compressed_calibration": (p, [p]),
        "kvf_compressed_serialize": (st, [p, p, sz, szp]),
        "kvf_compressed_deserialize": (st, [p, p, sz, C.POINTER(p), p]),
        "kvf_compressed_free": (st, [p]),
        "kvf_bandwidth_bytes_per_us": (C.c_double, [i32]),
        "kvf_cost_measure": (st, [p, p, p, i32, sz, sz, sz, C.c_int, C.POINTER(PresetCost), p]),
        "kvf_cost_estimate": (st, [C.POINTER(PresetCost), sz, sz, i32, C.c_double, C.POINTER(CostEstimate)]),
        "kvf_cost_select": (st, [C.POINTER(PresetCost), sz, sz, C.c_double, C.c_double, C.POINTER(CostEstimate),
                                 szp]),
        "kvf_launch_count": (C.c_uint64, []),
        "kvf_stage_name": (C.c_char_p, [i32]),
        "kvf_profile_enable": (st, [p, C.c_int]),
        "kvf_profile_read": (st, [p, p, p, p]),
        "kvf_calibrate_noalloc": (st, [p, p, i32, sz, sz, sz, sz, p, p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def lib():
    """The loaded library (raises ImportError when it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise ImportError(f"{LIB_PATH} is missing; build it with `python -m kvforge_b200.build`")
                _lib = _declare(C.CDLL(LIB_PATH))
    return _lib


def check(status: int):
    if status != OK:
        msg = lib().kvf_last_error()
        raise KvForgeError(status, msg.decode() if msg else "")


_ctx = {}


def context(device: int = 0):
    """One kvf_ctx per device for the life of the process."""
    c = _ctx.get(device)
    if c is None:
        with _lock:
            c = _ctx.get(device)
            if c is None:
                h = C.c_void_p()
                check(lib().kvf_init(device, C.byref(h)))
                c = h
                _ctx[device] = c
    return c


def profile_read(device: int = 0) -> dict:
    """Per-stage {name: (ms, launches, algorithmic bytes)} since the last read."""
    import numpy as np
    ms = np.zeros(NUM_STAGES, np.float64)
    cnt = np.zeros(NUM_STAGES, np.uint64)
    by = np.zeros(NUM_STAGES, np.float64)
    check(lib().kvf_profile_read(context(device), ms.ctypes.data_as(C.c_void_p), cnt.ctypes.data_as(C.c_void_p),
                                 by.ctypes.data_as(C.c_void_p)))
    return {STAGES[i]: (float(ms[i]), int(cnt[i]), float(by[i])) for i in range(NUM_STAGES)}
