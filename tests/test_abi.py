"""CPU tests of the C-ABI library: it loads, exports every symbol that
include/kvforge.h declares, and its host-only entry points behave like the
reference's PipelineConfig::from_preset and error mapping. No kernel runs."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "kvforge.h")).read()
    return sorted(set(re.findall(r"\b(kvf_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from kvforge_b200 import _lib as L
    lib = L.lib()
    declared = _declared()
    assert len(declared) >= 38
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(L.EXPORTS) == declared


def test_abi_version():
    from kvforge_b200 import _lib as L
    assert L.lib().kvf_abi_version() == 1


@pytest.mark.parametrize("name,expect", [
    ("conservative", (1, 1, 0, 0.99, 0, 0)),
    ("balanced", (0, 0, 1, 0.90, 0, 0)),
    ("aggressive", (0, 0, 1, 0.75, 1, 1)),
    ("adaptive", (0, 0, 1, 0.90, 1, 1)),
])
def test_presets_match_reference(name, expect):  # crates/kvforge-core/src/pipeline.rs:31-70
    import kvforge_b200 as K
    c = K.config_from_preset(name.upper())
    got = (c.key_data_type, c.value_data_type, c.enable_projection, c.projection_variance_threshold,
           c.enable_entropy_coding, c.enable_calibration)
    assert got == expect


def test_bad_preset_and_shapes():
    import numpy as np
    import kvforge_b200 as K
    with pytest.raises(ValueError, match="Unknown preset"):
        K.parse_preset("turbo")
    with pytest.raises(ValueError, match="same shape"):
        K.KVCache(np.zeros((2, 3, 4), np.float32), np.zeros((2, 3, 5), np.float32), 0)
    kv = K.KVCache(np.zeros((2, 3, 4), np.float32), np.zeros((2, 3, 4), np.float32), 7)
    assert kv.shape == (2, 3, 4) and kv.layer_idx == 7 and kv.size_bytes() == 2 * 24 * 4
    from kvforge_b200 import _lib as L
    cfg = L.PipelineConfig()
    assert L.lib().kvf_pipeline_config_from_preset(9, C.byref(cfg)) == L.ERR_INVALID_CONFIG
    assert b"preset" in L.lib().kvf_last_error()
    with pytest.raises(L.KvForgeError) as e:
        L.check(L.ERR_INVALID_CONFIG)
    assert e.value.status == L.ERR_INVALID_CONFIG


def test_init_without_device_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    from kvforge_b200 import _lib as L
    h = C.c_void_p()
    assert L.lib().kvf_init(0, C.byref(h)) == L.ERR_CUDA


def test_rans_capacity_formula():
    from kvforge_b200 import _lib as L
    from oracle import oracle as O
    for n in (0, 1, 100, 8192, 8193, 16384, 16385, 10 ** 6):
        assert L.lib().kvf_rans_max_encoded_len(n) == O.lib().orc_rans_max_encoded_len(n, O.DEFAULT_CHUNK)
