"""The C-ABI library on the CPU: it loads, exports every symbol include/ygg_b200.h declares, and its host-side
validation answers with error codes (no GPU needed: parsing fails before any CUDA call)."""
import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT

from yggdrasil_b200 import _native, synth


def declared_symbols():
    text = (ROOT / "include" / "ygg_b200.h").read_text()
    return sorted(set(re.findall(r"\b(ygg_[a-z_]+)\s*\(", text)))


def test_header_declares_the_binding_exports():
    assert declared_symbols() == sorted(_native.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.ygg_version().decode().endswith("sm_100a")


def test_strerror_covers_every_code():
    for code in range(0, -11, -1):
        assert _native.strerror(code) != "unknown error"
    assert _native.strerror(-99) == "unknown error"


def _load(data, device=0):
    h = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(data), len(data))
    return _native.lib().ygg_load(buf, len(data), device, ctypes.byref(h)), h


def test_load_rejects_non_model_bytes():
    assert _load(b"not a model at all, just bytes" * 4)[0] == _native.YGG_E_FORMAT
    assert _load(b"YGG1")[0] == _native.YGG_E_FORMAT


def test_load_rejects_unsupported_header(tmp_path):
    p = tmp_path / "m.bin"
    synth.write_random_model(synth.ModelShape(64, 8, 3, 5, 2, 8, 0), p, seed=1)
    data = bytearray(p.read_bytes())
    data[8:12] = np.int32(80).tobytes()            # d_state 80: outside the YGG1 limits and the extension
    assert _load(data)[0] == _native.YGG_E_UNSUPPORTED
    data[8:12] = np.int32(96).tobytes()            # the extension's d_state, but arrays sized for 64
    assert _load(data)[0] == _native.YGG_E_MISSING
    data[8:12] = np.int32(64).tobytes()
    data[20:24] = np.int32(12).tobytes()           # readout rank 12 with arrays of rank 8
    assert _load(data)[0] == _native.YGG_E_MISSING


def test_load_rejects_truncated_arrays(tmp_path):
    p = tmp_path / "m.bin"
    synth.write_random_model(synth.ModelShape(64, 8, 3, 5, 2, 8, 0), p, seed=1)
    data = p.read_bytes()
    assert _load(data[: len(data) // 2])[0] == _native.YGG_E_FORMAT


def test_load_rejects_a_missing_array(tmp_path):
    p = tmp_path / "m.bin"
    synth.write_random_model(synth.ModelShape(64, 8, 3, 5, 2, 8, 0), p, seed=1)
    data = bytearray(p.read_bytes())
    i = data.find(b"l1_w\0")
    data[i:i + 4] = b"l1_X"                          # rename the router rows of layer 1
    assert _load(data)[0] == _native.YGG_E_MISSING


def test_load_without_device_reports_it(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    p = tmp_path / "m.bin"
    synth.write_random_model(synth.ModelShape(64, 8, 3, 5, 2, 8, 0), p, seed=1)
    assert _load(p.read_bytes())[0] == _native.YGG_E_DEVICE


def test_null_arguments():
    lib = _native.lib()
    assert lib.ygg_load(None, 0, 0, None) == _native.YGG_E_ARG
    assert lib.ygg_step(None, 1, None, None, None, None, None) == _native.YGG_E_ARG
    assert lib.ygg_score(None, 1, 1, None, None, None, None) == _native.YGG_E_ARG
    lib.ygg_free(None)


def test_selftest_wait_arguments():
    lib = _native.lib()
    status = ctypes.c_int(7)
    assert lib.ygg_selftest_wait(0, -1, None, ctypes.byref(status)) == _native.YGG_E_ARG
    assert lib.ygg_selftest_wait(0, 1000, None, None) == _native.YGG_E_ARG
