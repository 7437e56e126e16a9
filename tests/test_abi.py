"""CPU tests of the C ABI boundary: the library builds, loads without a GPU, and
exports exactly what include/mockbird_kv.h declares.  No compute calls."""
import ctypes
import os
import re
import subprocess

import pytest

from mockbird_b200 import _lib
from mockbird_b200.build import LIB, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mockbird_kv.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MB_API\s+[\w\s\*]+?\b(mb_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    for name in ["mb_create", "mb_destroy", "mb_reset", "mb_rope_append", "mb_attend", "mb_append_attend",
                 "mb_prefill", "mb_gather", "mb_sync", "mb_last_error"]:
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (mb_\w+)", out))
    declared = set(declared_symbols())
    assert declared <= exported, declared - exported
    # nothing but the declared C ABI is visible (the rest is hidden)
    assert {s for s in exported if s.startswith("mb_")} == declared


def test_python_bindings_cover_the_header(lib):
    assert set(_lib.SIGNATURES) == set(declared_symbols())
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_config_struct_layout_matches_header(lib):
    cfg = _lib.MbConfig()
    lib.mb_config_default(ctypes.byref(cfg))
    assert (cfg.layers, cfg.heads, cfg.head_dim, cfg.capacity) == (12, 12, 64, 570)  # gpu.ts:362 maxSlots
    assert cfg.dtype == _lib.MB_F32 and cfg.wrap == 0 and abs(cfg.rope_theta - 10000.0) < 1e-3
    assert ctypes.sizeof(_lib.MbConfig) == 11 * 4
    assert lib.mb_version().decode().startswith("mockbird-b200")


def test_create_reports_missing_device_or_bad_config(lib):
    cfg = _lib.MbConfig()
    lib.mb_config_default(ctypes.byref(cfg))
    cfg.head_dim = 32  # only 64 is supported
    h = ctypes.c_void_p()
    assert lib.mb_create(ctypes.byref(cfg), ctypes.byref(h)) == 1  # MB_ERR_ARG
    assert not h.value


def test_null_context_is_an_argument_error(lib):
    assert lib.mb_destroy(None) == 1
    assert lib.mb_sync(None, None) == 1
    assert lib.mb_reset(None, -1, None) == 1


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib._lib = None
        try:
            _lib.load(str(tmp_path / "libmockbird_kv.so"))
        finally:
            _lib._lib = None


def test_host_buffers_are_checked_before_the_call():
    """The host-array entry points read and write caller buffers through their
    addresses, so the Python mirror rejects a buffer of the wrong dtype, shape or
    layout (or one on the GPU) before the call."""
    import numpy as np
    import torch

    from mockbird_b200.engine import _host_array

    ok = np.zeros((2, 3), np.float32)
    assert _host_array("x", ok, (2, 3), "float32") is ok
    assert _host_array("x", torch.zeros(2, 3), (2, 3), "float32") is not None
    for bad in (np.zeros((2, 3), np.float64), np.zeros((3, 2), np.float32).T, np.zeros((2, 4), np.float32),
                torch.zeros(3, 2).t(), torch.zeros(2, 3, dtype=torch.int32), [[0.0] * 3] * 2):
        with pytest.raises(TypeError):
            _host_array("x", bad, (2, 3), "float32")


@pytest.mark.parametrize("field,offset", [("rope", 4), ("slot_pos", 2), ("status", 1), ("kv", 8),
                                          ("streams", 2), ("positions", 1), ("qkv", 8), ("out", 4)])
def test_noalloc_rejects_misaligned_pointers(lib, field, offset):
    """mb_append_attend_noalloc refuses, before any CUDA call, a pointer that its
    kernel would read with a wider access than the pointer's alignment allows
    (16-byte rows, 8-byte RoPE pairs, 4-byte ids and status atomics): MB_ERR_ARG
    instead of a misaligned access on the device.  No GPU is needed: with every
    pointer aligned the same call gets past the checks and fails at the device
    query (MB_ERR_CUDA here)."""
    base = 0x10000  # a fake 256-byte-aligned address; never dereferenced
    ring = _lib.MbRingRef(base, base, base, base, 1, 12, 64, 1, _lib.MB_F32, 1, 64)
    args = {"streams": base, "positions": base, "qkv": base, "out": base}
    if field in args:
        args[field] += offset
    else:
        setattr(ring, field, base + offset)
    rc = lib.mb_append_attend_noalloc(ctypes.byref(ring), 0, 1, args["streams"], args["positions"], args["qkv"],
                                      args["out"], None)
    assert rc == 1  # MB_ERR_ARG


def test_noalloc_checks_pass_for_aligned_pointers(lib):
    """The counterpart of the test above, on a machine without a GPU: aligned
    pointers pass every argument check and the call stops at the device query."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("only meaningful without a GPU (the call would otherwise run)")
    base = 0x10000
    ring = _lib.MbRingRef(base, base, base, base, 1, 12, 64, 1, _lib.MB_F32, 1, 64)
    assert lib.mb_append_attend_noalloc(ctypes.byref(ring), 0, 1, base, base, base, base, None) == 6  # MB_ERR_CUDA


def test_host_buffer_helpers():
    """The host-array wrappers read buffers through their addresses: inputs are
    used in place when they are C-contiguous fp32 (numpy or CPU torch) and copied
    otherwise; outputs are never copied; stream ids and positions must have one
    length (the C call reads n of each)."""
    import numpy as np
    import torch

    from mockbird_b200.engine import _host_addr, _host_ids, _host_input

    a = np.zeros((2, 3), np.float32)
    assert _host_input(a) is a and _host_addr("x", a, (2, 3), "float32") == a.ctypes.data
    t = torch.zeros(2, 3)
    assert _host_input(t) is t and _host_addr("x", t, (2, 3), "float32") == t.data_ptr()
    for conv in (np.zeros((2, 3)), np.zeros((3, 2), np.float32).T, torch.zeros(3, 2).t(), [[1, 2, 3], [4, 5, 6]]):
        c = _host_input(conv)
        assert _host_addr("x", c, (2, 3), "float32")
        assert np.array_equal(np.asarray(c), np.asarray(conv, np.float32))
    with pytest.raises(TypeError):
        _host_addr("out", np.zeros((3, 2), np.float32).T, (2, 3), "float32")
    s, p = _host_ids([3, 1], np.array([5, 6], np.int64))
    assert s.dtype == p.dtype == np.int32 and list(p) == [5, 6]
    with pytest.raises(ValueError):
        _host_ids([0, 1], [5])
    with pytest.raises(ValueError):
        _host_ids([[0, 1]], [[5, 6]])
