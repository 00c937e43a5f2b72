"""The C-ABI library loads on a CPU-only host and exports what the header declares.

No compute calls here: host-only plans (device < 0) exercise validation and
error mapping without a GPU.
"""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from paged_decode import _native
from paged_decode.layout import Layout

HEADER = Path(__file__).resolve().parents[1] / "include" / "paged_decode.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(pd_[a-z_]+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for required in ("pd_plan_create", "pd_plan_bind", "pd_decode", "pd_decode_with_stats",
                     "pd_merge_shards", "pd_gather_debug", "pd_plan_destroy", "pd_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) == set(_native.SIGNATURES)


def test_abi_version_and_status_strings():
    lib = _native.load()
    assert lib.pd_abi_version() == 8
    assert lib.pd_status_string(0) == b"ok"
    assert lib.pd_status_string(2) == b"invalid dtype"


def _create(layout, table, lengths, split=256, merge=0, device=-1, ctas=4):
    lib = _native.load()
    c_layout = _native.Layout(*layout)
    table = np.ascontiguousarray(table, dtype=np.int32)
    lengths = np.ascontiguousarray(lengths, dtype=np.int32)
    handle = ctypes.c_void_p()
    status = lib.pd_plan_create(ctypes.byref(c_layout), table.ctypes.data, table.shape[1],
                                lengths.ctypes.data, split, merge, 0, device, ctas, ctypes.byref(handle))
    return status, handle


@pytest.mark.parametrize("layout,table,lengths,split,merge,message", [
    ((1, 4, 2, 96, 16, 2), [[0, 1]], [1], 256, 0, "head_dim must be 64 or 128"),
    ((1, 4, 2, 64, 8, 2), [[0, 1]], [1], 256, 0, "page_size must be 16 or 32"),
    ((1, 3, 2, 64, 16, 2), [[0, 1]], [1], 256, 0, "divisible"),
    ((1, 4, 2, 64, 16, 2), [[0, 1]], [33], 256, 0, "capacity"),
    ((1, 4, 2, 64, 16, 2), [[0, 5]], [17], 256, 0, "outside physical cache"),
    ((1, 4, 2, 64, 16, 2), [[0, 1]], [1], 0, 0, "split_tokens"),
    ((1, 4, 2, 64, 16, 2), [[0, 1]], [1], 256, 3, "merge must be"),
    ((70000, 4, 2, 64, 16, 2), np.zeros((70000, 1)), np.zeros(70000), 256, 0, "grid limits"),
])
def test_create_rejects_like_the_reference(layout, table, lengths, split, merge, message):
    status, handle = _create(layout, table, lengths, split, merge)
    assert status == _native.PD_ERR_VALUE and not handle.value
    assert message in _native.load().pd_last_error().decode()
    with pytest.raises(ValueError, match=message):
        _native.check(status)


def test_host_only_plan_cannot_bind_or_launch():
    lib = _native.load()
    status, handle = _create((2, 8, 2, 128, 16, 4), [[0, 1], [2, 3]], [17, 32])
    assert status == _native.PD_OK
    try:
        assert lib.pd_plan_device_bytes(handle) > 0
        assert lib.pd_plan_bind(handle, 256, 1 << 20, None) == _native.PD_ERR_VALUE
        assert lib.pd_decode(handle, 16, 16, 16, 0, 16, None) == _native.PD_ERR_VALUE
        assert b"host-only" in lib.pd_last_error()
    finally:
        lib.pd_plan_destroy(handle)


def test_null_arguments_are_errors_not_crashes():
    lib = _native.load()
    assert lib.pd_plan_create(None, None, 0, None, 256, 0, 0, -1, 1, None) == _native.PD_ERR_VALUE
    assert lib.pd_plan_get_info(None, None) == _native.PD_ERR_VALUE
    assert lib.pd_decode(None, None, None, None, 0, None, None) == _native.PD_ERR_VALUE
    assert lib.pd_merge_shards(None, None, 1, 0, 1, 128, None, None) == _native.PD_ERR_VALUE
    assert lib.pd_plan_device_bytes(None) == 0
    lib.pd_plan_destroy(None)


def test_exception_mapping():
    with pytest.raises(TypeError):
        _native.check(_native.PD_ERR_TYPE)
    with pytest.raises(RuntimeError):
        _native.check(_native.PD_ERR_CUDA)
    with pytest.raises(RuntimeError):
        _native.check(_native.PD_ERR_UNBOUND)


def test_header_is_plain_c_and_links_from_c(tmp_path):
    """A C99 caller compiles against include/paged_decode.h, links the library
    and calls it (no GPU needed for the ABI version)."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    src = tmp_path / "caller.c"
    src.write_text('#include "paged_decode.h"\n'
                   "int main(void) { return pd_abi_version() == PD_ABI_VERSION ? 0 : 1; }\n")
    lib = Path(_native.LIB_PATH)
    exe = tmp_path / "caller"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-pedantic", f"-I{HEADER.parent}", str(src),
                    str(lib), f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], check=True)
    subprocess.run([str(exe)], check=True)


def test_exchange_buffer_size():
    """pd_exchange_bytes: launch counts (4 KiB after 256 B), then two parities of
    `world` slots of B*Hq*(D + 4) floats rounded up to 256 bytes."""
    lib = _native.load()
    layout = (3, 8, 2, 64, 16, 6)
    status, handle = _create(layout, np.arange(6, dtype=np.int32).reshape(3, 2), [17, 0, 32])
    assert status == 0
    try:
        slot = -(-(3 * 8 * (64 + 4) * 4) // 256) * 256
        for world in (1, 2, 8):
            assert lib.pd_exchange_bytes(handle, world) == 256 + 4096 + 2 * world * slot
        assert lib.pd_exchange_bytes(handle, 9) == 0 and lib.pd_exchange_bytes(None, 2) == 0
    finally:
        lib.pd_plan_destroy(handle)


def test_barrier_mode_and_counters_on_a_host_only_plan():
    """pd_plan_set_barrier accepts the three modes and nothing else; the counter
    reads and the barrier self-test reject what they cannot use without touching
    a GPU."""
    lib = _native.load()
    status, handle = _create((2, 8, 2, 128, 16, 4), [[0, 1], [2, 3]], [17, 32])
    assert status == _native.PD_OK
    try:
        for mode in (_native.PD_BARRIER_PLAIN, _native.PD_BARRIER_COOPERATIVE, _native.PD_BARRIER_LEAVE_AT_ONCE):
            assert lib.pd_plan_set_barrier(handle, mode) == _native.PD_OK
        for bad in (-1, 3, 99):
            assert lib.pd_plan_set_barrier(handle, bad) == _native.PD_ERR_VALUE
        count = ctypes.c_uint32(7)
        assert lib.pd_plan_read_barrier_fallbacks(handle, ctypes.byref(count), None) != _native.PD_OK
        assert count.value == 7                               # untouched on error
    finally:
        lib.pd_plan_destroy(handle)
    assert lib.pd_plan_set_barrier(None, 0) == _native.PD_ERR_VALUE
    outcomes = (ctypes.c_uint32 * 4)()
    assert lib.pd_selftest_barrier_leave(0, 0, outcomes) == _native.PD_ERR_VALUE        # leave_us 0
    assert lib.pd_selftest_barrier_leave(0, 200000, outcomes) == _native.PD_ERR_VALUE   # above 1e5
    assert lib.pd_selftest_barrier_leave(0, 200, None) == _native.PD_ERR_VALUE


def test_header_constants_match_the_python_binding():
    """Every #define the Python binding mirrors has the header's value."""
    import re
    from pathlib import Path
    text = (Path(__file__).resolve().parents[1] / "include" / "paged_decode.h").read_text()
    defines = {m.group(1): int(m.group(2), 0) for m in re.finditer(r"#define (PD_\w+) (0x[0-9a-fA-F]+|\d+)u?", text)}
    for name in ("PD_ENGINE_WARP", "PD_ENGINE_TCGEN05", "PD_BARRIER_PLAIN", "PD_BARRIER_COOPERATIVE",
                 "PD_BARRIER_LEAVE_AT_ONCE", "PD_DEVERR_TIMEOUT", "PD_DEVERR_BAD_PAGE"):
        assert defines[name] == getattr(_native, name), name
