"""The C-ABI library loads, exports every entry point its header declares,
and rejects bad arguments on the host before any CUDA call."""

from __future__ import annotations

import ctypes

import pytest

from ria_b200 import _ext


def test_library_exports_every_header_symbol():
    lib = _ext.lib()
    names = _ext.header_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(_ext._SIGNATURES), "every declared entry point has a ctypes signature"
    assert lib.ria_abi_version() == 1


def test_argument_errors_are_reported_without_a_gpu():
    lib = _ext.lib()
    rc = lib.ria_gdn_decode_step(*([None, 0] * 4), None, None, None, None, None, None, None, 0, None, 0, -1, None)
    assert rc == _ext.RIA_ERR_INVALID and "batch" in _ext.last_error()
    rc = lib.ria_gdn_decode_step(*([None, 0] * 4), None, None, None, None, None, None, None, 0, None, 0, 0, None)
    assert rc == 0  # empty batch is a no-op
    rc = lib.ria_gdn_decode_step(*([None, 0] * 4), None, None, None, None, None, None, None, 0, None, 0, 2, None)
    assert rc == _ext.RIA_ERR_INVALID and "null" in _ext.last_error()
    args = [None, 0, None, 0, None, 0, None, None, None, None, None, 64, None, 1, None, None, 0, 0, None, 0, None, 0,
            3, 1, 1, None]
    rc = lib.ria_gqa_decode_paged(*args)
    assert rc == _ext.RIA_ERR_INVALID
    assert lib.ria_rmsnorm_rows(None, 0, None, None, 0, 1, 3, None) == _ext.RIA_ERR_INVALID
    assert lib.ria_rope_apply(None, 1, 256, 63, None, 0, None) == _ext.RIA_ERR_INVALID


def test_workspace_and_split_helpers():
    assert _ext.gqa_workspace_bytes(1, 1) == 16 * 257 * 4
    assert _ext.gqa_workspace_bytes(0, 4) == 0
    assert _ext.gqa_split_pages(1, 2) == 1
    big = _ext.gqa_split_pages(10**6, 2)
    assert big > 1


def test_errors_map_to_python_exceptions():
    with pytest.raises(ValueError):
        _ext._check(_ext.RIA_ERR_INVALID, "x")
    with pytest.raises(RuntimeError):
        _ext._check(2, "x")
    _ext._check(0, "x")
    assert isinstance(_ext.lib(), ctypes.CDLL)


def test_new_entry_points_reject_bad_arguments_on_the_host():
    lib = _ext.lib()
    # kv append: null pointers, NULL seq_lens with batch > 1, a scalar length past the block table
    assert lib.ria_kv_append_paged(None, 512, None, 512, 0, None, None, 64, None, 1, None, 0, 2, None) == \
        _ext.RIA_ERR_INVALID
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf) // 256 * 256 + 256 if ctypes.addressof(buf) % 256 else ctypes.addressof(buf)
    assert lib.ria_kv_append_paged(p, 512, p, 512, 0, p, p, 64, p, 1, None, 0, 2, None) == _ext.RIA_ERR_INVALID
    assert "batch 1" in _ext.last_error()
    assert lib.ria_kv_append_paged(p, 512, p, 512, 0, p, p, 64, p, 1, None, 64, 1, None) == _ext.RIA_ERR_INVALID
    assert "block table" in _ext.last_error()
    assert lib.ria_kv_append_paged(p, 100, p, 512, 0, p, p, 64, p, 1, None, 0, 1, None) == _ext.RIA_ERR_INVALID
    assert lib.ria_kv_append_paged(None, 0, None, 0, 0, None, None, 0, None, 0, None, 0, 0, None) == 0  # empty batch
    # fp16 norm: bad sizes
    assert lib.ria_rmsnorm_rows_f16(None, 0, None, None, 0, 1, 3, None) == _ext.RIA_ERR_INVALID
    # GQA decode with scalar lengths: a split plan covering fewer pages than the sequence needs
    args = [p, 8192, p, 512, p, 512, p, p, p, p, p, 64 * 64, p, 64, None, None, 1000, 1000, p, 4096, p, 1 << 20,
            1, 2, 3, None]
    assert lib.ria_gqa_decode_paged(*args) == _ext.RIA_ERR_INVALID
    assert "pages" in _ext.last_error()
