"""The C-ABI library loads and exports every symbol include/cherimoya_b200.h
declares; host-only queries work without a GPU."""

import ctypes
import os
import re

import pytest

from cherimoya_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "cherimoya_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(chm_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_expected_entry_points():
    syms = declared_symbols()
    assert sorted(_lib.EXPORTED) == syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_abi_version_and_error_strings():
    lib = _lib.load()
    assert lib.chm_abi_version() == _lib.ABI_VERSION
    assert _lib.error_string(0) == "ok"
    for s in range(1, 7):
        assert _lib.error_string(s) not in ("ok", "unknown status")
    assert _lib.error_string(99) == "unknown status"


def _desc(**kw):
    d = dict(n_filters=128, n_layers=9, expansion=2, n_outputs=1, n_groups=1,
             n_control_tracks=0, trimming=557, seq_len=2114, residual_scale=0.15, mode=1)
    d.update(kw)
    return _lib.make_desc(**d)


def test_validate_and_sizes():
    lib = _lib.load()
    d = _desc()
    assert lib.chm_validate(ctypes.byref(d)) == 0
    pk = lib.chm_packed_weights_bytes(ctypes.byref(d))
    assert pk > 9 * 2 * 128 * 256 * 2
    ws1 = lib.chm_forward_workspace_bytes(ctypes.byref(d), 1)
    ws2 = lib.chm_forward_workspace_bytes(ctypes.byref(d), 2)
    assert ws2 > ws1 > 2 * 2114 * 128 * 2
    d32 = _desc(mode=0)
    # fp32 activations: twice the bytes per sequence (bf16 mode also holds the
    # fixed-size partials of the fused statistics)
    ws32 = [lib.chm_forward_workspace_bytes(ctypes.byref(d32), n) for n in (1, 2)]
    assert ws32[1] - ws32[0] > ws2 - ws1
    assert lib.chm_ism_workspace_bytes(ctypes.byref(d), 4, 512) > 0
    assert lib.chm_variant_workspace_bytes(ctypes.byref(d), 10) > 0
    assert lib.chm_block_packed_bytes(128, 256) > 0
    assert lib.chm_block_workspace_bytes(2, 100, 128, 0) > 0


@pytest.mark.parametrize("kw,status", [
    (dict(n_filters=0), 1), (dict(mode=7), 1), (dict(trimming=1057), 2),
    (dict(seq_len=0), 1), (dict(n_outputs=0), 1), (dict(n_layers=-1), 1),
])
def test_validate_rejects(kw, status):
    lib = _lib.load()
    d = _desc(**kw)
    assert lib.chm_validate(ctypes.byref(d)) == status
    assert lib.chm_packed_weights_bytes(ctypes.byref(d)) == 0
    assert lib.chm_forward_workspace_bytes(ctypes.byref(d), 4) == 0


def test_calls_reject_null_pointers_without_touching_the_device():
    lib = _lib.load()
    d = _desc()
    assert lib.chm_forward(ctypes.byref(d), None, 1, None, 0, None, None, None, None, 0,
                           None) == 1
    assert lib.chm_ism(ctypes.byref(d), None, 1, None, 0, 10, 8, None, None, None, 0,
                       None) == 1
    assert lib.chm_block_forward(1, 10, 128, 256, 1, 0, None, None, None, None, 0, None) == 1
    assert lib.chm_block_forward(1, 10, 128, 256, 1, 5, None, None, None, None, 0, None) == 1
    assert lib.chm_ism_ex(ctypes.byref(d), None, 1, None, 0, 10, 8, None, None, None, None,
                          0, None) == 1
    # epilogues: null outputs/inputs, group sizes that do not cover the tracks
    assert lib.chm_wrapper_epilogue(ctypes.byref(d), 1, None, None, None, None, None, None, 0,
                                    None) == 1
    bogus = ctypes.c_void_p(16)              # never dereferenced: rejected first
    bad_groups = (ctypes.c_int32 * 1)(2)     # one track in the description, group of 2
    assert lib.chm_wrapper_epilogue(ctypes.byref(d), 1, bogus, bogus, bad_groups, bogus, None,
                                    None, 0, None) == 1
    assert lib.chm_wrapper_epilogue(ctypes.byref(d), 1, bogus, bogus, None, None, bogus, None,
                                    0, None) == 3   # the profile wrapper needs a workspace
