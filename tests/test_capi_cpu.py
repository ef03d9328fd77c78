"""CPU checks of the C ABI: the library loads, exports every symbol the
header declares, and rejects invalid arguments before touching a device."""

import ctypes

import pytest

from vllm_ernie_b200 import _lib


def test_library_exports_every_header_symbol():
    decls = _lib.parse_header()
    assert len(decls) >= 20
    handle = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in decls if not hasattr(handle, n)]
    assert not missing, missing


def test_status_strings_and_version():
    lib = _lib.lib()
    assert lib.hca_version() >= 100
    for s in (0, -1, -2, -3, -4):
        assert lib.hca_status_string(s)
    assert lib.hca_status_string(-2) == b"shape not instantiated in this build"


def test_invalid_arguments_return_status_without_launch():
    lib = _lib.lib()
    # block_size 0 is rejected before any device work
    assert lib.hca_slot_mapping(None, None, None, None, 0, 1, 0, None) == -1
    # unsupported head dim
    assert lib.hca_quantize_insert_k(None, 64, 0, None, 0, None, 1, 96, 32, None) == -2
    # empty calls are no-ops
    assert lib.hca_token_to_req(None, None, 0, 0, None) == 0
    assert lib.hca_sparse_decode_workspace_bytes(64, 3, 64, 128, 1) == 0
    assert lib.hca_sparse_decode_workspace_bytes(64, 3, 64, 128, 4) > 64 * 4 * 192 * 128 * 4
    # split-K without workspace (pointers are placeholders: nothing launches)
    rc = lib.hca_sparse_decode(256, 64 * 128, 128, None, 256, 64 * 128, 128, 1, 64, 128, 64, 256, 64, 12416,
                               256, 128, 256, None, 2, 0, None, 0, None, None, 0, 1, 0.1, None, 4, None, 0,
                               None)
    assert rc == -4
    # misaligned output
    rc = lib.hca_sparse_decode(258, 64 * 128, 128, None, 256, 64 * 128, 128, 1, 64, 128, 64, 256, 64, 12416,
                               256, 128, 256, None, 2, 0, None, 0, None, None, 0, 1, 0.1, None, 1, None, 0,
                               None)
    assert rc == -1


def test_call_raises_on_error_status():
    with pytest.raises(_lib.HcaError):
        _lib.call("hca_slot_mapping", None, None, None, None, 0, 1, 0, None)
