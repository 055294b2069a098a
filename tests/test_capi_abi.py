"""The C-ABI library loads without a GPU and exports exactly what include/kvx.h declares.

No kernel runs here; only host-side entry points (validation, tuning,
status names) are called.
"""
import ctypes
import re
from pathlib import Path

import pytest

from lmpool_b200 import _capi

HEADER = Path(__file__).resolve().parent.parent / "include" / "kvx.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kvx_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_binding_table():
    assert declared_functions() == sorted(_capi.SIGNATURES)


def test_library_exports_every_declared_symbol(kvx_lib):
    for name in declared_functions():
        assert hasattr(kvx_lib, name), name


def test_abi_version_and_status_names(kvx_lib):
    assert kvx_lib.kvx_abi_version() == _capi.ABI_VERSION
    assert kvx_lib.kvx_status_name(_capi.KVX_EINVAL) == b"KVX_EINVAL"
    assert kvx_lib.kvx_status_name(99) == b"KVX_UNKNOWN"


def _ids(values):
    return (ctypes.c_int64 * max(1, len(values)))(*values)


def test_validate_block_ids(kvx_lib):
    assert kvx_lib.kvx_validate_block_ids(_ids([0, 3, 3]), 3, 4, 0) == _capi.KVX_OK
    assert kvx_lib.kvx_validate_block_ids(_ids([0, 3, 3]), 3, 4, 1) == _capi.KVX_EINVAL
    assert b"more than once" in kvx_lib.kvx_last_error()
    assert kvx_lib.kvx_validate_block_ids(_ids([0, 4]), 2, 4, 0) == _capi.KVX_EINVAL
    assert b"outside [0, 4)" in kvx_lib.kvx_last_error()
    assert kvx_lib.kvx_validate_block_ids(_ids([-1]), 1, 4, 0) == _capi.KVX_EINVAL
    assert kvx_lib.kvx_validate_block_ids(_ids([]), 0, 4, 1) == _capi.KVX_OK


def test_ids_overlap(kvx_lib):
    out = ctypes.c_int32(-1)
    assert kvx_lib.kvx_ids_overlap(_ids([1, 2]), 2, _ids([3, 2]), 2, 8, ctypes.byref(out)) == 0
    assert out.value == 1
    assert kvx_lib.kvx_ids_overlap(_ids([1, 2]), 2, _ids([3, 4]), 2, 8, ctypes.byref(out)) == 0
    assert out.value == 0


def test_check_desc_rejects_bad_layouts(kvx_lib):
    good = _capi.CacheDesc(base=1 << 20, kv_stride=64, layer_stride=128, block_stride=16, num_blocks=4,
                           chunk_bytes=16, num_layers=2, reserved=0)
    assert kvx_lib.kvx_check_desc(ctypes.byref(good)) == 0
    for field, value in (("base", 0), ("num_layers", 0), ("num_blocks", 0), ("chunk_bytes", 0), ("reserved", 1)):
        bad = _capi.CacheDesc.from_buffer_copy(good)
        setattr(bad, field, value)
        assert kvx_lib.kvx_check_desc(ctypes.byref(bad)) == _capi.KVX_EINVAL, field


def test_tuning_roundtrip_and_validation(kvx_lib):
    old = _capi.Tuning()
    assert kvx_lib.kvx_get_tuning(ctypes.byref(old)) == 0
    try:
        t = _capi.Tuning(variant=2, ctas_per_sm=1, tile_bytes=32768, stages=8, store_pdl=2)
        assert kvx_lib.kvx_set_tuning(ctypes.byref(t)) == 0
        back = _capi.Tuning()
        kvx_lib.kvx_get_tuning(ctypes.byref(back))
        assert (back.variant, back.ctas_per_sm, back.tile_bytes, back.stages, back.store_pdl) == (2, 1, 32768, 8, 2)
        assert kvx_lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(variant=3))) == _capi.KVX_EINVAL
        assert kvx_lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(tile_bytes=100))) == _capi.KVX_EINVAL
        assert kvx_lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(stages=5))) == _capi.KVX_EINVAL
        assert kvx_lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(store_pdl=3))) == _capi.KVX_EINVAL
        assert kvx_lib.kvx_set_tuning(ctypes.byref(_capi.Tuning(reserved=1))) == _capi.KVX_EINVAL
    finally:
        kvx_lib.kvx_set_tuning(ctypes.byref(old))


def test_mailbox_bytes(kvx_lib):
    out = ctypes.c_uint64(0)
    assert kvx_lib.kvx_mailbox_bytes(8, 1536, ctypes.byref(out)) == 0
    assert out.value >= 8 * 1536 * 8 and out.value % 8 == 0
    assert kvx_lib.kvx_mailbox_bytes(0, 1, ctypes.byref(out)) == _capi.KVX_EINVAL


def test_launch_entry_points_validate_before_touching_a_gpu(kvx_lib):
    # Argument checks run first, so these return EINVAL even without a device.
    desc = _capi.CacheDesc(base=0, num_layers=1, num_blocks=1, chunk_bytes=16)
    assert kvx_lib.kvx_move_blocks(0, ctypes.byref(desc), ctypes.byref(desc), None, None, 1, None, None) == \
        _capi.KVX_EINVAL
    mb = _capi.Mailbox()
    assert kvx_lib.kvx_pair_publish(0, ctypes.byref(mb), 0, None, 0, 1, None) == _capi.KVX_EINVAL
    good = _capi.Mailbox(base=1 << 20, max_peers=2, reserved=0, max_blocks=8)
    # pull request: token 0 and tokens with the FAIL bit are refused, counts are bounded by the mailbox
    assert kvx_lib.kvx_pair_request(0, ctypes.byref(good), 0, 4, 0, None) == _capi.KVX_EINVAL
    assert kvx_lib.kvx_pair_request(0, ctypes.byref(good), 0, 4, 1 << 63, None) == _capi.KVX_EINVAL
    assert kvx_lib.kvx_pair_request(0, ctypes.byref(good), 0, 9, 1, None) == _capi.KVX_EINVAL
    assert kvx_lib.kvx_pair_request(0, ctypes.byref(good), 2, 4, 1, None) == _capi.KVX_EINVAL
    # grant: a status word is required, ranks must fit both mailboxes
    assert kvx_lib.kvx_pair_grant(0, ctypes.byref(good), ctypes.byref(good), 0, 1, 4, 10, None, None) == \
        _capi.KVX_EINVAL
    assert kvx_lib.kvx_pair_grant(0, ctypes.byref(good), ctypes.byref(good), 0, 5, 4, 10, 8, None) == \
        _capi.KVX_EINVAL
    assert kvx_lib.kvx_pair_grant(0, ctypes.byref(good), ctypes.byref(good), 0, 1, -1, 10, 8, None) == \
        _capi.KVX_EINVAL
    assert kvx_lib.kvx_mailbox_reset_peer(0, ctypes.byref(good), 2, None) == _capi.KVX_EINVAL
    assert kvx_lib.kvx_mailbox_reset_peer(0, ctypes.byref(mb), 0, None) == _capi.KVX_EINVAL
    assert kvx_lib.kvx_store_kvcache(0, None, None, 0, 0, None, None, 0, 0, None, 1, 0, 16, 16, None, None) == \
        _capi.KVX_EINVAL


def test_error_messages_are_thread_local_strings(kvx_lib):
    kvx_lib.kvx_validate_block_ids(_ids([9]), 1, 4, 0)
    assert isinstance(_capi.last_error(), str) and "9" in _capi.last_error()


def test_check_raises_runtime_error():
    with pytest.raises(RuntimeError):
        _capi.check(_capi.KVX_EINVAL, "something")
