"""ctypes binding of the C ABI in ``include/kvx.h`` (library ``_kvx.so``).

Only plain integers and pointers cross this boundary; tensors are reduced
to ``data_ptr()`` and byte strides by the callers. Every non-zero status is
raised as :class:`KvxError` (a ``RuntimeError``, so LMPool's executor turns
it into ``{"success": False, "reason": "executor_error"}`` unchanged,
control_plane.py:544-559).

There is no fallback: if the library is missing or was built for another
ABI version, importing the transfer path raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_LIB_PATH = Path(__file__).resolve().parent / "_kvx.so"
ABI_VERSION = 2

KVX_OK = 0
KVX_EINVAL = 1
KVX_ENOMEM = 2
KVX_ETIMEDOUT = 3
KVX_EPEER = 4
KVX_ECUDA = 5
KVX_EUNSUPPORTED = 6
NOALLOC_MAX_PEERS = 64

DEV_BAD_SRC_ID = 0x01
DEV_BAD_DST_ID = 0x02
DEV_BAD_SLOT = 0x04
DEV_TIMEOUT = 0x08
DEV_COUNT_MISMATCH = 0x10
DEV_PEER_FAILED = 0x20
DEV_PIPE_TIMEOUT = 0x40

_DEV_BITS = {
    DEV_BAD_SRC_ID: "source block id out of range",
    DEV_BAD_DST_ID: "destination block id out of range",
    DEV_BAD_SLOT: "slot_mapping entry out of range",
    DEV_TIMEOUT: "timed out waiting for the peer",
    DEV_COUNT_MISMATCH: "peer posted a different block count",
    DEV_PEER_FAILED: "peer reported failure",
    DEV_PIPE_TIMEOUT: "bulk-copy pipeline wait ran out",
}


class KvxError(RuntimeError):
    """A C-ABI call or a kernel reported failure."""

    def __init__(self, message: str, status: int = 0, device_bits: int = 0):
        super().__init__(message)
        self.status = status
        self.device_bits = device_bits


def describe_device_status(bits: int) -> str:
    names = [text for bit, text in _DEV_BITS.items() if bits & bit]
    unknown = bits & ~sum(_DEV_BITS)
    if unknown:
        names.append(f"unknown bits 0x{unknown:x}")
    return ", ".join(names) if names else "ok"


class CacheDesc(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_uint64),
        ("kv_stride", ctypes.c_int64),
        ("layer_stride", ctypes.c_int64),
        ("block_stride", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("chunk_bytes", ctypes.c_int64),
        ("num_layers", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class Mailbox(ctypes.Structure):
    _fields_ = [
        ("base", ctypes.c_uint64),
        ("max_peers", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("max_blocks", ctypes.c_int64),
    ]


class PushTarget(ctypes.Structure):
    _fields_ = [
        ("dst", CacheDesc),
        ("dst_mailbox", Mailbox),
        ("src_ids_dev", ctypes.c_void_p),
        ("num_ids", ctypes.c_int64),
        ("dst_rank", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class PullSource(ctypes.Structure):
    _fields_ = [
        ("src", CacheDesc),
        ("src_mailbox", Mailbox),
        ("src_ids_dev", ctypes.c_void_p),
        ("dst_ids_dev", ctypes.c_void_p),
        ("num_ids", ctypes.c_int64),
        ("token", ctypes.c_uint64),
        ("src_rank", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class Tuning(ctypes.Structure):
    _fields_ = [
        ("variant", ctypes.c_int32),
        ("ctas_per_sm", ctypes.c_int32),
        ("tile_bytes", ctypes.c_int32),
        ("stages", ctypes.c_int32),
        ("store_pdl", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_vp = ctypes.c_void_p
_P = ctypes.POINTER

# name -> (restype, argtypes); the exact list of entry points in kvx.h.
SIGNATURES: dict[str, tuple] = {
    "kvx_abi_version": (_i32, []),
    "kvx_last_error": (ctypes.c_char_p, []),
    "kvx_status_name": (ctypes.c_char_p, [_i32]),
    "kvx_set_tuning": (_i32, [_P(Tuning)]),
    "kvx_get_tuning": (_i32, [_P(Tuning)]),
    "kvx_validate_block_ids": (_i32, [_vp, _i64, _i64, _i32]),
    "kvx_ids_overlap": (_i32, [_vp, _i64, _vp, _i64, _i64, _P(_i32)]),
    "kvx_check_desc": (_i32, [_P(CacheDesc)]),
    "kvx_device_count": (_i32, [_P(_i32)]),
    "kvx_device_sm_count": (_i32, [_i32, _P(_i32)]),
    "kvx_can_access_peer": (_i32, [_i32, _i32, _P(_i32)]),
    "kvx_move_blocks": (_i32, [_i32, _P(CacheDesc), _P(CacheDesc), _vp, _vp, _i64, _vp, _vp]),
    "kvx_pair_publish": (_i32, [_i32, _P(Mailbox), _i32, _vp, _i64, _u64, _vp]),
    "kvx_pair_wait_done": (_i32, [_i32, _P(Mailbox), _i32, _u64, _u64, _vp, _vp]),
    "kvx_pair_wait_armed": (_i32, [_i32, _P(Mailbox), _P(Mailbox), _i32, _i32, _i64, _u64, _vp, _vp]),
    "kvx_pair_push": (_i32, [_i32, _P(CacheDesc), _P(Mailbox), _i32, _P(PushTarget), _i32, _vp, _vp]),
    "kvx_pair_request": (_i32, [_i32, _P(Mailbox), _i32, _i64, _u64, _vp]),
    "kvx_pair_grant": (_i32, [_i32, _P(Mailbox), _P(Mailbox), _i32, _i32, _i64, _u64, _vp, _vp]),
    "kvx_pair_pull": (_i32, [_i32, _P(CacheDesc), _P(Mailbox), _i32, _P(PullSource), _i32, _vp, _vp]),
    "kvx_pair_wait_pulled": (_i32, [_i32, _P(Mailbox), _i32, _u64, _vp, _vp]),
    "kvx_pair_push_noalloc": (_i32, [_i32, _P(CacheDesc), _P(Mailbox), _i32, _P(PushTarget), _i32, _vp, _vp]),
    "kvx_mailbox_bytes": (_i32, [_i32, _i64, _P(_u64)]),
    "kvx_mailbox_create": (_i32, [_i32, _i32, _i64, _P(Mailbox)]),
    "kvx_mailbox_destroy": (_i32, [_i32, _P(Mailbox)]),
    "kvx_mailbox_read_done": (_i32, [_i32, _P(Mailbox), _i32, _P(_u64)]),
    "kvx_mailbox_reset_peer": (_i32, [_i32, _P(Mailbox), _i32, _vp]),
    "kvx_ipc_export": (_i32, [_i32, _vp, _vp, _P(_u64)]),
    "kvx_ipc_open": (_i32, [_i32, _vp, _u64, _P(_u64)]),
    "kvx_ipc_close": (_i32, [_i32, _u64, _u64]),
    "kvx_enable_peer_access": (_i32, [_i32, _i32]),
    "kvx_store_kvcache": (
        _i32,
        [_i32, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _i32, _i64, _vp, _vp],
    ),
    "kvx_store_kvcache_layers": (
        _i32,
        [_i32, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i32,
         _i64, _vp, _vp],
    ),
    "kvx_wait_flag": (_i32, [_i32, _vp, _u64, _u64, _vp, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def library_path() -> Path:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load ``_kvx.so`` (once). Raises if it is missing or mismatched."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _LIB_PATH.exists():
            raise ImportError(
                f"{_LIB_PATH} is missing: build it with `python -m lmpool_b200._build` "
                "(the KV data path has no CPU or PyTorch fallback)"
            )
        handle = ctypes.CDLL(str(_LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = handle.kvx_abi_version()
        if version != ABI_VERSION:
            raise ImportError(f"{_LIB_PATH} has ABI version {version}, expected {ABI_VERSION}: rebuild it")
        _lib = handle
        return _lib


def last_error() -> str:
    msg = lib().kvx_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str) -> None:
    if rc != KVX_OK:
        name = lib().kvx_status_name(rc).decode()
        raise KvxError(f"{what} failed: {name}: {last_error()}", status=rc)


def stream_handle(stream) -> int:
    """cudaStream_t of a torch.cuda.Stream (0 = legacy default stream)."""
    return int(stream.cuda_stream) if stream is not None else 0
