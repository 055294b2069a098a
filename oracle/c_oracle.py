"""ctypes wrapper of ``kv_oracle.c`` working on torch CPU tensors or numpy arrays.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Each wrapper names the
reference lines it restates; arguments mirror the reference functions.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import build as _build


class Layout(ctypes.Structure):
    _fields_ = [
        ("kv_stride", ctypes.c_int64),
        ("layer_stride", ctypes.c_int64),
        ("block_stride", ctypes.c_int64),
        ("num_blocks", ctypes.c_int64),
        ("chunk_bytes", ctypes.c_int64),
        ("num_layers", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        h = ctypes.CDLL(str(path))
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        LP = ctypes.POINTER(Layout)
        h.kvo_pack_all_layer_blocks.argtypes = [vp, LP, vp, i64, vp, i32]
        h.kvo_unpack_all_layer_blocks.argtypes = [vp, i64, vp, LP, vp, i32]
        h.kvo_swap_planned.argtypes = [vp, LP, vp, vp, LP, vp, i64, vp, i32]
        h.kvo_store_kvcache.argtypes = [vp, vp, i64, i64, vp, vp, i64, i64, vp, i64, i64, i64, i64,
                                        ctypes.POINTER(i64)]
        for name in ("kvo_pack_all_layer_blocks", "kvo_unpack_all_layer_blocks", "kvo_swap_planned",
                     "kvo_store_kvcache"):
            getattr(h, name).restype = i32
        _lib = h
    return _lib


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1))


def layout_of_6d(cache: torch.Tensor) -> Layout:
    """Layout of a contiguous [2, L, N, bs, H, D] CPU tensor."""
    assert cache.dim() == 6 and cache.is_contiguous() and cache.device.type == "cpu"
    e = cache.element_size()
    _, L, N = cache.shape[:3]
    chunk = int(cache[0, 0, 0].numel()) * e
    return Layout(kv_stride=cache.stride(0) * e, layer_stride=cache.stride(1) * e, block_stride=cache.stride(2) * e,
                  num_blocks=N, chunk_bytes=chunk, num_layers=L, reserved=0)


def _ids(ids) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids, dtype=np.int64))


def pack_all_layer_blocks(cache: torch.Tensor, block_ids, nthreads: int = 1) -> torch.Tensor:
    """kv_transfer.py:229-248 on a 6-D CPU cache; returns [L, 2, B, bs, H, D]."""
    lay = layout_of_6d(cache)
    ids = _ids(block_ids)
    payload = torch.empty((lay.num_layers, 2, len(ids), *cache.shape[3:]), dtype=cache.dtype)
    rc = lib().kvo_pack_all_layer_blocks(cache.data_ptr(), ctypes.byref(lay), ids.ctypes.data, len(ids),
                                         payload.data_ptr(), nthreads)
    if rc:
        raise RuntimeError(f"oracle pack rejected the request (rc={rc})")
    return payload


def unpack_all_layer_blocks(payload: torch.Tensor, cache: torch.Tensor, block_ids, nthreads: int = 1) -> None:
    """kv_transfer.py:264-276 into a 6-D CPU cache (in place)."""
    lay = layout_of_6d(cache)
    ids = _ids(block_ids)
    if payload.shape[0] <= 0 or payload.shape[2] != len(ids):
        raise RuntimeError("packed multi-layer KV payload does not match destination blocks")
    payload = payload.contiguous()
    rc = lib().kvo_unpack_all_layer_blocks(payload.data_ptr(), len(ids), cache.data_ptr(), ctypes.byref(lay),
                                           ids.ctypes.data, nthreads)
    if rc:
        raise RuntimeError(f"oracle unpack rejected the request (rc={rc})")


def swap_planned(src_cache: torch.Tensor, src_ids, dst_cache: torch.Tensor, dst_ids, nthreads: int = 1,
                 payload: torch.Tensor | None = None) -> None:
    """kv_transfer.py:395-475 (negotiate_blocks=False) between two 6-D CPU caches."""
    sl, dl = layout_of_6d(src_cache), layout_of_6d(dst_cache)
    s, d = _ids(src_ids), _ids(dst_ids)
    if len(s) != len(d):
        raise RuntimeError("transfer_in negotiated mismatched block counts")
    ptr = payload.data_ptr() if payload is not None else None
    rc = lib().kvo_swap_planned(src_cache.data_ptr(), ctypes.byref(sl), s.ctypes.data, dst_cache.data_ptr(),
                                ctypes.byref(dl), d.ctypes.data, len(s), ptr, nthreads)
    if rc:
        raise RuntimeError(f"oracle swap rejected the request (rc={rc})")


def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  slot_mapping: torch.Tensor, block_size: int) -> int:
    """attention.py:67-108 on CPU tensors (in place); returns the count of rejected slots."""
    key, value = key.contiguous(), value.contiguous()
    T = key.shape[0]
    e = key.element_size()
    row = int(key[0].numel()) * e if T else 0
    slots = slot_mapping.to(torch.int64).contiguous()
    N = k_cache.shape[0]
    bad = ctypes.c_int64(0)
    if T == 0:
        return 0
    rc = lib().kvo_store_kvcache(key.data_ptr(), value.data_ptr(), key.stride(0) * e, value.stride(0) * e,
                                 k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0) * e,
                                 k_cache.stride(1) * e, slots.data_ptr(), T, N, block_size, row, ctypes.byref(bad))
    if rc:
        raise RuntimeError(f"oracle store_kvcache rejected the request (rc={rc})")
    return int(bad.value)
