"""Drop-in ``store_kvcache`` (src/lmpool/layers/attention.py:67-108) on B200.

The reference launches a Triton program per (token, kv head) that copies
``head_dim`` elements of K and V into ``cache[slot // bs, slot % bs, h]``
(attention.py:7-64). Here one sm_100a kernel moves a token's whole row
(all heads: ``kv_heads * head_dim`` contiguous elements, e.g. 2 KiB) per warp
with 16-byte vectors, K and V on neighbouring warps. ``store_kvcache_layers``
writes every layer of a step in one launch.

Both run on the current CUDA stream, never synchronise and never allocate,
so they can be captured in a CUDA graph (model_runner.py:630-683). Slots
outside ``[-1, num_blocks * block_size)`` are skipped and recorded in a
per-device status word (``kv_transfer.check_device_status``); the reference
kernel would write out of bounds for them.
"""
from __future__ import annotations

import torch

from . import _capi
from .kv_transfer import _status_word


def _cache_strides(k_cache: torch.Tensor, v_cache: torch.Tensor) -> tuple[int, int]:
    if k_cache.dim() != 4:
        raise RuntimeError("k_cache must be [num_blocks, block_size, num_kv_heads, head_dim]")
    st = k_cache.stride()
    if st != v_cache.stride():
        raise RuntimeError("k_cache and v_cache must have the same strides")
    H, D = k_cache.shape[2], k_cache.shape[3]
    if st[3] != 1 or (H > 1 and st[2] != D):
        raise RuntimeError("each cache slot [num_kv_heads, head_dim] must be contiguous")
    e = k_cache.element_size()
    return st[0] * e, st[1] * e


def _device_of(*tensors: torch.Tensor) -> int:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError("store_kvcache needs CUDA tensors: the B200 path has no CPU implementation")
    for t in tensors[1:]:
        if t.device != dev:
            raise RuntimeError(f"all tensors must be on {dev}, got {t.device}")
    return dev.index if dev.index is not None else torch.cuda.current_device()


def _raw_stream(device: int) -> int:
    """cudaStream_t of the current stream (cheap path; capture streams included)."""
    try:
        return torch._C._cuda_getCurrentRawStream(device)
    except AttributeError:
        return torch.cuda.current_stream(device).cuda_stream


def store_kvcache(
    key: torch.Tensor,
    value: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
) -> None:
    """attention.py:67-108: ``cache[slot // bs, slot % bs] = key[t]`` for every slot != -1."""
    num_tokens, num_kv_heads, head_dim = key.shape
    if not key.is_contiguous():
        key = key.contiguous()
    if not value.is_contiguous():
        value = value.contiguous()
    assert k_cache.shape == v_cache.shape, "K and V cache shapes must match"
    assert slot_mapping.numel() == num_tokens, "Slot mapping size must match number of tokens"
    if slot_mapping.dtype != torch.int64:
        raise TypeError(f"slot_mapping must be int64, got {slot_mapping.dtype}")
    if key.dtype != k_cache.dtype or value.dtype != v_cache.dtype:
        raise TypeError("key/value and cache dtypes must match (the copy is bit-exact)")
    kshape = k_cache.shape
    if kshape[2] != num_kv_heads or kshape[3] != head_dim or value.shape != key.shape:
        raise RuntimeError("key/value [T, H, D] must match the cache's [H, D]")
    device = _device_of(key, value, k_cache, v_cache, slot_mapping)
    if num_tokens == 0:
        return
    if not slot_mapping.is_contiguous():
        slot_mapping = slot_mapping.contiguous()
    block_stride, slot_stride = _cache_strides(k_cache, v_cache)
    e = key.element_size()
    rc = _capi.lib().kvx_store_kvcache(
        device, key.data_ptr(), value.data_ptr(), key.stride(0) * e, value.stride(0) * e, k_cache.data_ptr(),
        v_cache.data_ptr(), block_stride, slot_stride, slot_mapping.data_ptr(), num_tokens, kshape[0],
        int(block_size), num_kv_heads * head_dim * e, _status_word(device).data_ptr(), _raw_stream(device))
    if rc:
        _capi.check(rc, "kvx_store_kvcache")


def store_kvcache_layers(
    keys: torch.Tensor,
    values: torch.Tensor,
    kv_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
) -> None:
    """Every layer in one launch.

    ``keys``/``values``: ``[L, T, H, D]`` (each layer's token rows contiguous);
    ``kv_cache``: the ``[2, L, N, bs, H, D]`` tensor of model_runner.py:397-400.
    Equivalent to ``store_kvcache(keys[l], values[l], kv_cache[0, l],
    kv_cache[1, l], slot_mapping, block_size)`` for every l.
    """
    if kv_cache.dim() != 6:
        raise RuntimeError("kv_cache must be [2, L, N, block_size, H, D]")
    L, T, H, D = keys.shape
    if values.shape != keys.shape:
        raise RuntimeError("keys and values must have the same shape")
    if tuple(kv_cache.shape[1:2]) != (L,) or tuple(kv_cache.shape[4:]) != (H, D):
        raise RuntimeError("keys [L, T, H, D] do not match kv_cache [2, L, N, bs, H, D]")
    assert slot_mapping.numel() == T, "Slot mapping size must match number of tokens"
    if slot_mapping.dtype != torch.int64:
        raise TypeError(f"slot_mapping must be int64, got {slot_mapping.dtype}")
    if keys.dtype != kv_cache.dtype or values.dtype != kv_cache.dtype:
        raise TypeError("key/value and cache dtypes must match (the copy is bit-exact)")
    for name, t in (("keys", keys), ("values", values)):
        if t.stride(3) != 1 or (H > 1 and t.stride(2) != D):
            raise RuntimeError(f"{name}: each token row [H, D] must be contiguous")
    device = _device_of(keys, values, kv_cache, slot_mapping)
    if T == 0:
        return
    slot_mapping = slot_mapping.contiguous()
    k0, v0 = kv_cache[0, 0], kv_cache[1, 0]
    block_stride, slot_stride = _cache_strides(k0, v0)
    e = keys.element_size()
    rc = _capi.lib().kvx_store_kvcache_layers(
        device, L, keys.data_ptr(), values.data_ptr(), keys.stride(0) * e, values.stride(0) * e, keys.stride(1) * e,
        values.stride(1) * e, k0.data_ptr(), v0.data_ptr(), kv_cache.stride(1) * e, kv_cache.stride(1) * e,
        block_stride, slot_stride, slot_mapping.data_ptr(), T, kv_cache.shape[2], int(block_size), H * D * e,
        _status_word(device).data_ptr(), _raw_stream(device))
    if rc:
        _capi.check(rc, "kvx_store_kvcache_layers")
