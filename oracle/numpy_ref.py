"""Plain-numpy restatement of LMPool's KV data path, for small cases.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``). Arrays are raw
element bits (e.g. ``uint16`` for bf16) so every comparison is bit-exact.
Shapes follow the reference: cache ``[2, L, N, bs, H, D]``
(model_runner.py:397-400), payload ``[L, 2, B, bs, H, D]`` (kv_transfer.py:236-240).
"""
from __future__ import annotations

import numpy as np


def pack_all_layer_blocks(cache: np.ndarray, block_ids) -> np.ndarray:
    """kv_transfer.py:229-248: payload[l, kv] = cache[kv, l][ids]."""
    ids = np.asarray(list(block_ids), dtype=np.int64)
    L = cache.shape[1]
    payload = np.empty((L, 2, len(ids), *cache.shape[3:]), dtype=cache.dtype)
    for layer in range(L):
        payload[layer, 0] = cache[0, layer][ids]
        payload[layer, 1] = cache[1, layer][ids]
    return payload


def unpack_all_layer_blocks(payload: np.ndarray, cache: np.ndarray, block_ids) -> None:
    """kv_transfer.py:264-276 / :199-215: cache[kv, l][ids] = payload[l, kv]."""
    ids = np.asarray(list(block_ids), dtype=np.int64)
    if payload.shape[0] <= 0 or payload.shape[2] != len(ids):
        raise RuntimeError("packed multi-layer KV payload does not match destination blocks")
    if len(set(ids.tolist())) != len(ids):
        raise RuntimeError("destination block ids must be distinct")
    for layer in range(payload.shape[0]):
        cache[0, layer][ids] = payload[layer, 0]
        cache[1, layer][ids] = payload[layer, 1]


def swap_planned(src_cache: np.ndarray, src_ids, dst_cache: np.ndarray, dst_ids) -> None:
    """kv_transfer.py:395-475 with negotiate_blocks=False (send/recv = copy)."""
    if len(list(src_ids)) != len(list(dst_ids)):
        raise RuntimeError("transfer_in negotiated mismatched block counts")
    payload = pack_all_layer_blocks(src_cache, src_ids)
    unpack_all_layer_blocks(payload.copy(), dst_cache, dst_ids)


def store_kvcache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
                  slot_mapping: np.ndarray, block_size: int) -> None:
    """attention.py:24-64: flat index (slot//bs)*bs*H*D + (slot%bs)*H*D + h*D + d."""
    N = k_cache.shape[0]
    kflat = k_cache.reshape(N * block_size, -1)
    vflat = v_cache.reshape(N * block_size, -1)
    for t, slot in enumerate(np.asarray(slot_mapping, dtype=np.int64).tolist()):
        if slot == -1:
            continue
        blk, off = slot // block_size, slot % block_size
        row = blk * block_size + off
        kflat[row] = key[t].reshape(-1)
        vflat[row] = value[t].reshape(-1)
