"""KV-cache layout normalisation: tensors -> ``kvx_cache_desc``.

LMPool hands the transfer path one of three layouts, normalised per layer by
``_get_layer_kv`` (src/lmpool/engine/kv_transfer.py:149-177):

* a list of per-layer ``(k_cache, v_cache)`` pairs (ModelRunner,
  model_runner.py:822-833; in practice views ``T[0, l]`` / ``T[1, l]`` of one
  ``[2, L, N, bs, H, D]`` tensor, model_runner.py:397-406);
* a 6-D tensor ``[2, L, N, bs, H, D]`` (the transfer benchmark);
* a 5-D tensor ``[2, N, bs, H, D]`` holding a single layer (every layer index
  maps to it).

All three reduce to one affine descriptor when the per-layer views sit at a
constant layer stride, which is what a single launch needs. Anything else is
described one layer at a time (``num_layers = 1`` descriptors). Only host
arithmetic on pointers and strides lives here; no data is touched.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _capi


def get_layer_kv(kv_cache, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Same contract as the reference's ``_get_layer_kv`` (kv_transfer.py:149-177)."""
    if isinstance(kv_cache, (list, tuple)):
        if not kv_cache:
            raise RuntimeError("empty kv_cache")
        first = kv_cache[0]
        if isinstance(first, (list, tuple)):
            return kv_cache[layer_idx][0], kv_cache[layer_idx][1]
        if len(kv_cache) == 2 and isinstance(kv_cache[0], torch.Tensor):
            return kv_cache[0], kv_cache[1]

    if isinstance(kv_cache, torch.Tensor):
        if kv_cache.dim() == 6:
            return kv_cache[0, layer_idx], kv_cache[1, layer_idx]
        if kv_cache.dim() == 5:
            return kv_cache[0], kv_cache[1]

    raise RuntimeError(
        "Unsupported kv_cache layout for transfer; expected per-layer "
        "(k_cache, v_cache) pairs or a tensor with leading K/V dimension"
    )


@dataclass(frozen=True)
class CacheLayout:
    """Byte-level description of ``num_layers`` layers of a paged KV cache."""

    base: int
    kv_stride: int
    layer_stride: int
    block_stride: int
    num_blocks: int
    chunk_bytes: int
    num_layers: int
    dtype: torch.dtype
    device: torch.device
    block_shape: tuple  # (block_size, num_kv_heads, head_dim)

    def desc(self) -> _capi.CacheDesc:
        return _capi.CacheDesc(
            base=self.base,
            kv_stride=self.kv_stride,
            layer_stride=self.layer_stride,
            block_stride=self.block_stride,
            num_blocks=self.num_blocks,
            chunk_bytes=self.chunk_bytes,
            num_layers=self.num_layers,
            reserved=0,
        )

    def block_offset(self, kv: int, layer: int, block: int) -> int:
        return kv * self.kv_stride + layer * self.layer_stride + block * self.block_stride

    def geometry(self) -> dict:
        """Plain-data record exchanged with peers at prewarm time."""
        return {
            "kv_stride": self.kv_stride,
            "layer_stride": self.layer_stride,
            "block_stride": self.block_stride,
            "num_blocks": self.num_blocks,
            "chunk_bytes": self.chunk_bytes,
            "num_layers": self.num_layers,
            "dtype": str(self.dtype),
            "block_shape": tuple(self.block_shape),
        }

    def with_base(self, base: int) -> "CacheLayout":
        return CacheLayout(
            base=base,
            kv_stride=self.kv_stride,
            layer_stride=self.layer_stride,
            block_stride=self.block_stride,
            num_blocks=self.num_blocks,
            chunk_bytes=self.chunk_bytes,
            num_layers=self.num_layers,
            dtype=self.dtype,
            device=self.device,
            block_shape=self.block_shape,
        )


def _check_layer_tensor(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} is not a tensor")
    if t.dim() < 1:
        raise RuntimeError(f"{name} must have a leading block dimension")
    # Each block must be one contiguous run of bytes (the kernel's chunk).
    expected = 1
    for size, stride in reversed(list(zip(t.shape[1:], t.stride()[1:]))):
        if size != 1 and stride != expected:
            raise RuntimeError(f"{name}: each block [block_size, heads, dim] must be contiguous")
        expected *= size


def _single_layer(k: torch.Tensor, v: torch.Tensor) -> CacheLayout:
    _check_layer_tensor(k, "k_cache")
    _check_layer_tensor(v, "v_cache")
    if k.shape != v.shape or k.dtype != v.dtype or k.device != v.device:
        raise RuntimeError("k_cache and v_cache must share shape, dtype and device")
    if k.stride(0) != v.stride(0):
        raise RuntimeError("k_cache and v_cache must share the block stride")
    e = k.element_size()
    chunk = e
    for s in k.shape[1:]:
        chunk *= int(s)
    return CacheLayout(
        base=k.data_ptr(),
        kv_stride=v.data_ptr() - k.data_ptr(),
        layer_stride=0,
        block_stride=k.stride(0) * e,
        num_blocks=int(k.shape[0]),
        chunk_bytes=chunk,
        num_layers=1,
        dtype=k.dtype,
        device=k.device,
        block_shape=tuple(int(s) for s in k.shape[1:]),
    )


def _tensor_layout(t: torch.Tensor, num_layers: int) -> CacheLayout:
    """Layout of a [2, L, N, ...] (6-D) or [2, N, ...] (5-D, one layer) tensor,
    read from its strides without building per-layer views."""
    six = t.dim() == 6
    if six and num_layers > t.shape[1]:
        raise IndexError(f"index {t.shape[1]} is out of bounds for dimension 1 with size {t.shape[1]}")
    inner = t.shape[3:] if six else t.shape[2:]
    inner_strides = t.stride()[3:] if six else t.stride()[2:]
    expected = 1
    for size, stride in reversed(list(zip(inner, inner_strides))):
        if size != 1 and stride != expected:
            raise RuntimeError("k_cache: each block [block_size, heads, dim] must be contiguous")
        expected *= size
    e = t.element_size()
    chunk = e
    for size in inner:
        chunk *= int(size)
    return CacheLayout(
        base=t.data_ptr(),
        kv_stride=t.stride(0) * e,
        layer_stride=(t.stride(1) * e) if six else 0,
        block_stride=(t.stride(2) if six else t.stride(1)) * e,
        num_blocks=int(t.shape[2] if six else t.shape[1]),
        chunk_bytes=chunk,
        num_layers=num_layers,
        dtype=t.dtype,
        device=t.device,
        block_shape=tuple(int(s) for s in inner),
    )


def _list_layouts(kv_cache, num_layers: int) -> list[CacheLayout]:
    """Per-layer (k, v) pairs, from the existing tensors: the first pair is
    checked in full, the others against its shape/strides/dtype/device; the
    result is one affine layout when the pointers sit at a constant stride."""
    k0, v0 = kv_cache[0][0], kv_cache[0][1]
    first = _single_layer(k0, v0)
    sig = (tuple(k0.shape), k0.stride(), k0.dtype, k0.device)
    kptr = [0] * num_layers
    vptr = [0] * num_layers
    uniform = True
    for layer in range(num_layers):
        k, v = kv_cache[layer][0], kv_cache[layer][1]
        if layer and ((tuple(k.shape), k.stride(), k.dtype, k.device) != sig
                      or (tuple(v.shape), v.stride(), v.dtype, v.device) != sig):
            uniform = False
            break
        kptr[layer] = k.data_ptr()
        vptr[layer] = v.data_ptr()
    if uniform:
        step = kptr[1] - kptr[0] if num_layers > 1 else 0
        kv = vptr[0] - kptr[0]
        if all(kptr[i] == kptr[0] + i * step and vptr[i] == kptr[i] + kv for i in range(num_layers)):
            return [CacheLayout(base=first.base, kv_stride=kv, layer_stride=step, block_stride=first.block_stride,
                                num_blocks=first.num_blocks, chunk_bytes=first.chunk_bytes, num_layers=num_layers,
                                dtype=first.dtype, device=first.device, block_shape=first.block_shape)]
    return [_single_layer(kv_cache[layer][0], kv_cache[layer][1]) for layer in range(num_layers)]


def cache_layouts(kv_cache, num_layers: int) -> list[CacheLayout]:
    """One affine layout covering all layers if possible, else one per layer."""
    if num_layers <= 0:
        raise RuntimeError(f"num_layers must be positive, got {num_layers}")
    if isinstance(kv_cache, torch.Tensor) and kv_cache.dim() in (5, 6):
        return [_tensor_layout(kv_cache, num_layers)]
    if isinstance(kv_cache, (list, tuple)) and kv_cache and isinstance(kv_cache[0], (list, tuple)):
        return _list_layouts(kv_cache, num_layers)
    per_layer = [_single_layer(*get_layer_kv(kv_cache, layer)) for layer in range(num_layers)]
    first = per_layer[0]
    for lay in per_layer[1:]:
        if (lay.chunk_bytes, lay.block_stride, lay.num_blocks, lay.dtype, lay.device, lay.kv_stride) != (
            first.chunk_bytes,
            first.block_stride,
            first.num_blocks,
            first.dtype,
            first.device,
            first.kv_stride,
        ):
            return per_layer
    layer_stride = per_layer[1].base - first.base if num_layers > 1 else 0
    for idx, lay in enumerate(per_layer):
        if lay.base != first.base + idx * layer_stride:
            return per_layer
    return [
        CacheLayout(
            base=first.base,
            kv_stride=first.kv_stride,
            layer_stride=layer_stride,
            block_stride=first.block_stride,
            num_blocks=first.num_blocks,
            chunk_bytes=first.chunk_bytes,
            num_layers=num_layers,
            dtype=first.dtype,
            device=first.device,
            block_shape=first.block_shape,
        )
    ]


def affine_layout(kv_cache, num_layers: int) -> CacheLayout:
    """The single affine layout of a cache, or RuntimeError if it has none."""
    lays = cache_layouts(kv_cache, num_layers)
    if len(lays) != 1:
        raise RuntimeError(
            "KV cache layers are not at a constant stride; the cross-GPU path needs one "
            "allocation such as model_runner.py's [2, L, N, block_size, heads, dim] tensor"
        )
    return lays[0]


def payload_layout(num_layers: int, num_blocks: int, block_shape, dtype, device, base: int) -> CacheLayout:
    """Layout of a packed payload ``[L, 2, B, *block_shape]`` (kv_transfer.py:236-240)."""
    e = torch.empty((), dtype=dtype).element_size()
    chunk = e
    for s in block_shape:
        chunk *= int(s)
    return CacheLayout(
        base=base,
        kv_stride=num_blocks * chunk,
        layer_stride=2 * num_blocks * chunk,
        block_stride=chunk,
        num_blocks=num_blocks,
        chunk_bytes=chunk,
        num_layers=num_layers,
        dtype=dtype,
        device=torch.device(device),
        block_shape=tuple(int(s) for s in block_shape),
    )
