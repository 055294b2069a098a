"""ModelRunner transfer boundary on the B200 path.

LMPool's data plane calls three ModelRunner methods around a transfer
(src/lmpool/engine/model_runner.py:747-833): ``execute_swap_out`` on the
source, ``execute_swap_in`` on the destination and ``kv_transfer_bytes`` for
its statistics. :class:`B200KVTransferMixin` provides the same three methods
(same arguments, same return values, same forwarding to ``swap_in`` with
``negotiate_blocks=False``) routed to :mod:`lmpool_b200.kv_transfer`, plus
``register_kv_cache_for_transfer`` to call at the end of
``allocate_kv_cache`` so prewarm can export the cache to peers.

The mixin needs from its host class what LMPool's ModelRunner already has:
``self.rank``, ``self.config`` (num_layers, num_kv_heads, head_dim or
hidden_size/num_heads), ``self.block_size`` and ``self.model`` whose modules
carry ``k_cache``/``v_cache``.
"""
from __future__ import annotations

import logging
from typing import List, Optional

from . import kv_transfer

logger = logging.getLogger(__name__)


class B200KVTransferMixin:
    def _transfer_head_dim(self) -> int:
        cfg = self.config
        return cfg["head_dim"] if "head_dim" in cfg else cfg["hidden_size"] // cfg["num_heads"]

    def _get_kv_cache(self):
        """model_runner.py:822-833: every layer's (k_cache, v_cache)."""
        layer_caches = []
        for module in self.model.modules():
            if hasattr(module, "k_cache") and hasattr(module, "v_cache"):
                if module.k_cache is not None and module.v_cache is not None:
                    if hasattr(module.k_cache, "numel") and module.k_cache.numel() == 0:
                        continue
                    layer_caches.append((module.k_cache, module.v_cache))
        if not layer_caches:
            raise RuntimeError("Cannot find k_cache/v_cache in model layers")
        return layer_caches

    def register_kv_cache_for_transfer(self):
        """Export-ready layout of this runner's cache (call after allocate_kv_cache)."""
        return kv_transfer.register_kv_cache(self._get_kv_cache(), self.config["num_layers"])

    def execute_swap_out(self, blocks: List[int], target_gpu: int):
        """model_runner.py:747-775: this rank is the source of the move."""
        kv_cache = self._get_kv_cache()
        logger.info("execute_transfer_out: GPU%s -> GPU%s | blocks=%s", self.rank, target_gpu, blocks)
        target_blocks = kv_transfer.swap_in(
            remote_gpu=self.rank,
            remote_blocks=blocks,
            local_gpu=target_gpu,
            kv_cache=kv_cache,
            num_layers=self.config["num_layers"],
            block_size=self.block_size,
            num_kv_heads=self.config["num_kv_heads"],
            head_dim=self._transfer_head_dim(),
            negotiate_blocks=False,
        )
        logger.info("execute_transfer_out done: blocks=%s -> target_blocks=%s", blocks, target_blocks)
        return target_blocks

    def execute_swap_in(self, remote_gpu: int, remote_blocks: List[int],
                        local_target_blocks: Optional[List[int]] = None):
        """model_runner.py:777-806: this rank is the destination of the move."""
        kv_cache = self._get_kv_cache()
        logger.info("execute_transfer_in: GPU%s -> GPU%s | blocks=%s", remote_gpu, self.rank, remote_blocks)
        local_blocks = kv_transfer.swap_in(
            remote_gpu=remote_gpu,
            remote_blocks=remote_blocks,
            local_gpu=self.rank,
            kv_cache=kv_cache,
            num_layers=self.config["num_layers"],
            block_size=self.block_size,
            num_kv_heads=self.config["num_kv_heads"],
            head_dim=self._transfer_head_dim(),
            local_target_blocks=local_target_blocks,
            negotiate_blocks=False,
        )
        logger.info("execute_transfer_in done: remote_blocks=%s -> local_blocks=%s", remote_blocks, local_blocks)
        return local_blocks

    def kv_transfer_bytes(self, num_blocks: int) -> int:
        """model_runner.py:808-820: exact K+V bytes of ``num_blocks`` blocks (all layers)."""
        if num_blocks <= 0:
            return 0
        kv_cache = self._get_kv_cache()
        if not kv_cache:
            return 0
        first_k, first_v = kv_cache[0]
        per_block = first_k[0].numel() * first_k.element_size() + first_v[0].numel() * first_v.element_size()
        return int(num_blocks) * len(kv_cache) * per_block
