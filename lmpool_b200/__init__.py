"""LMPool's KV-cache data path, rebuilt for B200 (sm_100a).

Modules:
  kv_transfer   drop-in for lmpool.engine.kv_transfer (pack/unpack, swap_in,
                swap_out, prewarm_p2p_pairs) plus move_blocks / swap_batch
  attention     drop-in store_kvcache (+ all-layer variant)
  model_runner  ModelRunner transfer boundary (execute_swap_out/in,
                kv_transfer_bytes)
  endpoint      per-GPU mailbox, peer mappings, pair protocol
  layout        KV-cache layouts -> byte descriptors
  topology      NVLink pair detection (drop-in for the nvidia-smi parser)
  benchmark_kv_transfer  LMPool's pair microbenchmark through this package
  latency_profiles/      B200 transfer-latency profiles for LMPool's admission
  _capi         ctypes binding of include/kvx.h (library _kvx.so)
  _build        nvcc recipe for _kvx.so
"""

__all__ = ["kv_transfer", "attention", "model_runner", "endpoint", "layout", "topology"]
__version__ = "0.1.0"
