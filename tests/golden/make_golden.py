"""Generate the golden fixtures in this folder from the reference itself.

Run where the reference is checked out (read-only), naming its root:

    LMPOOL_REF=<path to the LMPool checkout> python tests/golden/make_golden.py

What it records, all produced by LMPool's own code:

* ``pack_unpack.npz`` -- ``_pack_layer_blocks`` / ``_unpack_layer_blocks`` /
  ``_pack_all_layer_blocks`` / ``_unpack_all_layer_blocks``
  (src/lmpool/engine/kv_transfer.py:180-276) on the reference tests' arange
  cases (tests/test_kv_transfer.py:66-102) and on seeded bf16/fp16 caches,
  including repeated source ids and the list-of-layers layout.
* ``swap_small.npz`` -- ``swap_in(..., negotiate_blocks=False)``
  (kv_transfer.py:395-475) run on two gloo CPU ranks with full arrays kept.
* ``swap_config1.json`` -- the same call at benchmark config 1 geometry
  ([2, 28, 64, 256, 8, 128] bf16, seeds 0/1, B=8); caches are too large to
  store, so SHA-256 digests of the inputs and outputs are kept and the inputs
  are regenerated from ``tests/kvgen.py``.
* ``store_kvcache.npz`` -- the reference Triton ``store_kvcache``
  (src/lmpool/layers/attention.py:7-108) executed by Triton's CPU interpreter
  (TRITON_INTERPRET=1) on seeded inputs with padding slots (-1).

The fixtures are inputs + outputs; nothing here runs on the GPU box.
"""
from __future__ import annotations

import importlib.util
import json
import os
import socket
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("LMPOOL_REF", "reference"))
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REF / "src"))

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from tests import kvgen  # noqa: E402


def _bits(t: torch.Tensor) -> np.ndarray:
    """Raw element bits (uint16 for 2-byte dtypes, uint32 for 4-byte)."""
    t = t.detach().contiguous()
    view = {2: torch.int16, 4: torch.int32, 1: torch.uint8}[t.element_size()]
    return t.view(view).numpy().copy()


def _load_ref_module(name: str, path: Path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_pack_unpack(kt) -> None:
    out = {}
    # Case A: tests/test_kv_transfer.py:66-79 (per-layer, float32 arange).
    source_k = torch.arange(24, dtype=torch.float32).reshape(4, 3, 2, 1)
    source_v = source_k + 100
    target_k = torch.zeros_like(source_k)
    target_v = torch.zeros_like(source_v)
    payload = kt._pack_layer_blocks(source_k, source_v, [3, 1])
    kt._unpack_layer_blocks(payload, target_k, target_v, [0, 2])
    out.update(a_source_k=source_k.numpy(), a_source_v=source_v.numpy(), a_payload=payload.numpy(),
               a_target_k=target_k.numpy(), a_target_v=target_v.numpy(), a_src_ids=np.array([3, 1]),
               a_dst_ids=np.array([0, 2]))

    # Case B: tests/test_kv_transfer.py:82-102 (list-of-layers, 2 layers).
    source = [(torch.arange(24, dtype=torch.float32).reshape(4, 3, 2, 1) + layer * 100,
               torch.arange(24, dtype=torch.float32).reshape(4, 3, 2, 1) + layer * 1000) for layer in range(2)]
    target = [(torch.zeros_like(k), torch.zeros_like(v)) for k, v in source]
    payload = kt._pack_all_layer_blocks(source, 2, [3, 1])
    kt._unpack_all_layer_blocks(payload, target, [0, 2])
    out.update(b_source=np.stack([np.stack([k.numpy(), v.numpy()]) for k, v in source]),
               b_payload=payload.numpy(),
               b_target=np.stack([np.stack([k.numpy(), v.numpy()]) for k, v in target]),
               b_src_ids=np.array([3, 1]), b_dst_ids=np.array([0, 2]))

    # Case C: seeded bf16 6-D caches, fragmented ids, B=5 of N=12.
    shape = (2, 3, 12, 4, 2, 8)
    src = kvgen.seeded_cache(shape, 10)
    dst = kvgen.seeded_cache(shape, 11)
    src_ids = kvgen.seeded_perm(12, 10)[:5]
    dst_ids = kvgen.seeded_perm(12, 11)[:5]
    dst_before = dst.clone()
    payload = kt._pack_all_layer_blocks(src, 3, src_ids)
    kt._unpack_all_layer_blocks(payload, dst, dst_ids)
    out.update(c_src=_bits(src), c_dst_before=_bits(dst_before), c_payload=_bits(payload), c_dst_after=_bits(dst),
               c_src_ids=np.array(src_ids), c_dst_ids=np.array(dst_ids), c_shape=np.array(shape))

    # Case D: fp16, repeated source ids (index_select allows them), bs=16.
    shape = (2, 2, 9, 16, 1, 8)
    src = kvgen.seeded_cache(shape, 20, dtype=torch.float16)
    dst = kvgen.seeded_cache(shape, 21, dtype=torch.float16)
    src_ids = [4, 4, 0, 8]
    dst_ids = [1, 7, 3, 2]
    dst_before = dst.clone()
    payload = kt._pack_all_layer_blocks(src, 2, src_ids)
    kt._unpack_all_layer_blocks(payload, dst, dst_ids)
    out.update(d_src=_bits(src), d_dst_before=_bits(dst_before), d_payload=_bits(payload), d_dst_after=_bits(dst),
               d_src_ids=np.array(src_ids), d_dst_ids=np.array(dst_ids), d_shape=np.array(shape))

    # Case E: list-of-layers layout taken from one [2, L, N, ...] tensor
    # (how ModelRunner binds k_cache/v_cache, model_runner.py:401-406).
    shape = (2, 4, 10, 8, 2, 16)
    big_src = kvgen.seeded_cache(shape, 30)
    big_dst = kvgen.seeded_cache(shape, 31)
    src_list = [(big_src[0, layer], big_src[1, layer]) for layer in range(4)]
    dst_list = [(big_dst[0, layer], big_dst[1, layer]) for layer in range(4)]
    src_ids = kvgen.seeded_perm(10, 30)[:6]
    dst_ids = kvgen.seeded_perm(10, 31)[:6]
    before = big_dst.clone()
    payload = kt._pack_all_layer_blocks(src_list, 4, src_ids)
    kt._unpack_all_layer_blocks(payload, dst_list, dst_ids)
    out.update(e_src=_bits(big_src), e_dst_before=_bits(before), e_payload=_bits(payload), e_dst_after=_bits(big_dst),
               e_src_ids=np.array(src_ids), e_dst_ids=np.array(dst_ids), e_shape=np.array(shape))
    np.savez_compressed(HERE / "pack_unpack.npz", **out)


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _swap_worker(rank: int, port: int, case: str, result_path: str) -> None:
    sys.path.insert(0, str(REF / "src"))
    sys.path.insert(0, str(REPO))
    from lmpool.engine import kv_transfer as kt  # noqa: PLC0415

    torch.set_num_threads(4)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2, rank=rank)
    if case == "small":
        shape = (2, 2, 6, 2, 1, 4)
        cache = kvgen.seeded_cache(shape, 40 + rank, dtype=torch.float32)
        src_ids, dst_ids = [5, 0, 3], [2, 4, 1]
    else:
        shape = (2, 28, 64, 256, 8, 128)
        cache = kvgen.seeded_cache(shape, rank)
        src_ids = kvgen.seeded_perm(64, 0)[:8]
        dst_ids = kvgen.seeded_perm(64, 1)[:8]
    before = kvgen.sha256_of(cache) if case != "small" else None
    before_arr = cache.clone() if case == "small" else None
    dist.barrier()
    got = kt.swap_in(remote_gpu=0, remote_blocks=src_ids, local_gpu=1, kv_cache=cache, num_layers=shape[1],
                     block_size=shape[3], num_kv_heads=shape[4], head_dim=shape[5],
                     local_target_blocks=dst_ids if rank == 1 else None, negotiate_blocks=False)
    dist.barrier()
    rec = {"rank": rank, "returned": list(map(int, got)), "src_ids": src_ids, "dst_ids": dst_ids}
    if case == "small":
        np.savez(result_path + f".{rank}.npz", before=before_arr.numpy(), after=cache.numpy())
    else:
        rec.update(before_sha256=before, after_sha256=kvgen.sha256_of(cache))
        # Digest of each moved destination block (plane, all layers) for a
        # readable per-block check.
        if rank == 1:
            rec["dst_block_sha256"] = {str(b): kvgen.sha256_of(cache[:, :, b]) for b in dst_ids}
        else:
            rec["src_block_sha256"] = {str(b): kvgen.sha256_of(cache[:, :, b]) for b in src_ids}
    with open(result_path + f".{rank}.json", "w") as f:
        json.dump(rec, f)
    dist.destroy_process_group()


def run_swap(case: str) -> list[dict]:
    port = _free_port()
    tmp = str(HERE / f"_tmp_swap_{case}")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_swap_worker, args=(r, port, case, tmp)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=900)
        if p.exitcode != 0:
            raise RuntimeError(f"reference swap worker failed (exit {p.exitcode})")
    recs = []
    for r in range(2):
        with open(tmp + f".{r}.json") as f:
            recs.append(json.load(f))
        os.remove(tmp + f".{r}.json")
    return recs


def make_swaps() -> None:
    recs = run_swap("small")
    arrs = {}
    for r in range(2):
        z = np.load(str(HERE / f"_tmp_swap_small.{r}.npz"))
        arrs[f"rank{r}_before"] = z["before"]
        arrs[f"rank{r}_after"] = z["after"]
        os.remove(HERE / f"_tmp_swap_small.{r}.npz")
    np.savez_compressed(HERE / "swap_small.npz", src_ids=np.array(recs[0]["src_ids"]),
                        dst_ids=np.array(recs[0]["dst_ids"]), returned0=np.array(recs[0]["returned"]),
                        returned1=np.array(recs[1]["returned"]), **arrs)
    recs = run_swap("config1")
    out = {
        "description": "reference kv_transfer.swap_in(negotiate_blocks=False) on two gloo CPU ranks, "
                       "benchmark config 1 geometry; inputs from tests/kvgen.config1_inputs()",
        "shape": [2, 28, 64, 256, 8, 128],
        "dtype": "bfloat16",
        "src_ids": recs[0]["src_ids"],
        "dst_ids": recs[0]["dst_ids"],
        "returned_rank0": recs[0]["returned"],
        "returned_rank1": recs[1]["returned"],
        "src_before_sha256": recs[0]["before_sha256"],
        "src_after_sha256": recs[0]["after_sha256"],
        "dst_before_sha256": recs[1]["before_sha256"],
        "dst_after_sha256": recs[1]["after_sha256"],
        "src_block_sha256": recs[0]["src_block_sha256"],
        "dst_block_sha256": recs[1]["dst_block_sha256"],
    }
    with open(HERE / "swap_config1.json", "w") as f:
        json.dump(out, f, indent=1)


def make_store_kvcache() -> None:
    attn = _load_ref_module("ref_attention", REF / "src" / "lmpool" / "layers" / "attention.py")
    out = {}
    cases = [
        ("f32", torch.float32, 37, 2, 8, 4, 16, 50),
        ("bf16", torch.bfloat16, 29, 2, 16, 16, 4, 51),
        ("h8", torch.bfloat16, 24, 8, 128, 16, 6, 52),
    ]
    for name, dtype, T, H, D, bs, N, seed in cases:
        key = kvgen.seeded_cache((T, H, D), seed, dtype=dtype)
        value = kvgen.seeded_cache((T, H, D), seed + 1000, dtype=dtype)
        k_cache = kvgen.seeded_cache((N, bs, H, D), seed + 2000, dtype=dtype)
        v_cache = kvgen.seeded_cache((N, bs, H, D), seed + 3000, dtype=dtype)
        slots = kvgen.slot_mapping(T, N * bs, seed, skip_fraction=0.15)
        kc0, vc0 = k_cache.clone(), v_cache.clone()
        attn.store_kvcache(key, value, k_cache, v_cache, slots, bs)
        out.update({f"{name}_key": _bits(key), f"{name}_value": _bits(value), f"{name}_kc_before": _bits(kc0),
                    f"{name}_vc_before": _bits(vc0), f"{name}_kc_after": _bits(k_cache),
                    f"{name}_vc_after": _bits(v_cache), f"{name}_slots": slots.numpy(),
                    f"{name}_dims": np.array([T, H, D, bs, N])})
    np.savez_compressed(HERE / "store_kvcache.npz", **out)


def main() -> None:
    from lmpool.engine import kv_transfer as kt  # noqa: PLC0415

    make_pack_unpack(kt)
    make_store_kvcache()
    make_swaps()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
