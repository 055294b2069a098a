"""The reference's KV move on CPU tensors: torch ops plus gloo, as LMPool runs it.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the timed CPU baseline
of ``bench.py`` and a third restatement checked against the reference's own
golden outputs (``tests/test_oracle_torch.py``). Nothing here is imported by
``lmpool_b200``.

Restated from LMPool (src/lmpool/engine/kv_transfer.py):

* ``pack_all_layer_blocks``   -- :229-248, one ``index_select`` per (layer,
  plane) into a ``[L, 2, B, bs, H, D]`` payload;
* ``unpack_all_layer_blocks`` -- :264-276 with the per-layer body of
  :199-215, one ``index_copy_`` per (layer, plane) after the shape check;
* ``swap_planned``            -- the planned path of ``swap_in`` (:431-437,
  :463-470): the source packs and ``dist.send``s the payload, the destination
  ``dist.recv``s it and unpacks. Over gloo on CPU tensors here.

``time_gloo_pair`` and ``time_local`` run those on the host cores for the
bench's CPU baseline: two spawned gloo ranks (127.0.0.1) on seeded bf16
N(0,1) caches, or pack+unpack in one process.
"""
from __future__ import annotations

import os
import socket
import time

import torch
import torch.distributed as dist


def pack_all_layer_blocks(cache: torch.Tensor, num_layers: int, block_ids) -> torch.Tensor:
    """kv_transfer.py:229-248 for a ``[2, L, N, bs, H, D]`` cache."""
    idx = torch.as_tensor(list(block_ids), dtype=torch.long)
    payload = torch.empty((num_layers, 2, len(idx), *cache.shape[3:]), dtype=cache.dtype)
    if len(idx) == 0:
        return payload
    for layer in range(num_layers):
        torch.index_select(cache[0, layer], 0, idx, out=payload[layer, 0])
        torch.index_select(cache[1, layer], 0, idx, out=payload[layer, 1])
    return payload


def unpack_all_layer_blocks(payload: torch.Tensor, cache: torch.Tensor, block_ids) -> None:
    """kv_transfer.py:264-276: shape check, then ``index_copy_`` per (layer, plane)."""
    ids = list(block_ids)
    if payload.dim() != 6 or payload.shape[0] != cache.shape[1] or payload.shape[2] != len(ids):
        raise RuntimeError("packed multi-layer KV payload does not match destination blocks")
    if not ids:
        return
    idx = torch.as_tensor(ids, dtype=torch.long)
    for layer in range(payload.shape[0]):
        cache[0, layer].index_copy_(0, idx, payload[layer, 0])
        cache[1, layer].index_copy_(0, idx, payload[layer, 1])


def swap_planned(rank: int, src_rank: int, dst_rank: int, cache: torch.Tensor, src_ids, dst_ids) -> list:
    """kv_transfer.py:431-437 + :463-470 on the calling rank of a gloo group.

    The source packs and sends, the destination receives into an empty
    payload and unpacks; each returns the block list the reference returns.
    """
    if len(src_ids) != len(dst_ids):
        raise RuntimeError(f"transfer_in negotiated mismatched block counts: remote={len(src_ids)} "
                           f"local={len(dst_ids)}")
    L = cache.shape[1]
    if rank == dst_rank and rank != src_rank:
        payload = torch.empty((L, 2, len(dst_ids), *cache.shape[3:]), dtype=cache.dtype)
        dist.recv(payload, src=src_rank)
        unpack_all_layer_blocks(payload, cache, dst_ids)
        return list(dst_ids)
    if rank == src_rank and rank != dst_rank:
        dist.send(pack_all_layer_blocks(cache, L, src_ids), dst=dst_rank)
    return list(src_ids)


# ---------------------------------------------------------------------------
# Timed CPU baseline
# ---------------------------------------------------------------------------

def _seeded_cache(shape, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(int(seed))
    return torch.empty(shape, dtype=torch.bfloat16).normal_(generator=g)


def _ids(n: int, count: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(int(seed))
    return torch.randperm(int(n), generator=g)[:count].tolist()


def block_digests(cache: torch.Tensor, blocks) -> list[int]:
    """One 64-bit digest per listed block of a [2, L, N, ...] CPU cache over
    its raw bytes: a wrapping dot product of its 32-bit words (every layer,
    both planes) with fixed odd weights. Two ranks compare digests instead
    of shipping or regenerating whole caches."""
    idx = torch.as_tensor(list(blocks), dtype=torch.long)
    words = cache.index_select(2, idx).transpose(0, 2).reshape(len(idx), -1).view(torch.int32)
    gen = torch.Generator().manual_seed(4321)
    weights = torch.randint(0, 2**31 - 1, (words.shape[1],), generator=gen, dtype=torch.int64) * 2 + 1
    out = []
    for row in words:   # one block at a time: bounded temporaries
        out.append(int((row.to(torch.int64) * weights).sum()))
    return out


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank: int, port: int, geom: dict, blocks: int, both_ways: bool, min_seconds: float,
               min_steps: int, threads: int, queue) -> None:
    # A parent launched by torchrun passes its elastic-agent settings down;
    # this pair has its own store on 127.0.0.1.
    for key in ("TORCHELASTIC_USE_AGENT_STORE", "MASTER_ADDR", "MASTER_PORT", "RANK", "WORLD_SIZE", "LOCAL_RANK"):
        os.environ.pop(key, None)
    torch.set_num_threads(max(1, threads))
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2)
    try:
        # each cache holds the blocks a rank gives and the blocks it receives
        # (the cost of a transfer depends on the blocks moved, not on N)
        n = 2 * blocks + 8
        shape = (2, geom["L"], n, geom["bs"], geom["H"], geom["D"])
        cache = _seeded_cache(shape, rank)
        src = {r: _ids(n, blocks, 100 + r) for r in (0, 1)}           # what rank r gives
        dst = {r: [b for b in _ids(n, n, 200 + r) if b not in set(src[r])][:blocks] for r in (0, 1)}

        def one():
            swap_planned(rank, 0, 1, cache, src[0], dst[1])
            if both_ways:
                swap_planned(rank, 1, 0, cache, src[1], dst[0])

        sent = {r: block_digests(cache, src[r]) if r == rank else None for r in (0, 1)}
        one()   # warm-up; then each destination's blocks must carry the source's digests
        mine = {"sent": sent[rank], "got": block_digests(cache, dst[rank])}
        both = [None, None]
        dist.all_gather_object(both, mine)
        ok = both[1]["got"] == both[0]["sent"] and (not both_ways or both[0]["got"] == both[1]["sent"])
        times = []
        start = time.perf_counter()
        while len(times) < min_steps or time.perf_counter() - start < min_seconds:
            dist.barrier()
            t0 = time.perf_counter()
            one()
            t = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times.append(float(t.item()))
            stop = torch.tensor([1.0 if time.perf_counter() - start > 4 * max(min_seconds, 1.0) else 0.0])
            dist.all_reduce(stop, op=dist.ReduceOp.MAX)
            if stop.item() and len(times) >= 1:
                break
        if rank == 0:
            queue.put({"times": times, "verified": bool(ok), "cache_blocks": n})
    finally:
        dist.destroy_process_group()


def cpu_description() -> dict:
    """Host facts the baseline is quoted with: CPU model, cores, torch threads."""
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    return {"cpu_model": model, "os_cpu_count": os.cpu_count(), "usable_cores": cores,
            "torch_threads_default": torch.get_num_threads()}


def time_gloo_pair(geom: dict, blocks: int, *, both_ways: bool = False, min_seconds: float = 10.0,
                   min_steps: int = 3, timeout_s: float = 300.0) -> dict:
    """Time the reference's planned ``swap_in`` (pack -> gloo send/recv ->
    unpack) between two spawned CPU ranks on this host: one direction, or
    0->1 then 1->0 (two sequential ``swap_in`` calls, as the reference
    serves a pair that sends both ways). Each rank gets half the host's
    cores. Returns seconds per step (max over the two ranks) and the sample."""
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    host = cpu_description()
    threads = max(1, host["usable_cores"] // 2)
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, port, geom, blocks, both_ways, min_seconds, min_steps,
                                                  threads, queue)) for r in (0, 1)]
    for p in procs:
        p.start()
    try:
        res = queue.get(timeout=timeout_s)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    payload = blocks * geom["L"] * 2 * geom["bs"] * geom["H"] * geom["D"] * 2
    moved = payload * (2 if both_ways else 1)
    mean = sum(res["times"]) / len(res["times"])
    return {"seconds_per_step": mean, "steps": len(res["times"]), "total_s": sum(res["times"]),
            "bytes_per_step": moved, "GB/s": moved / mean / 1e9, "verified": res["verified"],
            "threads_per_rank": threads, "ranks": 2, "cores": 2 * threads, "cache_blocks": res["cache_blocks"],
            "host": host}


def time_local(geom: dict, blocks: int, *, min_seconds: float = 10.0, min_steps: int = 3) -> dict:
    """Time pack + unpack in one process (the reference's two helpers with no
    transport between them), with every host thread."""
    host = cpu_description()
    torch.set_num_threads(host["usable_cores"])
    n = 2 * blocks + 8
    shape = (2, geom["L"], n, geom["bs"], geom["H"], geom["D"])
    cache = _seeded_cache(shape, 0)
    perm = _ids(n, n, 0)
    src, dst = perm[:blocks], perm[blocks:2 * blocks]
    unpack_all_layer_blocks(pack_all_layer_blocks(cache, geom["L"], src), cache, dst)   # warm-up
    ok = torch.equal(cache[:, :, dst].view(torch.int16), cache[:, :, src].view(torch.int16))
    times = []
    start = time.perf_counter()
    while len(times) < min_steps or time.perf_counter() - start < min_seconds:
        t0 = time.perf_counter()
        unpack_all_layer_blocks(pack_all_layer_blocks(cache, geom["L"], src), cache, dst)
        times.append(time.perf_counter() - t0)
    payload = blocks * geom["L"] * 2 * geom["bs"] * geom["H"] * geom["D"] * 2
    mean = sum(times) / len(times)
    return {"seconds_per_step": mean, "steps": len(times), "total_s": sum(times), "bytes_per_step": payload,
            "GB/s": payload / mean / 1e9, "verified": bool(ok), "cores": host["usable_cores"],
            "cache_blocks": n, "host": host}
