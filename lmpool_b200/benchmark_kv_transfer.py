"""KV transfer microbenchmark on B200, through this package's ``swap_in``.

Counterpart of LMPool's ``benchmarks/benchmark_kv_transfer.py``: the same
command-line flags, the same two-process pair case (rank 0's blocks
``0..B-1`` move to rank 1's blocks ``B..2B-1``, benchmark_kv_transfer.py:92-193;
here seeded random caches checked afterwards by per-block digests of the
raw bytes on both ranks), and the same result schema (``{"metadata": ..., "results": [...]}`` with
``num_transfer_blocks``, ``bytes_per_iteration``, mean/p50/p95 latency and
GiB/s per row, :176-193, :334-350). LMPool's own profile builder
(benchmarks/build_transfer_profile.py -> transfer_profile.py:113-196) reads
the output unchanged, so its admission cost model can be fed B200 numbers.

Each row also carries device-timed figures (CUDA events around the transfer
on the destination) next to the reference's host wall time.

    python -m lmpool_b200.benchmark_kv_transfer --num-layers 36 --block-counts 1,2,4,8,16,32,64 \
        --iterations 100 --warmup 20 --dtype bfloat16 --output-json kv_transfer_b200.json
"""
from __future__ import annotations

import argparse
import json
import math
import os
import platform
import queue
import socket
import statistics
import sys
import time
from pathlib import Path

import torch
import torch.multiprocessing as mp

_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def parse_block_counts(raw: str, fallback: int) -> list[int]:
    """Block counts of the sweep in first-seen order, each once; ``fallback``
    when the list is empty. Same contract as the reference's flag
    (benchmark_kv_transfer.py:196-201): every count must be positive."""
    sweep: list[int] = []
    for piece in (raw or "").split(","):
        if not piece.strip():
            continue
        count = int(piece)
        if count < 1:
            raise ValueError(f"transfer block counts must all be >= 1, got {count}")
        if count not in sweep:
            sweep.append(count)
    return sweep or [int(fallback)]


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="KV transfer microbenchmark (B200 NVLink push)")
    p.add_argument("--dtype", choices=["auto", "float16", "bfloat16", "float32"], default="auto",
                   help="payload dtype; auto = float16, as the reference without a model")
    p.add_argument("--num-layers", type=int, default=28)
    p.add_argument("--block-size", type=int, default=256)
    p.add_argument("--num-kv-heads", type=int, default=8)
    p.add_argument("--head-dim", type=int, default=128)
    p.add_argument("--num-transfer-blocks", type=int, default=2)
    p.add_argument("--block-counts", default="", help="comma-separated sweep; overrides --num-transfer-blocks")
    p.add_argument("--iterations", type=int, default=5)
    p.add_argument("--warmup", type=int, default=1)
    p.add_argument("--model-label", default="", help="label recorded in metadata.model.label")
    p.add_argument("--output-json", default="")
    args = p.parse_args(argv)
    args.resolved_dtype = "float16" if args.dtype == "auto" else args.dtype
    return args


def _block_digests(kv_cache: torch.Tensor, blocks: list[int]) -> list[int]:
    """One 64-bit digest per listed block over its raw bytes (every layer,
    both planes): a wrapping dot product of the block's 32-bit words with
    fixed odd weights. Source and destination compare digests, so the check
    sees the actual bytes, including two blocks swapped or a layer moved."""
    idx = torch.tensor(blocks, dtype=torch.long, device=kv_cache.device)
    words = kv_cache.index_select(2, idx).transpose(0, 2).reshape(len(blocks), -1).view(torch.int32).to(torch.int64)
    gen = torch.Generator().manual_seed(1234)
    weights = (torch.randint(0, 2**31 - 1, (words.shape[1],), generator=gen, dtype=torch.int64) * 2 + 1)
    return (words * weights.to(words.device)).sum(dim=1).tolist()


def _p95(values: list[float]) -> float:
    """Nearest-rank 95th percentile."""
    ordered = sorted(values)
    return ordered[max(0, math.ceil(0.95 * len(ordered)) - 1)]


def _worker(rank: int, args, blocks: int, port: int, out) -> None:
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt

    try:
        torch.cuda.set_device(rank)
        os.environ["LOCAL_RANK"] = str(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", world_size=2, rank=rank,
                                device_id=torch.device("cuda", rank))
        dtype = _DTYPES[args.resolved_dtype]
        src_blocks = list(range(blocks))
        dst_blocks = list(range(blocks, 2 * blocks))
        cache = torch.empty(2, args.num_layers, 2 * blocks, args.block_size, args.num_kv_heads, args.head_dim,
                            dtype=dtype, device=f"cuda:{rank}")
        cache.normal_(generator=torch.Generator(device=f"cuda:{rank}").manual_seed(100 + rank))
        kt.register_kv_cache(cache, args.num_layers)
        kt.prewarm_p2p_pairs([(0, 1)], num_layers=args.num_layers, block_size=args.block_size,
                             num_kv_heads=args.num_kv_heads, head_dim=args.head_dim, num_blocks=blocks, dtype=dtype)
        dist.barrier()
        host_ms, dev_ms = [], []
        stream = torch.cuda.current_stream()
        for iteration in range(args.warmup + args.iterations):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start = time.perf_counter()
            e0.record(stream)
            kt.swap_in(remote_gpu=0, remote_blocks=src_blocks, local_gpu=1, kv_cache=cache,
                       num_layers=args.num_layers, block_size=args.block_size, num_kv_heads=args.num_kv_heads,
                       head_dim=args.head_dim, local_target_blocks=dst_blocks if rank == 1 else None,
                       negotiate_blocks=False)
            e1.record(stream)
            torch.cuda.synchronize()
            elapsed = (time.perf_counter() - start) * 1000.0
            if iteration >= args.warmup:
                host_ms.append(elapsed)
                dev_ms.append(e0.elapsed_time(e1))
        digests = [None, None]
        dist.all_gather_object(digests, _block_digests(cache, src_blocks if rank == 0 else dst_blocks))
        ok = digests[0] == digests[1]
        bytes_per_iter = blocks * args.num_layers * args.block_size * args.num_kv_heads * args.head_dim * 2 \
            * cache.element_size()
        kt.shutdown()
        out.put({"rank": rank, "ok": bool(ok), "mean_ms": statistics.mean(host_ms),
                 "p50_ms": statistics.median(host_ms), "p95_ms": _p95(host_ms),
                 "device_mean_ms": statistics.mean(dev_ms), "device_p95_ms": _p95(dev_ms),
                 "bytes_per_iter": bytes_per_iter})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        out.put({"rank": rank, "ok": False, "error": repr(exc)})
        raise


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_transfer_case(args, blocks: int, timeout_s: float = 600.0) -> dict:
    """benchmark_kv_transfer.py:287-350: one block count, two spawned ranks."""
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, args, blocks, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results, deadline = [], time.time() + timeout_s
    try:
        while len(results) < 2 and time.time() < deadline:
            try:
                results.append(out.get(timeout=1))
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=10)
    if len(results) != 2 or not all(r["ok"] for r in results):
        raise RuntimeError(f"transfer validation failed for {blocks} blocks: results={results}")
    dst = next(r for r in results if r["rank"] == 1)
    gib = dst["bytes_per_iter"] / 2**30
    return {
        "num_transfer_blocks": int(blocks),
        "bytes_per_iteration": int(dst["bytes_per_iter"]),
        "gib_per_iteration": float(gib),
        "mean_latency_ms": float(dst["mean_ms"]),
        "p50_latency_ms": float(dst["p50_ms"]),
        "p95_latency_ms": float(dst["p95_ms"]),
        "effective_bandwidth_gib_s": float(gib / max(dst["mean_ms"] / 1000.0, 1e-9)),
        "device_mean_latency_ms": float(dst["device_mean_ms"]),
        "device_p95_latency_ms": float(dst["device_p95_ms"]),
        "device_bandwidth_gb_s": float(dst["bytes_per_iter"] / (dst["device_mean_ms"] * 1e-3) / 1e9),
        "data_validation": "passed",
    }


def build_metadata(args) -> dict:
    """The fields LMPool's profile builder reads (transfer_profile.py:38-80)."""
    dtype = _DTYPES[args.resolved_dtype]
    names = [torch.cuda.get_device_name(i) for i in range(min(2, torch.cuda.device_count()))] \
        if torch.cuda.is_available() else []
    from .kv_transfer import transfer_mode

    return {
        "benchmark": "benchmark_kv_transfer",
        "implementation": f"lmpool_b200 NVLink {transfer_mode()} (CUDA IPC), sm_100a",
        "transfer_mode": transfer_mode(),
        "model": {"label": args.model_label or f"custom-{args.resolved_dtype}"},
        "resolved_config": {
            "num_layers": args.num_layers,
            "block_size": args.block_size,
            "num_kv_heads": args.num_kv_heads,
            "head_dim": args.head_dim,
            "torch_dtype": args.resolved_dtype,
            "kv_dtype_bytes": torch.empty((), dtype=dtype).element_size(),
        },
        "environment": {"CUDA_VISIBLE_DEVICES": os.environ.get("CUDA_VISIBLE_DEVICES", "0,1"),
                        "gpus": names, "hostname": socket.gethostname(), "python": platform.python_version(),
                        "torch": torch.__version__},
        "args": {k: v for k, v in vars(args).items() if isinstance(v, (int, float, str, bool))},
    }


def main(argv=None) -> list[dict]:
    args = parse_args(argv)
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        raise SystemExit("requires at least 2 visible CUDA devices")
    if args.iterations < 1:
        raise SystemExit("--iterations must be >= 1")
    if args.warmup < 0:
        raise SystemExit("--warmup must be >= 0")
    counts = parse_block_counts(args.block_counts, args.num_transfer_blocks)
    results = [run_transfer_case(args, b) for b in counts]
    print(f"{'blocks':>8} {'payload(GiB)':>14} {'mean(ms)':>10} {'p95(ms)':>10} {'GiB/s':>9} {'device GB/s':>12}")
    for r in results:
        print(f"{r['num_transfer_blocks']:>8d} {r['gib_per_iteration']:>14.3f} {r['mean_latency_ms']:>10.3f} "
              f"{r['p95_latency_ms']:>10.3f} {r['effective_bandwidth_gib_s']:>9.2f} "
              f"{r['device_bandwidth_gb_s']:>12.1f}")
    if args.output_json:
        out = Path(args.output_json)
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(json.dumps({"metadata": build_metadata(args), "results": results}, indent=2))
        print(f"saved json: {out}", file=sys.stderr)
    return results


if __name__ == "__main__":
    main()
