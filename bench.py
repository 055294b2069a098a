#!/usr/bin/env python
"""Benchmark of LMPool's KV move path on B200 (one JSON line on rank 0).

Metric: "KV move GB/s per pair (gather->NVLink->scatter,
device-timed) vs blocks moved"; GB = 1e9 bytes of KV payload
P = B * L * 2 * block_size * kv_heads * head_dim * 2 bytes moved per step
(ModelRunner.kv_transfer_bytes, model_runner.py:808-820).

Workloads (synthetic bf16 N(0,1) caches, seeded randperm block ids):
  --gpus 1   benchmark config 2: one GPU, Qwen3-0.6B KV geometry (L=28, H=8,
             D=128, block_size=256), 2048-block cache (60 GB); a step moves
             B=512 fragmented blocks inside the cache (gather+scatter in one
             launch). The B sweep {1,4,16,64,256,512} is reported in "sweep".
  --gpus N>1 benchmark config 4 phase A: ranks (0,1), (2,3), ... move
             B=128 blocks each way at once at Qwen3-8B geometry (L=36,
             1536-block cache per rank, 58 GB); a step is one exchange in
             push mode (arm, push, completion wait). The line adds config 3
             (N=2), config 4 phase B (N>=4) and config 5, each verified.
  --impl reference  the reference's CPU path on the host cores (rank 0 only):
             pack + unpack with torch ops in one process (N=1), or two gloo
             ranks exchanging one pair's blocks both ways (N>1).

Timing: W untimed warm-up steps, then K steps between a barrier and a
device synchronisation, CUDA events on the launching stream, max over ranks.
Every step's inputs exceed the 126 MB L2 (config 2: 15 GB read + 15 GB
written per step; config 4: 4.8 GB per direction), so no flush is needed for
the headline; the sweeps flush L2 before each timed launch.

Verification: every moved block is compared byte for byte -- with its
source (1 GPU), or with the bytes the reference's own algorithm delivers on
the same GPUs (index_select -> NCCL send/recv, per plane and layer) -- and
every other block is checked unchanged through a 64-bit per-block
fingerprint taken before and after.
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "KV move GB/s per pair (gather→NVLink→scatter, device-timed) vs blocks moved"
LOCAL = dict(workload="config2: 1-GPU local gather+scatter, Qwen3-0.6B KV geometry", L=28, N=2048, bs=256, H=8,
             D=128, B=512)
PAIRS = dict(workload="config4 phase A: disjoint NVLink pairs, both directions at once, Qwen3-8B KV geometry", L=36,
             N=1536, bs=256, H=8, D=128, B=128)
CONFIG5 = dict(workload="config5: 70B-like transfer (B=1024 to the NVLink partner, both directions) under "
                        "concurrent store_kvcache (T=256 tokens x 80 layers per step)",
               L=80, N=16384, bs=16, H=8, D=128, B=1024, T=256)
STORE = dict(L=80, H=8, D=128, bs=16, N=4096, T=256)
SWEEP_B = [1, 4, 16, 64, 256, 512]
PAIR_SWEEP_B = [1, 8, 64, 256]
PHASE_B_BLOCKS = 32
# Per-direction NVLink 5 bandwidth of one B200 (900 GB/s nominal): the pair
# roofline. A plain peer copy is measured in the same run for comparison.
NVLINK_NOMINAL_GBS = 900.0
FALLBACK_HBM_GBS = 6650.0
CPU_SAMPLE_BLOCKS = 16
L2_FLUSH_BYTES = 512 << 20
FP_MULT = -7046029254386353131   # odd 64-bit constant (as a signed int64) folding planes and layers


class L2Flush:
    """Evicts L2 between timed launches: writes a buffer larger than L2, then
    reads another one, so the timed launch finds neither its own data nor
    dirty lines of the flush (whose write-back would otherwise be charged to
    it: +2 to +8 us per launch at 1-4 blocks, measured). ``dirty=True``
    skips the read, for the write-only figure."""

    def __init__(self, dev):
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.r = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)

    def __call__(self, dirty: bool = False) -> None:
        self.w.zero_()
        if not dirty:
            torch.sum(self.r, dim=0, out=self.sink)


def payload_bytes(g: dict, blocks: int) -> int:
    return blocks * g["L"] * 2 * g["bs"] * g["H"] * g["D"] * 2


def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback (profiling recipe, 6.65 TB/s)"


def profile_value(name: str, key: str) -> float | None:
    """A ``key: value`` figure recorded in a committed ncu summary (profiles/<name>.txt)."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    m = re.search(rf"^{re.escape(key)}:\s*([0-9.eE+]+)", p.read_text(), re.M)
    return float(m.group(1)) if m else None


def seeded_perm(n: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(int(seed))
    return torch.randperm(int(n), generator=g).tolist()


def line_config(g: dict, world: int) -> dict:
    """The ``config`` object of the JSON line; both arms print the same one."""
    cfg = {"workload": g["workload"], "num_layers": g["L"], "num_blocks": g["N"], "block_size": g["bs"],
           "num_kv_heads": g["H"], "head_dim": g["D"], "dtype": "bf16"}
    if world <= 1:
        cfg.update({"blocks_moved": g["B"], "payload_bytes_per_step": payload_bytes(g, g["B"]),
                    "src_ids": "randperm[:512]", "dst_ids": "randperm[512:1024]",
                    "l2": "inputs larger than L2 (15 GB read + 15 GB written per step); the sweep flushes L2 "
                          "before each launch by writing 512 MB then reading 512 MB (ms_dirty_l2: write only)",
                    "parallelism": "replicas only"})
    else:
        cfg.update({"blocks_moved_per_direction": g["B"], "payload_bytes_per_rank_per_step": payload_bytes(g, g["B"]),
                    "pairs": [(r, r + 1) for r in range(0, world, 2)],
                    "l2": "inputs larger than L2 (4.8 GB per direction per step)",
                    "parallelism": f"{world // 2} NVLink pairs over CUDA IPC, no collective on the data path"})
    return cfg


class ClockSampler:
    """nvidia-smi clock/throttle samples of one GPU during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.out = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.out, stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.25)
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi unavailable"}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.flush()
        self.out.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.out.read())) if len(r) >= 9]
        os.unlink(self.out.name)
        sm, smax, power = [], [], []
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
                power.append(float(r[3]))
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": sorted(reasons), "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


def merge_clocks(items: list[dict]) -> dict:
    sms = [c["sm_mhz"] for c in items if c.get("sm_mhz")]
    return {"sm_mhz": statistics.median(sms) if sms else None,
            "sm_max_mhz": max((c["sm_max_mhz"] for c in items if c.get("sm_max_mhz")), default=None),
            "reasons": sorted({r for c in items for r in c.get("reasons", [])}),
            "samples": sum(c.get("samples", 0) for c in items)}


# ---------------------------------------------------------------------------
# Verification (outside every timed region)
# ---------------------------------------------------------------------------

def block_fingerprints(cache: torch.Tensor, chunk: int = 256) -> torch.Tensor:
    """64-bit fingerprint of every block of a [2, L, N, ...] cache, on the
    device: per (plane, layer) a wrapping dot product of the block's 64-bit
    words with fixed random odd weights, folded over planes and layers. Any
    single changed word changes it (odd weights are invertible mod 2^64)."""
    L, N = cache.shape[1], cache.shape[2]
    words = cache[0, 0, 0].numel() * cache.element_size() // 8
    gen = torch.Generator().manual_seed(97)
    w = (torch.randint(-2**62, 2**62, (words,), generator=gen, dtype=torch.int64) * 2 + 1).to(cache.device)
    fp = torch.zeros(N, dtype=torch.int64, device=cache.device)
    for kv in range(2):
        for layer in range(L):
            x = cache[kv, layer].reshape(N, -1).view(torch.int64)
            h = torch.cat([(x[i:i + chunk] * w).sum(dim=1) for i in range(0, N, chunk)])
            fp.mul_(FP_MULT).add_(h)
    return fp


def untouched_unchanged(before: torch.Tensor, after: torch.Tensor, written: list[int]) -> dict:
    keep = torch.ones(before.numel(), dtype=torch.bool, device=before.device)
    if written:
        keep[torch.tensor(sorted(set(written)), dtype=torch.long, device=before.device)] = False
    changed = int(((before != after) & keep).sum().item())
    return {"blocks_checked": int(keep.sum().item()), "blocks_changed": changed}


def verify_local(cache: torch.Tensor, src_ids: list[int], dst_ids: list[int]) -> dict:
    """1 GPU: every destination chunk equals its source chunk byte for byte."""
    dev = cache.device
    s = torch.tensor(src_ids, dtype=torch.long, device=dev)
    d = torch.tensor(dst_ids, dtype=torch.long, device=dev)
    bad = torch.zeros((), dtype=torch.int64, device=dev)
    for kv in range(2):
        for layer in range(cache.shape[1]):
            a = cache[kv, layer].index_select(0, s).view(torch.int16).reshape(len(src_ids), -1)
            b = cache[kv, layer].index_select(0, d).view(torch.int16).reshape(len(dst_ids), -1)
            bad += (a != b).any(dim=1).sum()
    return {"chunks_checked": 2 * cache.shape[1] * len(src_ids), "chunks_mismatched": int(bad.item())}


def verify_moves(cache: torch.Tensor, outgoing: dict, incoming: dict, dist) -> dict:
    """N GPUs: compare every moved chunk with what the reference's algorithm
    delivers on the same GPUs (kv_transfer.py:463-470): per (plane, layer)
    each source index_selects its blocks and NCCL-sends them, each
    destination receives them and compares byte for byte with the blocks the
    kernel wrote. ``outgoing`` = {dst: src ids}, ``incoming`` = {src: dst
    ids}, positionally matched with the peer's lists. Sums over ranks."""
    dev = cache.device
    out_idx = {d: torch.tensor(v, dtype=torch.long, device=dev) for d, v in outgoing.items() if v}
    in_idx = {s: torch.tensor(v, dtype=torch.long, device=dev) for s, v in incoming.items() if v}
    bad = torch.zeros((), dtype=torch.int64, device=dev)
    checked = 0
    for kv in range(2):
        for layer in range(cache.shape[1]):
            plane = cache[kv, layer]
            sends = {d: plane.index_select(0, idx) for d, idx in out_idx.items()}
            recvs = {s: torch.empty((len(idx), *plane.shape[1:]), dtype=plane.dtype, device=dev)
                     for s, idx in in_idx.items()}
            ops = [dist.P2POp(dist.isend, t, d) for d, t in sends.items()] + \
                  [dist.P2POp(dist.irecv, t, s) for s, t in recvs.items()]
            if ops:
                for work in dist.batch_isend_irecv(ops):
                    work.wait()
            for s, idx in in_idx.items():
                mine = plane.index_select(0, idx).view(torch.int16).reshape(len(idx), -1)
                bad += (mine != recvs[s].view(torch.int16).reshape(len(idx), -1)).any(dim=1).sum()
                checked += len(idx)
    t = torch.tensor([int(bad.item()), checked], dtype=torch.int64, device=dev)
    dist.all_reduce(t)
    return {"chunks_checked": int(t[1]), "chunks_mismatched": int(t[0])}


# ---------------------------------------------------------------------------
# CPU baselines (the reference's path on the host cores)
# ---------------------------------------------------------------------------

def cpu_reference_c_port(g: dict, blocks: int, steps: int, warmup: int, min_seconds: float = 0.0) -> dict:
    """The reference algorithm (pack into a payload, then unpack; kv_transfer.py:229-276)
    on the host cores through the C oracle, on a bounded sample of the workload."""
    from oracle import c_oracle

    threads = c_oracle.default_threads()
    n = 2 * blocks + 8
    shape = (2, g["L"], n, g["bs"], g["H"], g["D"])
    cache = torch.zeros(shape, dtype=torch.bfloat16)
    perm = seeded_perm(n, 0)
    src, dst = perm[:blocks], perm[blocks:2 * blocks]
    payload = torch.empty((g["L"], 2, blocks, g["bs"], g["H"], g["D"]), dtype=torch.bfloat16)
    cache.fill_(1.0)
    for _ in range(max(1, warmup)):
        c_oracle.swap_planned(cache, src, cache, dst, nthreads=threads, payload=payload)
    times = []
    t_start = time.perf_counter()
    while len(times) < steps or (time.perf_counter() - t_start) < min_seconds:
        t0 = time.perf_counter()
        c_oracle.swap_planned(cache, src, cache, dst, nthreads=threads, payload=payload)
        times.append(time.perf_counter() - t0)
    p = payload_bytes(g, blocks)
    mean = sum(times) / len(times)
    return {"value": p / mean / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{blocks} blocks ({p / 2**20:.0f} MiB payload) of the same geometry, cache of {n} blocks, "
                      f"{len(times)} timed pack+unpack passes ({sum(times):.1f} s), C oracle, {threads} threads",
            "ms_per_step": mean * 1e3, "steps": len(times)}


def cpu_baseline_gloo(g: dict, blocks: int, both_ways: bool, seconds: float) -> dict:
    """The reference path on CPU tensors with gloo (oracle/torch_ref.py):
    index_select pack -> gloo send/recv -> index_copy_ unpack between two
    spawned ranks on this host's cores."""
    from oracle import torch_ref

    r = torch_ref.time_gloo_pair(g, blocks, both_ways=both_ways, min_seconds=seconds)
    what = "0->1 then 1->0 (two sequential swap_in, as one pair serves both directions)" if both_ways \
        else "one direction 0->1"
    return {"value": r["GB/s"], "unit": "GB/s", "cores": r["cores"], "kind": "port",
            "sample": f"LMPool's swap_in planned path restated with its torch ops (kv_transfer.py:229-276, "
                      f":463-470) on CPU tensors: 2 spawned gloo ranks (127.0.0.1) x {r['threads_per_rank']} "
                      f"threads, {blocks} blocks of the same geometry per transfer ({what}), caches of "
                      f"{r['cache_blocks']} blocks (cost scales with blocks moved, not cache size), "
                      f"{r['steps']} timed steps ({r['total_s']:.1f} s), verified={r['verified']}",
            "ms_per_step": r["seconds_per_step"] * 1e3, "steps": r["steps"], "host": r["host"]}


def cpu_baseline_local(g: dict, blocks: int, seconds: float) -> dict:
    from oracle import torch_ref

    r = torch_ref.time_local(g, blocks, min_seconds=seconds)
    return {"value": r["GB/s"], "unit": "GB/s", "cores": r["cores"], "kind": "port",
            "sample": f"LMPool's _pack_all_layer_blocks + _unpack_all_layer_blocks restated with its torch ops "
                      f"(index_select / index_copy_, kv_transfer.py:229-276) in one process on "
                      f"{r['cores']} threads, {blocks} blocks of the same geometry, cache of {r['cache_blocks']} "
                      f"blocks, {r['steps']} timed steps ({r['total_s']:.1f} s), verified={r['verified']}",
            "ms_per_step": r["seconds_per_step"] * 1e3, "steps": r["steps"], "host": r["host"]}


# ---------------------------------------------------------------------------
# 1 GPU: config 2 and store_kvcache
# ---------------------------------------------------------------------------

def reference_gpu_local(cache: torch.Tensor, L: int, src_ids: list[int], dst_ids: list[int], steps: int) -> dict:
    """The reference's own GPU algorithm on the same device and data, restated
    with the same torch ops: _pack_all_layer_blocks (kv_transfer.py:229-248,
    2*L index_select into a staging payload) then _unpack_all_layer_blocks
    (:264-276, 2*L index_copy_). Comparison leg, not the product."""
    dev = cache.device
    B = len(src_ids)
    idx_s = torch.tensor(src_ids, dtype=torch.long, device=dev)
    idx_d = torch.tensor(dst_ids, dtype=torch.long, device=dev)

    def step():
        payload = torch.empty((L, 2, B, *cache.shape[3:]), dtype=cache.dtype, device=dev)
        for layer in range(L):
            torch.index_select(cache[0, layer], 0, idx_s, out=payload[layer, 0])
            torch.index_select(cache[1, layer], 0, idx_s, out=payload[layer, 1])
        for layer in range(L):
            cache[0, layer].index_copy_(0, idx_d, payload[layer, 0])
            cache[1, layer].index_copy_(0, idx_d, payload[layer, 1])

    for _ in range(2):
        step()
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    P = B * L * 2 * int(torch.tensor(cache.shape[3:]).prod()) * cache.element_size()
    return {"algorithm": "torch index_select -> payload -> index_copy_ (kv_transfer.py:229-276), same GPU and data",
            "launches_per_step": 4 * L, "ms_per_step": ms, "GB/s": P / (ms * 1e-3) / 1e9}


def reference_store_kvcache_step(keys, values, cache, slots, block_size: int) -> None:
    """LMPool's store_kvcache (attention.py:24-64, one program per (token,
    kv head) writing row `slot` of the flat cache unless slot == -1),
    restated with torch ops per layer as Attention.forward calls it
    (attention.py:490-507): the valid tokens are selected once per step
    (slot_mapping is shared by every layer), then per layer the K and V rows
    are index_copy_'d into the flattened caches. Comparison leg only."""
    L, T, H, D = keys.shape
    valid = (slots != -1).nonzero().flatten()
    rows = slots.index_select(0, valid)
    for layer in range(L):
        cache[0, layer].view(-1, H, D).index_copy_(0, rows, keys[layer].index_select(0, valid))
        cache[1, layer].view(-1, H, D).index_copy_(0, rows, values[layer].index_select(0, valid))


def bench_store_kvcache(dev_idx: int, peak: float, iters: int = 30, num_blocks: int = 0) -> dict:
    """store_kvcache at benchmark config 5 geometry (L=80, H=8, D=128,
    block_size=16, T=256 tokens per step, ~10% padding slots; the cache is
    shrunk to 4096 blocks: the cost does not depend on N). A step writes every
    layer: 80 single-layer launches as the model issues them (eager, and
    captured in a CUDA graph as the decode path does), or one all-layer
    launch; beside them the reference's algorithm restated with torch ops.
    L2 is flushed (written, then another buffer read) between timed steps.
    Every leg's result is checked against the reference leg's."""
    from lmpool_b200.attention import store_kvcache, store_kvcache_layers
    from lmpool_b200.kv_transfer import check_device_status

    c = dict(STORE)
    c["N"] = num_blocks or c["N"]
    dev = torch.device("cuda", dev_idx)
    gen = torch.Generator(device=dev).manual_seed(5)
    cache = torch.empty((2, c["L"], c["N"], c["bs"], c["H"], c["D"]), dtype=torch.bfloat16, device=dev)
    cache.normal_(generator=gen)
    keys = torch.empty((c["L"], c["T"], c["H"], c["D"]), dtype=torch.bfloat16, device=dev).normal_(generator=gen)
    values = torch.empty_like(keys).normal_(generator=gen)
    g = torch.Generator().manual_seed(55)
    slots = torch.randperm(c["N"] * c["bs"], generator=g)[:c["T"]].to(torch.int64)
    slots[torch.rand(c["T"], generator=g) < 0.1] = -1
    valid = int((slots >= 0).sum())
    slots = slots.to(dev)
    stream = torch.cuda.current_stream(dev)
    flush = L2Flush(dev)

    def per_layer():
        for layer in range(c["L"]):
            store_kvcache(keys[layer], values[layer], cache[0, layer], cache[1, layer], slots, c["bs"])

    def all_layers():
        store_kvcache_layers(keys, values, cache, slots, c["bs"])

    def reference():
        reference_store_kvcache_step(keys, values, cache, slots, c["bs"])

    # correctness of every leg against the reference leg, on the same start
    start = cache.clone()
    reference()
    expect = cache.clone()
    results = {}
    for name, fn in (("per_layer", per_layer), ("all_layers", all_layers)):
        cache.copy_(start)
        fn()
        results[name] = bool(torch.equal(cache.view(torch.int16), expect.view(torch.int16)))
    del start, expect
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        per_layer()
    torch.cuda.synchronize()

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        times = []
        for _ in range(iters):
            flush()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    ms_eager = timed(per_layer)
    ms_graph = timed(graph.replay)
    ms_all = timed(all_layers)
    ms_ref = timed(reference)
    check_device_status(dev_idx)
    row = c["H"] * c["D"] * 2
    traffic = c["L"] * (2 * c["T"] * row + 2 * valid * row + c["T"] * 8)
    del graph, cache, keys, values, flush
    torch.cuda.empty_cache()

    def entry(ms, launches):
        gbs = traffic / (ms * 1e-3) / 1e9
        return {"ms_per_step": ms, "us_per_layer": ms * 1e3 / c["L"], "launches_per_step": launches, "GB/s": gbs,
                "frac_hbm": gbs / peak}

    return {"geometry": dict(c, valid_tokens=valid), "bytes_per_step": traffic,
            "per_layer_eager": entry(ms_eager, c["L"]), "per_layer_graph": entry(ms_graph, c["L"]),
            "all_layers_one_launch": entry(ms_all, 1),
            "reference_torch_ops": dict(entry(ms_ref, None), algorithm=(
                "attention.py:24-64 restated with torch ops per layer (valid slots selected once per step, "
                "then index_copy_ of K and V rows per layer), eager")),
            "speedup_per_layer_graph_vs_reference": ms_ref / ms_graph,
            "bit_exact_vs_reference": results,
            "note": "bytes = per layer: read K,V rows of all T tokens + write K,V rows of valid tokens + slot ids"}


def bench_local(args) -> dict:
    from lmpool_b200 import _capi
    from lmpool_b200 import kv_transfer as kt
    from lmpool_b200.layout import affine_layout

    g = dict(LOCAL)
    g["N"] = args.cache_blocks or g["N"]
    g["B"] = args.blocks or g["B"]
    if 2 * g["B"] > g["N"]:
        raise SystemExit("--blocks must be at most half of --cache-blocks (source and destination are disjoint)")
    dev_idx = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(dev_idx)
    dev = torch.device("cuda", dev_idx)
    shape = (2, g["L"], g["N"], g["bs"], g["H"], g["D"])
    cache = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    cache.normal_(generator=torch.Generator(device=dev).manual_seed(0))
    lay = affine_layout(cache, g["L"])
    perm = seeded_perm(g["N"], 0)
    stream = torch.cuda.current_stream(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def ids_for(b):
        return (torch.tensor(perm[:b], dtype=torch.int64, device=dev),
                torch.tensor(perm[b:2 * b], dtype=torch.int64, device=dev))

    B = g["B"]
    src_t, dst_t = ids_for(B)
    P = payload_bytes(g, B)
    fp_before = None if args.quick else block_fingerprints(cache)

    def step():
        kt._launch_move(dev_idx, lay, lay, src_t, dst_t, B, status, stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(dev_idx).start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(args.steps):
        step()
    end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(end) / args.steps
    if int(status.item()) != 0:
        raise RuntimeError(f"kernel status {status.item()}")
    value = P / (ms * 1e-3) / 1e9
    peak, peak_src = hbm_peak()
    achieved = 2 * P / (ms * 1e-3) / 1e9
    traffic = profile_value("move_local_config2", "dram_bytes_per_launch_full_size")
    if args.quick:
        print(json.dumps({"quick": True, "blocks": B, "cache_blocks": g["N"], "ms_per_step": ms, "GB/s": value,
                          "hbm_GB/s": achieved, "frac": achieved / peak}), flush=True)
        return None
    verification = {"moved": verify_local(cache, perm[:B], perm[B:2 * B]),
                    "untouched": untouched_unchanged(fp_before, block_fingerprints(cache), perm[B:2 * B])}

    # B sweep, L2 flushed before each timed launch (clean, and write-only);
    # every swept move checked byte for byte after its timing
    flush = L2Flush(dev)
    sweep = []
    for b in SWEEP_B:
        s_t, d_t = ids_for(b)
        pb = payload_bytes(g, b)
        for _ in range(3):
            kt._launch_move(dev_idx, lay, lay, s_t, d_t, b, status, stream)
        iters = 30 if b <= 64 else 10
        med = {}
        for dirty in (False, True):
            times = []
            for _ in range(iters):
                flush(dirty)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                kt._launch_move(dev_idx, lay, lay, s_t, d_t, b, status, stream)
                e1.record(stream)
                e1.synchronize()
                times.append(e0.elapsed_time(e1))
            med[dirty] = statistics.median(times) * 1e-3
        t = med[False]
        chk = verify_local(cache, perm[:b], perm[b:2 * b])
        sweep.append({"blocks": b, "bytes": pb, "ms": t * 1e3, "GB/s": pb / t / 1e9,
                      "hbm_GB/s": 2 * pb / t / 1e9, "frac_hbm": 2 * pb / t / 1e9 / peak,
                      "ms_dirty_l2": med[True] * 1e3, "frac_hbm_dirty_l2": 2 * pb / med[True] / 1e9 / peak,
                      "verified_bitexact": chk["chunks_mismatched"] == 0})
    del flush
    if int(status.item()) != 0:
        raise RuntimeError(f"kernel status {status.item()}")

    # end to end through the public API: host id lists -> pinned -> device,
    # one launch, device -> host status read, every step
    e2e_steps = max(3, min(args.steps, 50))
    for _ in range(2):
        kt.move_blocks(cache, g["L"], perm[:B], perm[B:2 * B], synchronize=True)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(e2e_steps):
        kt.move_blocks(cache, g["L"], perm[:B], perm[B:2 * B], synchronize=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps

    ref_gpu = reference_gpu_local(cache, g["L"], perm[:B], perm[B:2 * B], steps=max(3, min(args.steps, 20)))
    ref_gpu["this_kernel_speedup"] = ref_gpu["ms_per_step"] / ms

    tune = _capi.Tuning()
    _capi.lib().kvx_get_tuning(_capi.ctypes.byref(tune))
    del cache
    torch.cuda.empty_cache()
    store = bench_store_kvcache(dev_idx, peak)
    cpu = cpu_baseline_gloo(g, CPU_SAMPLE_BLOCKS, both_ways=False, seconds=10.0)
    cpu_local = cpu_baseline_local(g, CPU_SAMPLE_BLOCKS, seconds=8.0)
    cpu_c = cpu_reference_c_port(g, CPU_SAMPLE_BLOCKS, steps=3, warmup=1, min_seconds=8.0)
    ok = verification["moved"]["chunks_mismatched"] == 0 and verification["untouched"]["blocks_changed"] == 0 \
        and all(r["verified_bitexact"] for r in sweep) and all(store["bit_exact_vs_reference"].values())
    return {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: bf16 N(0,1) KV cache (device generator seed 0), block ids from randperm(2048, seed 0)",
        "config": line_config(g, 1),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": 2 * P, "kernel_ms": ms},
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "cpu_baseline_host": cpu["host"],
        "cpu_baseline_local": {k: cpu_local[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "cpu_baseline_c_port": {k: cpu_c[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": P / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 2 * B * 8, "d2h_bytes_per_step": 4,
                "api": "lmpool_b200.kv_transfer.move_blocks(host id lists, synchronize=True)"},
        "gpu_launches": args.steps,
        "clocks": clk,
        "verified_bitexact": ok,
        "verification": dict(verification, method=(
            "moved: every (plane, layer, block) chunk of the timed workload compared byte for byte with its "
            "source on the device; untouched: 64-bit per-block fingerprints before and after; sweep: each "
            "swept move compared byte for byte after its timing")),
        "sweep": sweep,
        "reference_gpu_path": ref_gpu,
        "store_kvcache": store,
        "kernel": {"variant": {0: "auto", 1: "register", 2: "bulk"}[tune.variant], "launches_per_step": 1},
    }


# ---------------------------------------------------------------------------
# N GPUs: configs 3, 4 and 5
# ---------------------------------------------------------------------------

def all_partner_sets(N: int, world: int, r: int, B: int = PHASE_B_BLOCKS):
    """(incoming targets by source, outgoing sources by destination) of rank r
    in benchmark config 4 phase B: seeded-random blocks, the incoming sets
    disjoint from each other and from every outgoing set."""
    others = [x for x in range(world) if x != r]
    perm = seeded_perm(N, 5000 + r)
    inc = {s: perm[i * B:(i + 1) * B] for i, s in enumerate(others)}
    pool = perm[B * len(others):]
    out = {}
    for d in others:
        sel = seeded_perm(len(pool), 6000 + 16 * r + d)[:B]
        out[d] = [pool[i] for i in sel]
    return inc, out


def timed_max(dist, dev, stream, fn, reps: int) -> float:
    """ms per call of ``fn`` over ``reps`` back-to-back calls, CUDA events on
    ``stream``, between a barrier and a synchronize; max over ranks."""
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def scrub(cache: torch.Tensor, ids: list[int]) -> None:
    """Zero the listed blocks, so that a verification after the next move
    shows that move's bytes and not an earlier one's."""
    if ids:
        cache[:, :, torch.tensor(sorted(set(ids)), dtype=torch.long, device=cache.device)] = 0


def pair_sweep(ep, cache, g: dict, rank: int, stream, dist, mode: str) -> list[dict]:
    """benchmark config 3 on ranks 0 -> 1: B in {1, 8, 64, 256}, contiguous and
    scattered source ids. Each timed run is K back-to-back transfers in the
    given mode, cycling through disjoint id sets so no transfer re-reads
    blocks still in L2; time = max over the two ranks. The destination
    blocks are zeroed before each case, which is then verified byte for byte
    against the reference's algorithm."""
    dev = torch.device("cuda", ep.device)
    N = g["N"]
    out = []
    for B in PAIR_SWEEP_B:
        for ids_kind in ("contiguous", "scattered"):
            K = 20 if B <= 64 else 8
            nsets = max(1, min(K, (N // 2) // B))
            gen = torch.Generator().manual_seed(3000 + B)
            if ids_kind == "contiguous":
                starts = torch.randint(0, N - B, (nsets,), generator=gen).tolist()
                src_sets = [list(range(st, st + B)) for st in starts]
            else:
                perm = seeded_perm(N, 3100 + B)
                src_sets = [perm[i * B:(i + 1) * B] for i in range(nsets)]
            dperm = seeded_perm(N, 3200 + B)
            dst_sets = [dperm[i * B:(i + 1) * B] for i in range(nsets)]
            src_t = [torch.tensor(x, dtype=torch.int64, device=dev) for x in src_sets]
            dst_t = [torch.tensor(x, dtype=torch.int64, device=dev) for x in dst_sets]
            k_box = [0]

            def one():
                k = k_box[0] % nsets
                k_box[0] += 1
                if rank == 1:
                    ep.exchange(mode, ep.cache, [], [(0, src_t[k], dst_t[k], B)], 60.0, stream)
                else:
                    ep.exchange(mode, ep.cache, [(1, src_t[k], B)], [], 60.0, stream)

            flat_src = [b for s in src_sets for b in s]
            flat_dst = [b for s in dst_sets for b in s]
            if rank == 1:
                scrub(cache, flat_dst)
            for _ in range(3):
                one()
            ms = timed_max(dist, dev, stream, one, K)
            chk = verify_moves(cache, {1: flat_src} if rank == 0 else {}, {0: flat_dst} if rank == 1 else {}, dist)
            pb = payload_bytes(g, B)
            out.append({"mode": mode, "blocks": B, "ids": ids_kind, "bytes": pb, "ms": ms,
                        "GB/s": pb / (ms * 1e-3) / 1e9, "frac_nvlink": pb / (ms * 1e-3) / 1e9 / NVLINK_NOMINAL_GBS,
                        "verified_bitexact": chk["chunks_mismatched"] == 0, "chunks_checked": chk["chunks_checked"]})
    return out


def reference_gpu_pair(cache: torch.Tensor, g: dict, rank: int, dist, blocks=PAIR_SWEEP_B) -> dict:
    """The reference's planned swap_in on the same two GPUs, restated with the
    same ops (kv_transfer.py:463-470): rank 0 packs with 2*L index_select and
    NCCL-sends the payload, rank 1 receives it and unpacks with 2*L
    index_copy_; timed like benchmark_kv_transfer.py:138-170 (barrier,
    synchronize, wall clock) per transfer, max over the two ranks, at every
    block count of the config 3 sweep (scattered ids). Comparison leg; the
    headline fields are the B=64 entry."""
    dev = cache.device
    L = g["L"]
    out = []
    for B in blocks:
        src_ids = seeded_perm(g["N"], 8000 + B)[:B]
        dst_ids = seeded_perm(g["N"], 8001 + B)[:B]
        idx = torch.tensor(src_ids if rank == 0 else dst_ids, dtype=torch.long, device=dev)
        shape = (L, 2, B, *cache.shape[3:])

        def one():
            if rank == 0:
                payload = torch.empty(shape, dtype=cache.dtype, device=dev)
                for layer in range(L):
                    torch.index_select(cache[0, layer], 0, idx, out=payload[layer, 0])
                    torch.index_select(cache[1, layer], 0, idx, out=payload[layer, 1])
                dist.send(payload, dst=1)
            elif rank == 1:
                payload = torch.empty(shape, dtype=cache.dtype, device=dev)
                dist.recv(payload, src=0)
                for layer in range(L):
                    cache[0, layer].index_copy_(0, idx, payload[layer, 0])
                    cache[1, layer].index_copy_(0, idx, payload[layer, 1])

        iters = 10 if B <= 64 else 5
        times = []
        for k in range(3 + iters):
            dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            one()
            torch.cuda.synchronize()
            if k >= 3:
                times.append((time.perf_counter() - t0) * 1e3)
        ms_dev = timed_max(dist, dev, torch.cuda.current_stream(dev), one, iters)
        t = torch.tensor([statistics.mean(times)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_wall = float(t.item())
        P = payload_bytes(g, B)
        out.append({"blocks": B, "ms": ms_dev, "GB/s": P / (ms_dev * 1e-3) / 1e9,
                    "ms_wall": ms_wall, "GB/s_wall": P / (ms_wall * 1e-3) / 1e9})
    torch.cuda.empty_cache()
    head = next((r for r in out if r["blocks"] == 64), out[-1])
    return {"algorithm": "index_select pack -> NCCL send/recv -> index_copy_ unpack (kv_transfer.py:463-470)",
            "timing": "ms: back-to-back transfers timed with CUDA events (as pair_sweep times this kernel), max "
                      "over ranks; ms_wall: one transfer between barriers, host clock, as "
                      "benchmark_kv_transfer.py:138-170 times it; this_kernel_speedup divides the smaller of "
                      "the two by this kernel's best device-timed scattered transfer",
            "blocks": head["blocks"], "ms": head["ms"], "GB/s": head["GB/s"], "ms_wall": head["ms_wall"],
            "sweep": out}


def reference_phase_a(cache: torch.Tensor, g: dict, rank: int, world: int, dist, src_ids, partner_src, dst_ids,
                      iters: int = 5) -> dict:
    """Phase A with the reference's algorithm on the same GPUs: per pair, the
    two directions as two sequential planned swap_in calls (LMPool runs one
    plan per pair at a time; two opposite NCCL swaps at once would block each
    other on the pair's stream): pack (2*L index_select) -> NCCL send/recv ->
    unpack (2*L index_copy_), 0->1 then 1->0. Device-timed, max over ranks."""
    dev = cache.device
    L, B = g["L"], g["B"]
    partner = rank + 1 if rank % 2 == 0 else rank - 1
    out_idx = torch.tensor(src_ids, dtype=torch.long, device=dev)
    in_idx = torch.tensor(dst_ids, dtype=torch.long, device=dev)
    shape = (L, 2, B, *cache.shape[3:])

    def send():
        payload = torch.empty(shape, dtype=cache.dtype, device=dev)
        for layer in range(L):
            torch.index_select(cache[0, layer], 0, out_idx, out=payload[layer, 0])
            torch.index_select(cache[1, layer], 0, out_idx, out=payload[layer, 1])
        dist.send(payload, dst=partner)

    def recv():
        payload = torch.empty(shape, dtype=cache.dtype, device=dev)
        dist.recv(payload, src=partner)
        for layer in range(L):
            cache[0, layer].index_copy_(0, in_idx, payload[layer, 0])
            cache[1, layer].index_copy_(0, in_idx, payload[layer, 1])

    def one():
        if rank % 2 == 0:
            send()
            recv()
        else:
            recv()
            send()

    for _ in range(2):
        one()
    ms = timed_max(dist, dev, torch.cuda.current_stream(dev), one, iters)
    torch.cuda.empty_cache()
    P = payload_bytes(g, B)
    return {"algorithm": "per pair: two sequential planned swap_in (index_select -> NCCL send/recv -> index_copy_, "
                         "kv_transfer.py:463-470), 0->1 then 1->0", "ms_per_step": ms,
            "value": world * P / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "GB/s_per_direction_averaged": P / (ms * 1e-3) / 1e9}


def reference_all_partner(cache: torch.Tensor, g: dict, rank: int, world: int, dist, iters: int = 5) -> dict:
    """Phase B with the reference's ops on the same GPUs: every rank packs each
    destination's blocks with 2*L index_select (kv_transfer.py:463-466), all
    payloads cross in one NCCL batch of send/recv pairs, and each received
    payload is unpacked with 2*L index_copy_ (kv_transfer.py:468-470); wall
    clock per step between barriers, max over ranks. Comparison leg."""
    dev = cache.device
    L, B = g["L"], PHASE_B_BLOCKS
    peers = [r for r in range(world) if r != rank]
    incoming, outgoing = all_partner_sets(g["N"], world, rank)
    out_idx = {d: torch.tensor(v, dtype=torch.long, device=dev) for d, v in outgoing.items()}
    in_idx = {s: torch.tensor(v, dtype=torch.long, device=dev) for s, v in incoming.items()}
    shape = (L, 2, B, *cache.shape[3:])
    send = {d: torch.empty(shape, dtype=cache.dtype, device=dev) for d in peers}
    recv = {s: torch.empty(shape, dtype=cache.dtype, device=dev) for s in peers}

    def one():
        for d in peers:
            for layer in range(L):
                torch.index_select(cache[0, layer], 0, out_idx[d], out=send[d][layer, 0])
                torch.index_select(cache[1, layer], 0, out_idx[d], out=send[d][layer, 1])
        ops = [dist.P2POp(dist.isend, send[d], d) for d in peers] + \
              [dist.P2POp(dist.irecv, recv[s], s) for s in peers]
        for work in dist.batch_isend_irecv(ops):
            work.wait()
        for s in peers:
            for layer in range(L):
                cache[0, layer].index_copy_(0, in_idx[s], recv[s][layer, 0])
                cache[1, layer].index_copy_(0, in_idx[s], recv[s][layer, 1])

    written = [b for v in incoming.values() for b in v]
    fp_before = block_fingerprints(cache)     # the kernel legs just wrote these blocks from the same sources
    times = []
    for k in range(2 + iters):
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        one()
        torch.cuda.synchronize()
        if k >= 2:
            times.append((time.perf_counter() - t0) * 1e3)
    t = torch.tensor([statistics.mean(times)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    fp_after = block_fingerprints(cache)
    same = bool(torch.equal(fp_before, fp_after))
    agree = [None] * world
    dist.all_gather_object(agree, same)
    del send, recv
    torch.cuda.empty_cache()
    pb = payload_bytes(g, B)
    per_gpu_out = (world - 1) * pb / (ms * 1e-3) / 1e9
    return {"algorithm": "index_select pack -> NCCL batched send/recv -> index_copy_ unpack",
            "blocks_per_destination": B, "ms_per_step": ms,
            "value": world * (world - 1) * pb / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "per_gpu_egress_GB/s": per_gpu_out, "blocks_rewritten": len(written),
            "same_blocks_as_kernel": all(agree)}


def all_partner(ep, cache, g: dict, rank: int, world: int, stream, dist, mode: str,
                schedule: str = "concurrent") -> dict:
    """benchmark config 4 phase B: every rank sends B=32 seeded-random blocks to
    every other rank, into disjoint reserved sets.

    ``concurrent``: one exchange per step carries every destination and
    source at once (one push or pull launch per rank). ``rotated``: one
    exchange per round of a round-robin tournament over the ranks; in each
    round every GPU exchanges both ways with one partner, the traffic
    pattern of disjoint pairs."""
    dev = torch.device("cuda", ep.device)
    N, B = g["N"], PHASE_B_BLOCKS
    peers = [r for r in range(world) if r != rank]
    incoming, outgoing = all_partner_sets(N, world, rank)
    peer_out = {s: all_partner_sets(N, world, s)[1][rank] for s in peers}   # what each peer sends here
    in_t = {s: torch.tensor(v, dtype=torch.int64, device=dev) for s, v in incoming.items()}
    out_t = {d: torch.tensor(v, dtype=torch.int64, device=dev) for d, v in outgoing.items()}
    psrc_t = {s: torch.tensor(v, dtype=torch.int64, device=dev) for s, v in peer_out.items()}

    if schedule == "concurrent":
        def step():
            ep.exchange(mode, ep.cache, [(d, out_t[d], B) for d in peers],
                        [(s, psrc_t[s], in_t[s], B) for s in peers], 60.0, stream)
    elif schedule == "rotated":
        def step():
            ep.exchange_rotated(mode, ep.cache, [(d, out_t[d], B) for d in peers],
                                [(s, psrc_t[s], in_t[s], B) for s in peers], 60.0, stream)
    else:
        raise ValueError(f"unknown schedule {schedule!r}")

    ep.status.zero_()
    written = [b for v in incoming.values() for b in v]
    scrub(cache, written)
    fp_before = block_fingerprints(cache)
    for _ in range(3):
        step()
    ms = timed_max(dist, dev, stream, step, 10)
    bits = int(ep.status.item())
    chk = verify_moves(cache, outgoing, incoming, dist)
    unt = untouched_unchanged(fp_before, block_fingerprints(cache), written)
    oks: list = [None] * world
    dist.all_gather_object(oks, bits == 0 and unt["blocks_changed"] == 0)
    ok = all(oks) and chk["chunks_mismatched"] == 0
    pb = payload_bytes(g, B)
    per_gpu_out = (world - 1) * pb / (ms * 1e-3) / 1e9
    return {"ok": bool(ok), "schedule": schedule, "mode": mode, "blocks_per_destination": B, "ms_per_step": ms,
            "value": world * (world - 1) * pb / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "per_gpu_egress_GB/s": per_gpu_out, "frac_nvlink_per_gpu_egress": per_gpu_out / NVLINK_NOMINAL_GBS,
            "verified_bitexact": bool(ok), "chunks_checked": chk["chunks_checked"]}


def peer_copy(ep, partner: int, rank: int, stream, dist, nbytes: int = 2 << 30) -> dict | None:
    """Plain peer copies over the same NVLink, for the record beside the
    kernel: cudaMemcpyAsync (copy engine) from the partner's cache (through
    this process's IPC mapping) into a local buffer, timed with CUDA events,
    one direction (even ranks copy, odd ranks idle) and both at once. Only
    reads the partner's memory."""
    try:
        from cuda.bindings import runtime as rt
    except ImportError:
        return None
    dev = torch.device("cuda", ep.device)
    link = ep.get_link(partner)
    src_ptr = link.cache.base
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)

    def cp(active: bool):
        if active:
            err, = rt.cudaMemcpyAsync(dst.data_ptr(), src_ptr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                      stream.cuda_stream)
            if err != rt.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cudaMemcpyAsync: {err}")

    for _ in range(2):
        cp(True)
    one = timed_max(dist, dev, stream, lambda: cp(rank % 2 == 0), 5)
    both = timed_max(dist, dev, stream, lambda: cp(True), 5)
    del dst
    torch.cuda.empty_cache()
    return {"method": "cudaMemcpyAsync from the partner's memory (IPC mapping) into local HBM, 2 GiB, CUDA events, "
                      "max over ranks",
            "one_direction_GB/s": nbytes / (one * 1e-3) / 1e9, "both_directions_GB/s_per_direction":
                nbytes / (both * 1e-3) / 1e9}


def e2e_swap_in(kt, cache, g, rank: int, partner: int, src_ids, partner_src, dst_ids, stream, dist,
                steps: int) -> dict:
    """Phase A end to end through the reference-facing API: per pair, swap_in
    0->1 then swap_in 1->0 (LMPool's data plane issues one plan per pair at a
    time, ModelRunner.execute_swap_out/in -> swap_in(negotiate_blocks=False),
    model_runner.py:747-806), host id lists in, status read back, in the
    process's transfer mode (pull). Also the source's call latency with the
    source returning after the read and once its grant is enqueued."""
    L, bs, H, D = g["L"], g["bs"], g["H"], g["D"]
    dev = torch.device("cuda", kt._local_device(rank))
    even = rank % 2 == 0

    def as_source():
        kt.swap_in(rank, src_ids, partner, cache, L, bs, H, D, negotiate_blocks=False)

    def as_destination():
        kt.swap_in(partner, partner_src, rank, cache, L, bs, H, D, local_target_blocks=dst_ids,
                   negotiate_blocks=False)

    def step():
        if even:
            as_source()
            as_destination()
        else:
            as_destination()
            as_source()

    for _ in range(2):
        step()
    ms = timed_max(dist, dev, stream, step, steps)
    # the source's call latency (host wall clock), both settings of LMPOOL_B200_SOURCE_RETURN
    lat = {}
    old = os.environ.get("LMPOOL_B200_SOURCE_RETURN")
    for setting in ("read", "granted"):
        os.environ["LMPOOL_B200_SOURCE_RETURN"] = setting
        vals = []
        for _ in range(5):
            torch.cuda.synchronize()
            dist.barrier()
            if even:
                t0 = time.perf_counter()
                as_source()
                vals.append((time.perf_counter() - t0) * 1e3)
            else:
                as_destination()
            torch.cuda.synchronize()
        if even:
            lat[setting] = statistics.median(vals)
    if old is None:
        os.environ.pop("LMPOOL_B200_SOURCE_RETURN", None)
    else:
        os.environ["LMPOOL_B200_SOURCE_RETURN"] = old
    kt._ENDPOINTS[dev.index].poll_deferred(wait=True)
    return {"ms_per_step": ms, "source_call_ms": lat}


def config5_leg(kt, rank: int, world: int, dist, steps: int, mode: str) -> dict:
    """benchmark config 5 on the pairs: the transfer alone, store_kvcache
    alone, and both at once on two streams. The cache is shrunk from 65536 to
    16384 blocks per rank (80 GiB; 65536 would be 320 GiB): transfer and store
    costs depend on B and T, not on N. Transfers verified byte for byte
    against the reference's algorithm; every stored row checked."""
    from lmpool_b200.attention import store_kvcache, store_kvcache_layers

    c = CONFIG5
    local = kt._local_device(rank)
    dev = torch.device("cuda", local)
    cache = torch.empty((2, c["L"], c["N"], c["bs"], c["H"], c["D"]), dtype=torch.bfloat16, device=dev)
    gen = torch.Generator(device=dev).manual_seed(rank)
    cache.normal_(generator=gen)
    keys = torch.empty((c["L"], c["T"], c["H"], c["D"]), dtype=torch.bfloat16, device=dev).normal_(generator=gen)
    values = torch.empty_like(keys).normal_(generator=gen)
    kt.register_kv_cache(cache, c["L"])
    pairs = [(r, r + 1) for r in range(0, world, 2)]
    kt.prewarm_p2p_pairs(pairs, num_layers=c["L"], block_size=c["bs"], num_kv_heads=c["H"], head_dim=c["D"],
                         num_blocks=2, dtype=torch.bfloat16, timeout_s=60)
    partner = rank + 1 if rank % 2 == 0 else rank - 1
    B = c["B"]
    perm = seeded_perm(c["N"], 7000 + rank)
    src_ids, dst_ids = perm[:B], perm[B:2 * B]          # fragmented, disjoint
    partner_src = seeded_perm(c["N"], 7000 + partner)[:B]
    # store_kvcache slots avoid both transfer sets (blocks being moved are
    # locked: the model never writes them)
    busy = torch.zeros(c["N"], dtype=torch.bool)
    busy[src_ids] = True
    busy[dst_ids] = True
    free_blocks = (~busy).nonzero().flatten()
    g = torch.Generator().manual_seed(77 + rank)
    pick = free_blocks[torch.randperm(len(free_blocks), generator=g)[:c["T"]]]
    slots = pick * c["bs"] + torch.randint(0, c["bs"], (c["T"],), generator=g)
    slots[torch.rand(c["T"], generator=g) < 0.1] = -1
    slots = slots.to(torch.int64).to(dev)
    ep = kt._ENDPOINTS[local]
    xs = torch.cuda.Stream(dev)
    ss = torch.cuda.Stream(dev)
    src_t = torch.tensor(src_ids, dtype=torch.int64, device=dev)
    dst_t = torch.tensor(dst_ids, dtype=torch.int64, device=dev)
    psrc_t = torch.tensor(partner_src, dtype=torch.int64, device=dev)
    P = B * c["L"] * 2 * c["bs"] * c["H"] * c["D"] * 2
    row = c["H"] * c["D"] * 2
    valid = int((slots >= 0).sum())
    store_bytes = c["L"] * (2 * c["T"] * row + 2 * valid * row + c["T"] * 8)

    def xfer():
        ep.exchange(mode, ep.cache, [(partner, src_t, B)], [(partner, psrc_t, dst_t, B)], 60.0, xs)

    def store_step():
        with torch.cuda.stream(ss):
            store_kvcache_layers(keys, values, cache, slots, c["bs"])

    with torch.cuda.stream(ss):
        for layer in range(c["L"]):   # warm the single-layer launch too
            store_kvcache(keys[layer], values[layer], cache[0, layer], cache[1, layer], slots, c["bs"])
    ep.status.zero_()
    for _ in range(3):
        xfer()
        store_step()
    torch.cuda.synchronize()
    K = max(3, min(steps, 10))
    x_ms = timed_max(dist, dev, xs, xfer, K)
    s_ms = timed_max(dist, dev, ss, store_step, 200)
    M = max(1, int(K * x_ms / s_ms))
    # both at once: K transfers on one stream, M store steps on another, same start
    dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    start.record(torch.cuda.current_stream(dev))
    xs.wait_event(start)
    ss.wait_event(start)
    xe, se = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for k in range(max(K, M)):
        if k < K:
            xfer()
        if k < M:
            store_step()
    xe.record(xs)
    se.record(ss)
    torch.cuda.synchronize()
    t = torch.tensor([start.elapsed_time(xe) / K, start.elapsed_time(se) / M], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    xo_ms, so_ms = float(t[0]), float(t[1])
    bits = int(ep.status.item())
    kt.check_device_status(local)
    chk = verify_moves(cache, {partner: src_ids}, {partner: dst_ids}, dist)
    vidx = (slots >= 0).nonzero().flatten()
    vs = slots.index_select(0, vidx)
    k_rows = cache[0].reshape(c["L"], -1, c["H"], c["D"]).index_select(1, vs)
    v_rows = cache[1].reshape(c["L"], -1, c["H"], c["D"]).index_select(1, vs)
    stored_ok = bool(torch.equal(k_rows.view(torch.int16), keys.index_select(1, vidx).view(torch.int16))) and \
        bool(torch.equal(v_rows.view(torch.int16), values.index_select(1, vidx).view(torch.int16)))
    oks: list = [None] * world
    dist.all_gather_object(oks, bits == 0 and stored_ok)
    kt.shutdown()
    del cache, keys, values
    torch.cuda.empty_cache()
    return {
        "workload": c["workload"], "config": {k: c[k] for k in ("L", "N", "bs", "H", "D", "B", "T")},
        "substitution": "num_blocks 65536 -> 16384 per rank (320 GiB does not fit one B200)",
        "transfer_mode": mode,
        "transfer_alone": {"ms": x_ms, "GB/s_per_direction": P / (x_ms * 1e-3) / 1e9,
                           "frac_nvlink": P / (x_ms * 1e-3) / 1e9 / NVLINK_NOMINAL_GBS},
        "store_alone": {"ms_per_step": s_ms, "GB/s": store_bytes / (s_ms * 1e-3) / 1e9,
                        "launch": "all 80 layers in one launch"},
        "overlapped": {"transfers": K, "store_steps": M, "transfer_ms": xo_ms,
                       "transfer_GB/s_per_direction": P / (xo_ms * 1e-3) / 1e9,
                       "store_ms_per_step": so_ms, "store_GB/s": store_bytes / (so_ms * 1e-3) / 1e9},
        "payload_bytes_per_direction": P, "store_bytes_per_step": store_bytes,
        "verified_bitexact": all(oks) and chk["chunks_mismatched"] == 0, "chunks_checked": chk["chunks_checked"],
    }


def bench_pairs(args) -> dict | None:
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world % 2:
        raise SystemExit("--gpus must be even for the pair benchmark")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    g = PAIRS
    shape = (2, g["L"], g["N"], g["bs"], g["H"], g["D"])
    cache = torch.empty(shape, dtype=torch.bfloat16, device=dev)
    cache.normal_(generator=torch.Generator(device=dev).manual_seed(rank))
    kt.register_kv_cache(cache, g["L"])
    pairs = [(r, r + 1) for r in range(0, world, 2)]
    kt.prewarm_p2p_pairs(pairs, num_layers=g["L"], block_size=g["bs"], num_kv_heads=g["H"], head_dim=g["D"],
                         num_blocks=2, dtype=torch.bfloat16, timeout_s=60)
    partner = rank + 1 if rank % 2 == 0 else rank - 1
    B = g["B"]
    src_ids = seeded_perm(g["N"], 1000 + rank)[:B]
    partner_src = seeded_perm(g["N"], 1000 + partner)[:B]
    # destination ids on this rank for the partner's blocks: distinct from
    # this rank's own outgoing sources
    free = [b for b in seeded_perm(g["N"], 2000 + rank) if b not in set(src_ids)]
    dst_ids = free[:B]
    ep = kt._ENDPOINTS[local]
    # Both directions of a pair at once: push measured faster (pull's read
    # requests share each direction with the other flow's data).
    mode = "push" if args.pair_mode == "auto" else args.pair_mode
    other = "pull" if mode == "push" else "push"
    stream = torch.cuda.current_stream(dev)
    src_t = torch.tensor(src_ids, dtype=torch.int64, device=dev)
    psrc_t = torch.tensor(partner_src, dtype=torch.int64, device=dev)
    dst_t = torch.tensor(dst_ids, dtype=torch.int64, device=dev)
    P = payload_bytes(g, B)

    def step(m=None):
        ep.exchange(m or mode, ep.cache, [(partner, src_t, B)], [(partner, psrc_t, dst_t, B)], 60.0, stream)

    fp_before = block_fingerprints(cache)
    ep.status.zero_()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local).start()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    clk = clocks.stop()
    ms_local = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms_local], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    bits = int(ep.status.item())
    # bit-exact verification of the timed workload (outside the timed region)
    phase_a_chk = verify_moves(cache, {partner: src_ids}, {partner: dst_ids}, dist)
    phase_a_unt = untouched_unchanged(fp_before, block_fingerprints(cache), dst_ids)
    gathered: list = [None] * world
    dist.all_gather_object(gathered, {"rank": rank, "bits": bits, "clk": clk, "untouched": phase_a_unt})
    ok = all(item["bits"] == 0 and item["untouched"]["blocks_changed"] == 0 for item in gathered)
    ok &= phase_a_chk["chunks_mismatched"] == 0

    # the same exchange in the other mode, for the record
    for _ in range(3):
        step(other)
    other_ms = timed_max(dist, dev, stream, lambda: step(other), 10)

    # Legs beside the headline run under a guard: an exception that every
    # rank meets at the same point is recorded in the line instead of losing
    # it; a byte mismatch is not an exception and still fails the run.
    errors: dict = {}

    def guarded(name, fn):
        try:
            return fn()
        except Exception as exc:  # noqa: BLE001 - recorded in the line
            errors[name] = f"{type(exc).__name__}: {exc}"[:400]
            return None

    copies = guarded("peer_copy", lambda: peer_copy(ep, partner, rank, stream, dist))
    sweep = None
    if world == 2:   # one direction at a time: both modes, pull is the default of swap_in
        sweep = guarded("pair_sweep", lambda: pair_sweep(ep, cache, g, rank, stream, dist, "pull") +
                        pair_sweep(ep, cache, g, rank, stream, dist, "push"))
        ok &= all(r["verified_bitexact"] for r in sweep or [])
    ref_pair = guarded("reference_gpu_pair", lambda: reference_gpu_pair(cache, g, rank, dist)) if world == 2 \
        else None
    if ref_pair is not None and sweep is not None:
        for row in [ref_pair] + ref_pair["sweep"]:
            mine = [r["ms"] for r in sweep if r["blocks"] == row["blocks"] and r["ids"] == "scattered"]
            if mine:   # against the reference's better timing of the two
                row["this_kernel_speedup"] = min(row["ms"], row["ms_wall"]) / min(mine)
    phase_b = None
    if world >= 4:
        phase_b = {}
        for sched in ("concurrent", "rotated"):
            for m in ("push", "pull"):
                key = m if sched == "concurrent" else f"{m}_{sched}"
                res = guarded(f"phase_b_{key}", lambda: all_partner(ep, cache, g, rank, world, stream, dist, m,
                                                                     sched))
                if res is not None:
                    phase_b[key] = res
                    ok &= res["ok"]
        ref_b = guarded("phase_b_reference", lambda: reference_all_partner(cache, g, rank, world, dist))
        if ref_b is not None:
            phase_b["reference_nccl"] = ref_b

    # the reference's algorithm on the same GPUs for the headline workload
    ref_a = guarded("reference_phase_a", lambda: reference_phase_a(cache, g, rank, world, dist, src_ids, partner_src,
                                                                    dst_ids))
    if ref_a is not None:
        ref_a["this_kernel_speedup"] = ref_a["ms_per_step"] / ms

    # end to end through swap_in (the API LMPool calls), then through swap_batch;
    # the destination blocks are zeroed before each and verified after it
    e2e_steps = max(3, min(args.steps, 20))
    scrub(cache, dst_ids)
    e2e_in = guarded("e2e_swap_in", lambda: e2e_swap_in(kt, cache, g, rank, partner, src_ids, partner_src, dst_ids,
                                                         stream, dist, e2e_steps))
    e2e_in_chk = verify_moves(cache, {partner: src_ids}, {partner: dst_ids}, dist) if e2e_in else None
    ok &= e2e_in_chk is None or e2e_in_chk["chunks_mismatched"] == 0
    scrub(cache, dst_ids)

    def batch_leg():
        for _ in range(2):
            kt.swap_batch([(partner, src_ids)], [(partner, partner_src, dst_ids)], mode=mode)
        return timed_max(dist, dev, stream,
                         lambda: kt.swap_batch([(partner, src_ids)], [(partner, partner_src, dst_ids)], mode=mode),
                         e2e_steps)

    batch_ms = guarded("e2e_swap_batch", batch_leg)
    e2e_chk = verify_moves(cache, {partner: src_ids}, {partner: dst_ids}, dist) if batch_ms else None
    ok &= e2e_chk is None or e2e_chk["chunks_mismatched"] == 0
    kt.shutdown()
    kt._REGISTERED.pop(local, None)
    del cache
    ep = None
    torch.cuda.empty_cache()

    c5 = guarded("config5", lambda: config5_leg(kt, rank, world, dist, args.steps, mode))
    ok &= c5 is None or c5["verified_bitexact"]
    oks = [None] * world
    dist.all_gather_object(oks, bool(ok))
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    if not all(oks):
        raise RuntimeError("pair transfer verification failed")
    cpu = guarded("cpu_baseline", lambda: cpu_baseline_gloo(g, CPU_SAMPLE_BLOCKS, both_ways=True, seconds=10.0))
    if e2e_in is not None:
        e2e = {"value": world * P / (e2e_in["ms_per_step"] * 1e-3) / 1e9, "unit": "GB/s",
               "ms_per_step": e2e_in["ms_per_step"], "h2d_bytes_per_step": 2 * B * 8, "d2h_bytes_per_step": 8,
               "api": "lmpool_b200.kv_transfer.swap_in(negotiate_blocks=False), host id lists: per pair 0->1 then "
                      "1->0 as two plans (LMPool runs one plan per pair at a time), pull mode",
               "source_call_ms": e2e_in["source_call_ms"]}
    elif batch_ms:
        e2e = {"value": world * P / (batch_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": batch_ms,
               "h2d_bytes_per_step": 3 * B * 8, "d2h_bytes_per_step": 4,
               "api": f"lmpool_b200.kv_transfer.swap_batch (both directions at once, {mode})"}
    else:
        e2e = None
    if e2e is not None and batch_ms:
        e2e["swap_batch"] = {"value": world * P / (batch_ms * 1e-3) / 1e9, "ms_per_step": batch_ms,
                             "api": f"lmpool_b200.kv_transfer.swap_batch (both directions at once, {mode})"}
    value = world * P / (ms * 1e-3) / 1e9
    per_dir = P / (ms * 1e-3) / 1e9
    wire_per_block = profile_value("push_nvlink_pair", "nvlink_tx_bytes_per_block")
    traffic = wire_per_block * B if wire_per_block else None
    return {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: bf16 N(0,1) KV caches (device generator seed = rank), seeded randperm ids",
        "config": line_config(g, world),
        "roofline": {"bound": "nvlink", "achieved": per_dir, "peak": NVLINK_NOMINAL_GBS, "unit": "GB/s",
                     "frac": per_dir / NVLINK_NOMINAL_GBS, "traffic": traffic,
                     "traffic_kind": "NVLink bytes on the wire per push launch and direction (payload + 18.75% "
                                     "posted-write packet overhead), from profiles/push_nvlink_pair.txt scaled by "
                                     "blocks",
                     "peak_source": "NVLink 5 per-direction bandwidth, 900 GB/s nominal (the north-star's figure)",
                     "posted_write_ceiling_GB/s": NVLINK_NOMINAL_GBS / 1.1875,
                     "frac_of_posted_write_ceiling": per_dir / (NVLINK_NOMINAL_GBS / 1.1875),
                     "peer_copy_measured": copies,
                     "frac_of_measured_peer_copy": (per_dir / copies["both_directions_GB/s_per_direction"])
                     if copies else None},
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")} if cpu else None,
        "cpu_baseline_host": cpu["host"] if cpu else None,
        "e2e": e2e,
        "gpu_launches": (4 if mode == "push" else 5) * args.steps,
        "transfer_mode": mode,
        "verified_bitexact": True,
        "verification": {"phase_a": phase_a_chk, "phase_a_untouched": [x["untouched"] for x in gathered],
                         "after_e2e_swap_in": e2e_in_chk, "after_e2e_swap_batch": e2e_chk,
                         "method": "every moved (plane, layer, block) chunk compared byte for byte with the bytes "
                                   "the reference's algorithm delivers on the same GPUs (index_select -> NCCL "
                                   "send/recv per plane and layer); untouched blocks: 64-bit per-block "
                                   "fingerprints before and after; config 3 cases, phase B schedules and config 5 "
                                   "verified the same way"},
        "other_mode": {"mode": other, "ms_per_step": other_ms,
                       "GB/s_per_direction": P / (other_ms * 1e-3) / 1e9,
                       "frac_nvlink": P / (other_ms * 1e-3) / 1e9 / NVLINK_NOMINAL_GBS},
        "clocks": merge_clocks([item["clk"] for item in gathered]),
        "reference_gpu_phase_a": ref_a,
        "pair_sweep": sweep,
        "reference_gpu_path": ref_pair,
        "phase_b": ({m: {k: v for k, v in r.items() if k != "ok"} for m, r in phase_b.items()} if phase_b else None),
        "config5": c5,
        "errors": errors or None,
    }


def bench_pair_one_process(args) -> dict:
    """One process drives cuda:0 (source) and cuda:1 (destination): the pair
    protocol at Qwen3-8B geometry with launches enqueued in dependency order
    (push: publish on 1, wait_armed + push on 0, wait_done on 1; pull:
    request on 1, grant on 0, wait for the grant + pull on 1), so every
    bounded wait is satisfied by a launch issued before it. Used for
    profiling the NVLink kernels with one process, and as a quick pair number."""
    from lmpool_b200.endpoint import TransferEndpoint
    from lmpool_b200.layout import affine_layout

    if torch.cuda.device_count() < 2:
        raise SystemExit("pair1p needs 2 GPUs")
    g = dict(PAIRS)
    g["N"] = args.cache_blocks or g["N"]
    g["B"] = args.blocks or g["B"]
    B, N = g["B"], g["N"]
    if 2 * B > N:
        raise SystemExit("--blocks must be at most half of --cache-blocks")
    caches, eps = [], []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        t = torch.empty((2, g["L"], N, g["bs"], g["H"], g["D"]), dtype=torch.bfloat16, device=dev)
        t.normal_(generator=torch.Generator(device=dev).manual_seed(d))
        caches.append(t)
        ep = TransferEndpoint(d, 2, d, N)
        ep.set_cache(affine_layout(t, g["L"]), t)
        eps.append(ep)
    l01 = eps[0].link(eps[1].export_record())
    l10 = eps[1].link(eps[0].export_record())
    perm = seeded_perm(N, 11)
    src_t = torch.tensor(perm[:B], dtype=torch.int64, device="cuda:0")
    dst_t = torch.tensor(perm[B:2 * B], dtype=torch.int64, device="cuda:1")
    s0, s1 = torch.cuda.current_stream(0), torch.cuda.current_stream(1)
    src_on_1 = src_t.to("cuda:1")

    def one():
        token = eps[1].next_token(0)
        if args.pull:
            eps[1].request(l10, B, token, s1)
            eps[0].grant(l01, B, 30.0, s0)
            eps[1].wait_done(0, token, 30.0, s1)
            eps[1].pull(eps[1].cache, [(l10, l10.cache, src_on_1, dst_t, B, token)], s1)
            eps[0].wait_pulled(1, 30.0, s0)
            return
        eps[1].publish(l10, dst_t, B, token, s1)
        eps[0].wait_armed(l01, B, 30.0, s0)
        eps[0].push(eps[0].cache, [(l01, l01.cache, src_t, B)], s0)
        eps[1].wait_done(0, token, 30.0, s1)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    timed_dev, timed_stream = (1, s1) if args.pull else (0, s0)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.device(timed_dev):
        e0.record(timed_stream)
    for _ in range(args.steps):
        one()
    with torch.cuda.device(timed_dev):
        e1.record(timed_stream)
    torch.cuda.synchronize(0)
    torch.cuda.synchronize(1)
    ms = e0.elapsed_time(e1) / args.steps
    eps[0].check_status(s0, "pair1p source")
    eps[1].check_status(s1, "pair1p destination")
    ok = all(torch.equal(caches[1][:, :, perm[B + i]].cpu().view(torch.int16),
                         caches[0][:, :, perm[i]].cpu().view(torch.int16)) for i in (0, B - 1))
    for ep in eps:
        ep.close_links()
    for ep in eps:
        ep.close()
    P = payload_bytes(g, B)
    return {"workload": "pair, one process, cuda:0 -> cuda:1, " + ("pull by cuda:1" if args.pull else "push by cuda:0"),
            "blocks": B, "cache_blocks": N, "ms_per_step": ms,
            "GB/s": P / (ms * 1e-3) / 1e9, "frac_nvlink": P / (ms * 1e-3) / 1e9 / NVLINK_NOMINAL_GBS, "verified": ok}


def bench_local_tuning(args) -> dict:
    """``--workload localtune``: 1-GPU moves at config 2 geometry for B in
    {1, 4, 16, 64} over a grid of launch settings (bulk ring stages x tile x
    CTAs per SM, and the register engine), L2 flushed (written, then another
    buffer read) before every timed launch, median of 20 launches; each
    setting's result checked byte for byte. Measurement sweep behind the
    automatic choice for small moves."""
    import itertools

    from lmpool_b200 import _capi
    from lmpool_b200 import kv_transfer as kt
    from lmpool_b200.layout import affine_layout

    g = dict(LOCAL)
    g["N"] = args.cache_blocks or 256
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cache = torch.empty((2, g["L"], g["N"], g["bs"], g["H"], g["D"]), dtype=torch.bfloat16, device=dev)
    cache.normal_(generator=torch.Generator(device=dev).manual_seed(0))
    lay = affine_layout(cache, g["L"])
    perm = seeded_perm(g["N"], 0)
    stream = torch.cuda.current_stream(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = L2Flush(dev)
    peak, _ = hbm_peak()
    lib = _capi.lib()
    old = _capi.Tuning()
    lib.kvx_get_tuning(_capi.ctypes.byref(old))
    grid = [(0, 0, 0, 0)]
    for stages, tile, cps in itertools.product([4, 6, 8], [8192, 16384, 32768], [0, 1, 2, 4]):
        grid.append((2, cps, tile, stages))
    grid += [(1, cps, tile, 0) for cps in (2, 4, 8) for tile in (16384, 32768)]
    out = {}
    try:
        for b in (1, 4, 16, 64):
            s_t = torch.tensor(perm[:b], dtype=torch.int64, device=dev)
            d_t = torch.tensor(perm[b:2 * b], dtype=torch.int64, device=dev)
            pb = payload_bytes(g, b)
            rows = []
            for variant, cps, tile, stages in grid:
                _capi.check(lib.kvx_set_tuning(_capi.ctypes.byref(_capi.Tuning(variant, cps, tile, stages))),
                            "kvx_set_tuning")
                for _ in range(3):
                    kt._launch_move(0, lay, lay, s_t, d_t, b, status, stream)
                times = []
                for _ in range(20):
                    flush()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    kt._launch_move(0, lay, lay, s_t, d_t, b, status, stream)
                    e1.record(stream)
                    e1.synchronize()
                    times.append(e0.elapsed_time(e1))
                us = statistics.median(times) * 1e3
                rows.append({"variant": {0: "auto", 1: "register", 2: "bulk"}[variant], "ctas_per_sm": cps,
                             "tile": tile, "stages": stages, "us": us,
                             "frac_hbm": 2 * pb / (us * 1e-6) / 1e9 / peak,
                             "verified_bitexact": verify_local(cache, perm[:b], perm[b:2 * b])["chunks_mismatched"] == 0})
            out[str(b)] = {"automatic": rows[0], "best": min(rows, key=lambda r: r["us"]), "rows": rows}
    finally:
        lib.kvx_set_tuning(_capi.ctypes.byref(old))
    if int(status.item()):
        raise RuntimeError(f"kernel status {int(status.item())}")
    return {"workload": "local move tuning sweep, config 2 geometry, small B, L2 flushed before each launch",
            "cache_blocks": g["N"], "results": out,
            "verified_bitexact": all(r["verified_bitexact"] for v in out.values() for r in v["rows"])}


def bench_pair_tuning(args) -> dict:
    """``--workload pairtune``: the pair transfer at Qwen3-8B geometry on
    cuda:0 and cuda:1 in one process, over a grid of launch settings (bulk
    ring stages x tile x CTAs per SM, and the register engine), for push and
    pull one way and both ways at once; plus plain peer copies (copy engine,
    cudaMemcpyAsync on a chosen device's stream) over the same link. Every
    wait is satisfied by a launch issued before it (one process, dependency
    order). Measurement sweep behind the kernel's automatic choice."""
    import itertools

    from cuda.bindings import runtime as rt

    from lmpool_b200 import _capi
    from lmpool_b200.endpoint import TransferEndpoint
    from lmpool_b200.layout import affine_layout

    if torch.cuda.device_count() < 2:
        raise SystemExit("pairtune needs 2 GPUs")
    g = dict(PAIRS)
    B = args.blocks or 64
    N = max(320, 4 * B + 8)
    caches, eps = [], []
    for d in (0, 1):
        t = torch.empty((2, g["L"], N, g["bs"], g["H"], g["D"]), dtype=torch.bfloat16, device=f"cuda:{d}")
        t.normal_(generator=torch.Generator(device=f"cuda:{d}").manual_seed(d))
        caches.append(t)
        ep = TransferEndpoint(d, 2, d, N)
        ep.set_cache(affine_layout(t, g["L"]), t)
        eps.append(ep)
    links = {(0, 1): eps[0].link(eps[1].export_record()), (1, 0): eps[1].link(eps[0].export_record())}
    perm = seeded_perm(N, 3)
    src = {0: torch.tensor(perm[:B], device="cuda:0"), 1: torch.tensor(perm[B:2 * B], device="cuda:1")}
    dst = {1: torch.tensor(perm[2 * B:3 * B], device="cuda:1"), 0: torch.tensor(perm[3 * B:4 * B], device="cuda:0")}
    src_on = {1: src[0].to("cuda:1"), 0: src[1].to("cuda:0")}      # the source ids where the puller holds them
    s = {0: torch.cuda.Stream(0), 1: torch.cuda.Stream(1)}
    P = payload_bytes(g, B)

    def push(pairs):
        tokens = {(a, b): eps[b].next_token(a) for a, b in pairs}
        for a, b in pairs:
            eps[b].publish(links[(b, a)], dst[b], B, tokens[(a, b)], s[b])
        for a, b in pairs:
            eps[a].wait_armed(links[(a, b)], B, 30.0, s[a])
        for a, b in pairs:
            eps[a].push(eps[a].cache, [(links[(a, b)], links[(a, b)].cache, src[a], B)], s[a])
        for a, b in pairs:
            eps[b].wait_done(a, tokens[(a, b)], 30.0, s[b])

    def pull(pairs):
        tokens = {(a, b): eps[b].next_token(a) for a, b in pairs}
        for a, b in pairs:
            eps[b].request(links[(b, a)], B, tokens[(a, b)], s[b])
        for a, b in pairs:
            eps[a].grant(links[(a, b)], B, 30.0, s[a])
        for a, b in pairs:
            eps[b].wait_done(a, tokens[(a, b)], 30.0, s[b])
            eps[b].pull(eps[b].cache, [(links[(b, a)], links[(b, a)].cache, src_on[b], dst[b], B, tokens[(a, b)])],
                        s[b])
        for a, b in pairs:
            eps[a].wait_pulled(b, 30.0, s[a])

    def timed(fn, reps=10) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        ev = {d: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for d in (0, 1)}
        for d in (0, 1):
            with torch.cuda.device(d):
                ev[d][0].record(s[d])
        for _ in range(reps):
            fn()
        for d in (0, 1):
            with torch.cuda.device(d):
                ev[d][1].record(s[d])
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        return max(ev[d][0].elapsed_time(ev[d][1]) for d in (0, 1)) / reps

    lib = _capi.lib()
    old = _capi.Tuning()
    lib.kvx_get_tuning(_capi.ctypes.byref(old))
    grid = [(0, 0, 0, 0)]
    for stages, tile, cps in itertools.product([4, 6, 8, 12], [8192, 16384, 32768, 65536], [0, 1, 2, 4]):
        if 1024 + stages * tile <= 227 * 1024:
            grid.append((2, cps, tile, stages))
    grid += [(1, cps, tile, 0) for cps in (2, 4, 8) for tile in (16384, 32768, 65536)]
    rows = []
    try:
        for variant, cps, tile, stages in grid:
            _capi.check(lib.kvx_set_tuning(_capi.ctypes.byref(_capi.Tuning(variant, cps, tile, stages))),
                        "kvx_set_tuning")
            row = {"variant": {0: "auto", 1: "register", 2: "bulk"}[variant], "ctas_per_sm": cps, "tile": tile,
                   "stages": stages}
            for name, fn in (("push", lambda: push([(0, 1)])), ("pull", lambda: pull([(0, 1)])),
                             ("push_both", lambda: push([(0, 1), (1, 0)])),
                             ("pull_both", lambda: pull([(0, 1), (1, 0)]))):
                row[name] = P / (timed(fn) * 1e-3) / 1e9
            for d in (0, 1):
                eps[d].check_status(s[d], "pairtune")
            rows.append(row)
    finally:
        lib.kvx_set_tuning(_capi.ctypes.byref(old))
    ok = torch.equal(caches[1][:, :, perm[2 * B:3 * B]].cpu().view(torch.int16),
                     caches[0][:, :, perm[:B]].cpu().view(torch.int16)) and \
        torch.equal(caches[0][:, :, perm[3 * B:4 * B]].cpu().view(torch.int16),
                    caches[1][:, :, perm[B:2 * B]].cpu().view(torch.int16))
    nbytes = 2 << 30
    bufs = {d: (torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{d}"),
                torch.empty(nbytes, dtype=torch.uint8, device=f"cuda:{d}")) for d in (0, 1)}

    def cp(dst_t, src_t, dev):
        err, = rt.cudaMemcpyAsync(dst_t.data_ptr(), src_t.data_ptr(), nbytes,
                                  rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice, s[dev].cuda_stream)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaMemcpyAsync: {err}")

    copies = {
        "read_by_1_GB/s": nbytes / (timed(lambda: cp(bufs[1][0], bufs[0][0], 1), 5) * 1e-3) / 1e9,
        "write_by_0_GB/s": nbytes / (timed(lambda: cp(bufs[1][0], bufs[0][0], 0), 5) * 1e-3) / 1e9,
        "both_ways_read_GB/s_per_direction": nbytes / (timed(
            lambda: (cp(bufs[1][0], bufs[0][0], 1), cp(bufs[0][1], bufs[1][1], 0)), 5) * 1e-3) / 1e9,
    }
    for ep in eps:
        ep.close_links()
    for ep in eps:
        ep.close()
    best = {k: max(rows, key=lambda r: r[k]) for k in ("push", "pull", "push_both", "pull_both")}
    return {"workload": f"pair tuning sweep, cuda:0 <-> cuda:1, one process, Qwen3-8B geometry, B={B}",
            "blocks": B, "cache_blocks": N, "unit": "GB/s per direction", "verified": bool(ok),
            "automatic": rows[0], "best": best, "peer_copy": copies, "rows": rows}


def bench_config5(args) -> dict | None:
    """``--workload config5``: config 5 alone on N GPUs (pairs)."""
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world < 2 or world % 2:
        raise SystemExit("config 5 needs an even number of GPUs >= 2")
    torch.cuda.set_device(local)
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    mode = "push" if args.pair_mode == "auto" else args.pair_mode   # both directions at once
    res = config5_leg(kt, rank, world, dist, args.steps, mode)
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    if not res["verified_bitexact"]:
        raise RuntimeError("config 5 verification failed")
    return dict(res, metric=METRIC, n_gpus=world, unit="GB/s")


def reference_arm(args, rank: int) -> None:
    """``--impl reference``: the reference's CPU path on this host's cores, on
    the same workload, metric and config as the B200 arm (rank 0 only)."""
    if rank != 0:
        return
    world = max(1, args.gpus)
    g = LOCAL if world <= 1 else PAIRS
    if world <= 1:
        res = cpu_baseline_local(g, CPU_SAMPLE_BLOCKS, seconds=min(20.0, 2.0 * max(1, args.steps)))
        note = ("pack + unpack with the reference's torch ops in one process (the 1-GPU workload is a local move; "
                "no transport between pack and unpack)")
    else:
        res = cpu_baseline_gloo(g, CPU_SAMPLE_BLOCKS, both_ways=True, seconds=min(20.0, 2.0 * max(1, args.steps)))
        note = "one pair over gloo on the host cores, both directions (more pairs would share the same cores)"
    line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": "GB/s", "n_gpus": args.gpus,
            "steps": res["steps"], "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic bf16 N(0,1) KV caches, seeded randperm block ids",
            "config": line_config(g, world),
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "cpu_baseline_host": res["host"], "note": note,
            "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--variant", choices=["auto", "register", "bulk"], default="auto")
    ap.add_argument("--cache-blocks", type=int, default=0,
                    help="1-GPU cache size in blocks (default: config 2's 2048); for small profiling cases")
    ap.add_argument("--blocks", type=int, default=0, help="1-GPU blocks moved per step (default 512)")
    ap.add_argument("--workload", choices=["default", "config5", "pair1p", "pairtune", "localtune", "store"],
                    default="default",
                    help="config5: benchmark config 5 transfer + store_kvcache overlap (N >= 2 GPUs); "
                         "pair1p: one process, two GPUs, pair push (profiling); pairtune: one process, two "
                         "GPUs, launch-setting sweep of push and pull plus plain peer copies; localtune: the same for "
                         "small 1-GPU moves; store: "
                         "store_kvcache only")
    ap.add_argument("--pull", action="store_true", help="pair1p: destination pulls instead of source pushing")
    ap.add_argument("--pair-mode", choices=["auto", "push", "pull"], default="auto",
                    help="N>1 exchanges that send both ways at once (phase A, config 5): auto = push")
    ap.add_argument("--store-pdl", choices=["auto", "on", "off"], default="auto",
                    help="store_kvcache launch with programmatic dependent launch (auto = on)")
    ap.add_argument("--quick", action="store_true",
                    help="1 GPU: time the headline loop only (no sweep, e2e or CPU baseline); for profiling")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        reference_arm(args, rank)
        return

    from lmpool_b200 import _capi

    if args.variant != "auto" or args.store_pdl != "auto":
        t = _capi.Tuning(variant={"auto": 0, "register": 1, "bulk": 2}[args.variant],
                         store_pdl={"auto": 0, "on": 1, "off": 2}[args.store_pdl])
        _capi.check(_capi.lib().kvx_set_tuning(_capi.ctypes.byref(t)), "kvx_set_tuning")
    if args.workload == "config5":
        res = bench_config5(args)
    elif args.workload == "pair1p":
        res = bench_pair_one_process(args)
    elif args.workload == "pairtune":
        res = bench_pair_tuning(args)
    elif args.workload == "localtune":
        res = bench_local_tuning(args)
    elif args.workload == "store":
        torch.cuda.set_device(0)
        res = bench_store_kvcache(0, hbm_peak()[0], iters=max(3, args.steps), num_blocks=args.cache_blocks)
    elif world > 1 or args.gpus > 1:
        res = bench_pairs(args)
    else:
        res = bench_local(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
