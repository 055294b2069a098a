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
             the transfer mode of lmpool_b200.kv_transfer (default pull: each
             rank bulk-loads its partner's blocks over NVLink, then waits for
             the partner's report; push: arm, push, completion wait).
  --impl reference  the reference algorithm on the host cores (C oracle:
             pack into a payload, then unpack; rank 0 only), same geometry.

Timing: W untimed warm-up steps, then K steps between a barrier and a
device synchronisation, CUDA events on the launching stream, max over ranks.
Every step's inputs exceed the 126 MB L2 (config 2: 15 GB read + 15 GB
written per step; config 4: 4.8 GB per direction), so no flush is needed for
the headline; the sweep flushes L2 before each timed launch.
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
SWEEP_B = [1, 4, 16, 64, 256, 512]
NVLINK_PEER_GBS = 770.0     # measured peer copy per direction on this pool (profiling recipe)
FALLBACK_HBM_GBS = 6650.0
CPU_SAMPLE_BLOCKS = 16
L2_FLUSH_BYTES = 512 << 20


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


def profile_traffic(name: str) -> float | None:
    """dram bytes per launch recorded in a committed ncu summary (profiles/<name>.txt)."""
    p = ROOT / "profiles" / f"{name}.txt"
    if not p.exists():
        return None
    m = re.search(r"^dram_bytes_per_launch_full_size:\s*([0-9.eE+]+)", p.read_text(), re.M)
    return float(m.group(1)) if m else None


def seeded_perm(n: int, seed: int) -> list[int]:
    g = torch.Generator().manual_seed(int(seed))
    return torch.randperm(int(n), generator=g).tolist()


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
    out = {"sm_mhz": statistics.median(sms) if sms else None,
           "sm_max_mhz": max((c["sm_max_mhz"] for c in items if c.get("sm_max_mhz")), default=None),
           "reasons": sorted({r for c in items for r in c.get("reasons", [])}),
           "samples": sum(c.get("samples", 0) for c in items)}
    return out


def cpu_reference(g: dict, blocks: int, steps: int, warmup: int, min_seconds: float = 0.0) -> dict:
    """The reference algorithm (pack into a payload, then unpack; kv_transfer.py:229-276)
    on the host cores through the C oracle, on a bounded sample of the workload."""
    from oracle import c_oracle

    threads = c_oracle.default_threads()
    torch.set_num_threads(threads)
    n = 2 * blocks + 64
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


# ---------------------------------------------------------------------------
# 1 GPU: config 2
# ---------------------------------------------------------------------------

STORE = dict(L=80, H=8, D=128, bs=16, N=4096, T=256)


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


def bench_store_kvcache(dev_idx: int, peak: float, iters: int = 30, num_blocks: int = 0) -> dict:
    """store_kvcache at benchmark config 5 geometry (L=80, H=8, D=128,
    block_size=16, T=256 tokens per step, ~10% padding slots; the cache is
    shrunk to 4096 blocks: the cost does not depend on N). A step writes every
    layer: 80 single-layer launches as the model issues them (eager, and
    captured in a CUDA graph as the decode path does), or one all-layer
    launch. L2 is flushed (written, then another buffer read) between timed
    steps."""
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

    per_layer()
    all_layers()
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
    check_device_status(dev_idx)
    row = c["H"] * c["D"] * 2
    traffic = c["L"] * (2 * c["T"] * row + 2 * valid * row + c["T"] * 8)
    del graph, cache, keys, values, flush
    torch.cuda.empty_cache()

    def entry(ms, launches):
        gbs = traffic / (ms * 1e-3) / 1e9
        return {"ms_per_step": ms, "launches_per_step": launches, "GB/s": gbs, "frac_hbm": gbs / peak}

    return {"geometry": dict(c, valid_tokens=valid), "bytes_per_step": traffic,
            "per_layer_eager": entry(ms_eager, c["L"]), "per_layer_graph": entry(ms_graph, c["L"]),
            "all_layers_one_launch": entry(ms_all, 1),
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
    # correctness spot check of the timed workload
    for i in (0, B // 2, B - 1):
        if not torch.equal(cache[:, :, perm[B + i]].view(torch.int16), cache[:, :, perm[i]].view(torch.int16)):
            raise RuntimeError("moved block differs from its source")

    value = P / (ms * 1e-3) / 1e9
    peak, peak_src = hbm_peak()
    achieved = 2 * P / (ms * 1e-3) / 1e9
    traffic = profile_traffic("move_local_config2")
    if args.quick:
        print(json.dumps({"quick": True, "blocks": B, "cache_blocks": g["N"], "ms_per_step": ms, "GB/s": value,
                          "hbm_GB/s": achieved, "frac": achieved / peak}), flush=True)
        return None

    # B sweep, L2 flushed before each timed launch (clean, and write-only)
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
        sweep.append({"blocks": b, "bytes": pb, "ms": t * 1e3, "GB/s": pb / t / 1e9,
                      "hbm_GB/s": 2 * pb / t / 1e9, "frac_hbm": 2 * pb / t / 1e9 / peak,
                      "ms_dirty_l2": med[True] * 1e3, "frac_hbm_dirty_l2": 2 * pb / med[True] / 1e9 / peak})
    del flush

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
    cpu = cpu_reference(g, CPU_SAMPLE_BLOCKS, steps=3, warmup=1, min_seconds=10.0)
    return {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: bf16 N(0,1) KV cache (device generator seed 0), block ids from randperm(2048, seed 0)",
        "config": {"workload": g["workload"], "num_layers": g["L"], "num_blocks": g["N"], "block_size": g["bs"],
                   "num_kv_heads": g["H"], "head_dim": g["D"], "blocks_moved": B, "payload_bytes_per_step": P,
                   "src_ids": "randperm[:512]", "dst_ids": "randperm[512:1024]",
                   "l2": "inputs larger than L2 (15 GB read + 15 GB written per step); the sweep flushes L2 "
                         "before each launch by writing 512 MB then reading 512 MB (ms_dirty_l2: write only)",
                   "parallelism": "replicas only"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_source": peak_src,
                     "algorithmic_bytes_per_launch": 2 * P, "kernel_ms": ms},
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": P / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 2 * B * 8, "d2h_bytes_per_step": 4,
                "api": "lmpool_b200.kv_transfer.move_blocks(host id lists, synchronize=True)"},
        "gpu_launches": args.steps,
        "clocks": clk,
        "sweep": sweep,
        "reference_gpu_path": ref_gpu,
        "store_kvcache": store,
        "kernel": {"variant": {0: "auto", 1: "register", 2: "bulk"}[tune.variant], "launches_per_step": 1},
    }


# ---------------------------------------------------------------------------
# N GPUs: config 4 phase A
# ---------------------------------------------------------------------------

def block_sums(cache: torch.Tensor, ids: list[int]) -> torch.Tensor:
    """Per (plane, layer, block) sum of the bf16 bit patterns of the listed
    blocks, int64, one (plane, layer) slice at a time (bounded temporaries)."""
    idx = torch.tensor(ids, dtype=torch.int64, device=cache.device)
    out = torch.empty(2, cache.shape[1], len(ids), dtype=torch.int64, device=cache.device)
    for kv in range(2):
        for layer in range(cache.shape[1]):
            sel = cache[kv, layer].index_select(0, idx).view(torch.int16).reshape(len(ids), -1)
            out[kv, layer] = sel.sum(-1, dtype=torch.int64)
    return out.cpu()


def pair_sweep(ep, link, g: dict, rank: int, stream, dist, mode: str) -> list[dict]:
    """benchmark config 3 on ranks 0 -> 1: B in {1, 8, 64, 256}, contiguous and
    scattered source ids. Each timed run is K back-to-back transfers in the
    configured mode, cycling through disjoint id sets so no transfer re-reads
    blocks still in L2; time = max over the two ranks."""
    dev = torch.device("cuda", ep.device)
    N = g["N"]
    out = []
    for B in (1, 8, 64, 256):
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

            def one(k):
                if rank == 1:
                    ep.exchange(mode, ep.cache, [], [(0, src_t[k % nsets], dst_t[k % nsets], B)], 60.0, stream)
                else:
                    ep.exchange(mode, ep.cache, [(1, src_t[k % nsets], B)], [], 60.0, stream)

            for k in range(3):
                one(k)
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for k in range(K):
                one(k)
            e1.record(stream)
            torch.cuda.synchronize()
            t = torch.tensor([e0.elapsed_time(e1) / K], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            pb = payload_bytes(g, B)
            out.append({"mode": mode, "blocks": B, "ids": ids_kind, "bytes": pb, "ms": ms,
                        "GB/s": pb / (ms * 1e-3) / 1e9,
                        "frac_nvlink": pb / (ms * 1e-3) / 1e9 / NVLINK_PEER_GBS})
    return out


def reference_gpu_pair(cache: torch.Tensor, g: dict, rank: int, dist, blocks=(1, 8, 64, 256)) -> dict:
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
        # the same transfers back to back, timed on the device like pair_sweep
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(iters):
            one()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([statistics.mean(times), e0.elapsed_time(e1) / iters], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_wall, ms_dev = float(t[0].item()), float(t[1].item())
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

    # the kernel legs just wrote these blocks from the same sources
    before = {s: block_sums(cache, v) for s, v in incoming.items()}
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
    same = all(torch.equal(before[s], block_sums(cache, v)) for s, v in incoming.items())
    agree = [None] * world
    dist.all_gather_object(agree, same)
    del send, recv
    torch.cuda.empty_cache()
    pb = payload_bytes(g, B)
    per_gpu_out = (world - 1) * pb / (ms * 1e-3) / 1e9
    return {"algorithm": "index_select pack -> NCCL batched send/recv -> index_copy_ unpack",
            "blocks_per_destination": B, "ms_per_step": ms,
            "value": world * (world - 1) * pb / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "per_gpu_egress_GB/s": per_gpu_out, "same_blocks_as_kernel": all(agree)}


def all_partner(ep, cache, g: dict, rank: int, world: int, stream, dist, mode: str,
                schedule: str = "concurrent") -> dict:
    """benchmark config 4 phase B: every rank sends B=32 seeded-random blocks to
    every other rank, into disjoint reserved sets.

    ``concurrent``: one exchange per step carries every destination and
    source at once (one push or pull launch per rank). ``rotated``: world-1
    exchanges per step; in exchange j rank r sends to r+j and receives from
    r-j, so at any moment every GPU has one sender and one receiver, the
    traffic pattern of disjoint pairs."""
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
    for _ in range(3):
        step()
    K = 10
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(K):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / K], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    mine = {"rank": rank, "bits": int(ep.status.item()),
            "out": {d: block_sums(cache, v) for d, v in outgoing.items()},
            "in": {s: block_sums(cache, v) for s, v in incoming.items()}}
    gathered: list = [None] * world
    dist.all_gather_object(gathered, mine)
    ok = all(x["bits"] == 0 for x in gathered)
    for x in gathered:
        for d, sums in x["out"].items():
            ok &= torch.equal(sums, gathered[d]["in"][x["rank"]])
    pb = payload_bytes(g, B)
    per_gpu_out = (world - 1) * pb / (ms * 1e-3) / 1e9
    return {"ok": bool(ok), "schedule": schedule, "blocks_per_destination": B, "ms_per_step": ms,
            "value": world * (world - 1) * pb / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "per_gpu_egress_GB/s": per_gpu_out, "frac_nvlink_per_gpu_egress": per_gpu_out / NVLINK_PEER_GBS,
            "verified": bool(ok)}


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
    link = ep.get_link(partner)
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
    # correctness: checksums of what this rank sent vs what its partner holds
    sums_src = block_sums(cache, src_ids)
    sums_dst = block_sums(cache, dst_ids)
    gathered: list = [None] * world
    dist.all_gather_object(gathered, {"rank": rank, "src": sums_src, "dst": sums_dst, "bits": bits, "clk": clk})
    ok = all(item["bits"] == 0 for item in gathered)
    ok &= torch.equal(gathered[partner]["src"], sums_dst)

    # the same exchange in the other mode, for the record
    for _ in range(3):
        step(other)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(10):
        step(other)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / 10], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    other_ms = float(t.item())

    sweep = None
    if world == 2:   # one direction at a time: both modes, pull is the default of swap_in
        sweep = pair_sweep(ep, link, g, rank, stream, dist, "pull") + pair_sweep(ep, link, g, rank, stream, dist,
                                                                               "push")
    ref_pair = reference_gpu_pair(cache, g, rank, dist) if world == 2 else None
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
                phase_b[key] = all_partner(ep, cache, g, rank, world, stream, dist, m, sched)
        ok &= all(v["ok"] for v in phase_b.values())
        phase_b["reference_nccl"] = reference_all_partner(cache, g, rank, world, dist)

    # end to end: host id lists through swap_batch (pinned H2D + status D2H per step)
    e2e_steps = max(3, min(args.steps, 30))
    for _ in range(2):
        kt.swap_batch([(partner, src_ids)], [(partner, partner_src, dst_ids)], mode=mode)
    dist.barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(stream)
    for _ in range(e2e_steps):
        kt.swap_batch([(partner, src_ids)], [(partner, partner_src, dst_ids)], mode=mode)
    e3.record(stream)
    torch.cuda.synchronize()
    t2 = torch.tensor([e2.elapsed_time(e3) / e2e_steps], dtype=torch.float64, device=dev)
    dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_ms = float(t2.item())
    oks = [None] * world
    dist.all_gather_object(oks, bool(ok))
    kt.shutdown()
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    if not all(oks):
        raise RuntimeError("pair transfer verification failed")
    value = world * P / (ms * 1e-3) / 1e9
    per_dir = P / (ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic: bf16 N(0,1) KV caches (device generator seed = rank), seeded randperm ids",
        "config": {"workload": g["workload"], "num_layers": g["L"], "num_blocks": g["N"], "block_size": g["bs"],
                   "num_kv_heads": g["H"], "head_dim": g["D"], "blocks_moved_per_direction": B,
                   "payload_bytes_per_rank_per_step": P, "pairs": pairs,
                   "l2": "inputs larger than L2 (4.8 GB per direction per step)",
                   "parallelism": f"{world // 2} NVLink pairs, push over CUDA IPC"},
        "roofline": {"bound": "nvlink", "achieved": per_dir, "peak": NVLINK_PEER_GBS, "unit": "GB/s",
                     "frac": per_dir / NVLINK_PEER_GBS, "traffic": None,
                     "peak_source": "peer copy per direction measured on this pool (profiling recipe); 900 nominal"},
        "e2e": {"value": world * P / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": 2 * B * 8, "d2h_bytes_per_step": 4,
                "api": "lmpool_b200.kv_transfer.swap_batch(host id lists)"},
        "gpu_launches": (4 if mode == "push" else 2) * args.steps,
        "transfer_mode": mode,
        "other_mode": {"mode": other, "ms_per_step": other_ms,
                       "GB/s_per_direction": P / (other_ms * 1e-3) / 1e9},
        "clocks": merge_clocks([item["clk"] for item in gathered]),
        "pair_sweep": sweep,
        "reference_gpu_path": ref_pair,
        "phase_b": ({m: {k: v for k, v in r.items() if k != "ok"} for m, r in phase_b.items()} if phase_b else None),
    }


def bench_pair_one_process(args) -> dict:
    """One process drives cuda:0 (source) and cuda:1 (destination): the pair
    protocol at Qwen3-8B geometry with launches enqueued in dependency order
    (publish on 1, wait_armed + push on 0, wait_done on 1), so every bounded
    wait is satisfied by a launch issued before it. Used for profiling the
    NVLink push with one process, and as a quick pair number."""
    from lmpool_b200 import kv_transfer as kt
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
    pull_status = torch.zeros(1, dtype=torch.int32, device="cuda:1")

    def one():
        if args.pull:
            # destination-driven: cuda:1 bulk-loads the source blocks from
            # cuda:0's cache over NVLink and stores them locally
            kt._launch_move(1, l10.cache, eps[1].cache, src_on_1, dst_t, B, pull_status, s1)
            return
        token = eps[1].next_token(0)
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
    if int(pull_status.item()):
        raise RuntimeError(f"pull reported status {int(pull_status.item())}")
    ok = all(torch.equal(caches[1][:, :, perm[B + i]].cpu().view(torch.int16),
                         caches[0][:, :, perm[i]].cpu().view(torch.int16)) for i in (0, B - 1))
    for ep in eps:
        ep.close_links()
    for ep in eps:
        ep.close()
    P = payload_bytes(g, B)
    return {"workload": "pair, one process, cuda:0 -> cuda:1, " + ("pull by cuda:1" if args.pull else "push by cuda:0"),
            "blocks": B, "cache_blocks": N, "ms_per_step": ms,
            "GB/s": P / (ms * 1e-3) / 1e9, "frac_nvlink": P / (ms * 1e-3) / 1e9 / NVLINK_PEER_GBS, "verified": ok}


CONFIG5 = dict(workload="config5: 70B-like transfer (B=1024 to the NVLink partner, both directions) under "
                        "concurrent store_kvcache (T=256 tokens x 80 layers per step)",
               L=80, N=16384, bs=16, H=8, D=128, B=1024, T=256)


def bench_config5(args) -> dict | None:
    """benchmark config 5 on N GPUs (pairs): the transfer alone, store_kvcache
    alone, and both at once on two streams. The cache is shrunk from 65536 to
    16384 blocks per rank (80 GiB; 65536 would be 320 GiB): transfer and store
    costs depend on B and T, not on N."""
    import torch.distributed as dist

    from lmpool_b200 import kv_transfer as kt
    from lmpool_b200.attention import store_kvcache, store_kvcache_layers

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", rank))
    if world < 2 or world % 2:
        raise SystemExit("config 5 needs an even number of GPUs >= 2")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta

    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    c = CONFIG5
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
    link = ep.get_link(partner)
    xs = torch.cuda.Stream(dev)
    ss = torch.cuda.Stream(dev)
    src_t = torch.tensor(src_ids, dtype=torch.int64, device=dev)
    dst_t = torch.tensor(dst_ids, dtype=torch.int64, device=dev)
    P = B * c["L"] * 2 * c["bs"] * c["H"] * c["D"] * 2
    row = c["H"] * c["D"] * 2
    valid = int((slots >= 0).sum())
    store_bytes = c["L"] * (2 * c["T"] * row + 2 * valid * row + c["T"] * 8)

    psrc_t = torch.tensor(seeded_perm(c["N"], 7000 + partner)[:B], dtype=torch.int64, device=dev)

    mode = "push" if args.pair_mode == "auto" else args.pair_mode   # both directions at once

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

    def timed_alone(fn, stream, reps) -> float:
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

    K = max(3, min(args.steps, 10))
    x_ms = timed_alone(xfer, xs, K)
    s_ms = timed_alone(store_step, ss, 200)
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
    oks: list = [None] * world
    dist.all_gather_object(oks, bits == 0)
    kt.check_device_status(local)
    kt.shutdown()
    dist.barrier()
    dist.destroy_process_group()
    if rank != 0:
        return None
    if not all(oks):
        raise RuntimeError("config 5 transfer reported a device error")
    return {
        "metric": METRIC, "workload": c["workload"], "n_gpus": world, "unit": "GB/s",
        "config": {k: c[k] for k in ("L", "N", "bs", "H", "D", "B", "T")},
        "substitution": "num_blocks 65536 -> 16384 per rank (320 GiB does not fit one B200)",
        "transfer_alone": {"ms": x_ms, "GB/s_per_direction": P / (x_ms * 1e-3) / 1e9,
                           "frac_nvlink": P / (x_ms * 1e-3) / 1e9 / NVLINK_PEER_GBS},
        "store_alone": {"ms_per_step": s_ms, "GB/s": store_bytes / (s_ms * 1e-3) / 1e9,
                        "launch": "all 80 layers in one launch"},
        "overlapped": {"transfers": K, "store_steps": M, "transfer_ms": xo_ms,
                       "transfer_GB/s_per_direction": P / (xo_ms * 1e-3) / 1e9,
                       "store_ms_per_step": so_ms, "store_GB/s": store_bytes / (so_ms * 1e-3) / 1e9},
        "payload_bytes_per_direction": P, "store_bytes_per_step": store_bytes, "transfer_mode": mode,
    }


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
    ap.add_argument("--workload", choices=["default", "config5", "pair1p", "store"], default="default",
                    help="config5: benchmark config 5 transfer + store_kvcache overlap (N >= 2 GPUs); "
                         "pair1p: one process, two GPUs, pair push (profiling); store: store_kvcache only")
    ap.add_argument("--pull", action="store_true", help="pair1p: destination pulls instead of source pushing")
    ap.add_argument("--pair-mode", choices=["auto", "push", "pull"], default="auto",
                    help="N>1 exchanges that send both ways at once (phase A, config 5): auto = push")
    ap.add_argument("--quick", action="store_true",
                    help="1 GPU: time the headline loop only (no sweep, e2e or CPU baseline); for profiling")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        g = LOCAL if args.gpus <= 1 else PAIRS
        res = cpu_reference(g, CPU_SAMPLE_BLOCKS, steps=args.steps, warmup=args.warmup)
        line = {"impl": "reference", "metric": METRIC, "value": res["value"], "unit": "GB/s", "n_gpus": args.gpus,
                "steps": res["steps"], "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic bf16 KV cache, seeded randperm block ids",
                "config": {"workload": g["workload"], "num_layers": g["L"], "block_size": g["bs"],
                           "num_kv_heads": g["H"], "head_dim": g["D"], "blocks_per_step": CPU_SAMPLE_BLOCKS},
                "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": res["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    from lmpool_b200 import _capi

    if args.variant != "auto":
        t = _capi.Tuning(variant={"register": 1, "bulk": 2}[args.variant])
        _capi.check(_capi.lib().kvx_set_tuning(_capi.ctypes.byref(t)), "kvx_set_tuning")
    if args.workload == "config5":
        res = bench_config5(args)
    elif args.workload == "pair1p":
        res = bench_pair_one_process(args)
    elif args.workload == "store":
        torch.cuda.set_device(0)
        res = bench_store_kvcache(0, hbm_peak()[0], num_blocks=args.cache_blocks)
    elif world > 1 or args.gpus > 1:
        res = bench_pairs(args)
    else:
        res = bench_local(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
