"""Pin the torch+gloo restatement of the reference's CPU path (oracle/torch_ref.py).

It is the bench's timed CPU baseline, so it must produce the reference's own
outputs: the pack/unpack fixtures and the two-rank gloo ``swap_in`` run that
tests/golden/make_golden.py recorded from LMPool's code.
"""
import os
import socket
import time
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import torch_ref

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def pu():
    return np.load(GOLDEN / "pack_unpack.npz")


@pytest.mark.parametrize("case", ["c", "d", "e"])
def test_pack_unpack_match_reference_fixtures(pu, case):
    src = torch.from_numpy(pu[f"{case}_src"].copy())
    dst = torch.from_numpy(pu[f"{case}_dst_before"].copy())
    payload = torch_ref.pack_all_layer_blocks(src, src.shape[1], pu[f"{case}_src_ids"].tolist())
    assert torch.equal(payload, torch.from_numpy(pu[f"{case}_payload"]))
    torch_ref.unpack_all_layer_blocks(payload, dst, pu[f"{case}_dst_ids"].tolist())
    assert torch.equal(dst, torch.from_numpy(pu[f"{case}_dst_after"]))


def test_unpack_refuses_a_count_mismatch_like_the_reference():
    cache = torch.zeros(2, 1, 4, 2, 1, 1)
    with pytest.raises(RuntimeError, match="does not match destination blocks"):
        torch_ref.unpack_all_layer_blocks(torch.ones(1, 2, 2, 2, 1, 1), cache, [1])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _swap_worker(rank, port, q):
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        z = np.load(GOLDEN / "swap_small.npz")
        cache = torch.from_numpy(z[f"rank{rank}_before"].copy())
        got = torch_ref.swap_planned(rank, 0, 1, cache, z["src_ids"].tolist(), z["dst_ids"].tolist())
        q.put({"rank": rank, "same": bool(torch.equal(cache, torch.from_numpy(z[f"rank{rank}_after"]))),
               "returned": got, "expected": z[f"returned{rank}"].tolist()})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put({"rank": rank, "error": repr(exc)})


def test_gloo_swap_reproduces_the_reference_two_rank_run():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_swap_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + 120
    while len(out) < 2 and time.time() < deadline:
        try:
            item = q.get(timeout=1)
            out[item["rank"]] = item
        except Exception:  # noqa: BLE001 - queue.Empty
            if all(p.exitcode is not None for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
    assert len(out) == 2, out
    for r in (0, 1):
        assert "error" not in out[r], out[r]
        assert out[r]["same"] and out[r]["returned"] == out[r]["expected"]


def test_timed_baselines_run_and_verify_on_a_tiny_geometry():
    geom = {"L": 2, "bs": 4, "H": 2, "D": 8}
    local = torch_ref.time_local(geom, 3, min_seconds=0.0, min_steps=2)
    assert local["verified"] and local["steps"] >= 2 and local["bytes_per_step"] == 3 * 2 * 2 * 4 * 2 * 8 * 2
    pair = torch_ref.time_gloo_pair(geom, 3, both_ways=True, min_seconds=0.0, min_steps=2, timeout_s=120)
    assert pair["verified"] and pair["steps"] >= 2 and pair["bytes_per_step"] == 2 * local["bytes_per_step"]
    assert pair["host"]["usable_cores"] >= 1
