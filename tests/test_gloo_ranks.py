"""World-size-2 gloo tests (CPU) of the multi-rank host logic.

What runs on the host around the NVLink push: the legacy id negotiation
messages (kv_transfer.py:283-303), swap_in's argument/count checks on both
ranks (kv_transfer.py:429-458), peer-record exchange, and failure on a rank
that dies mid-protocol (the survivor's receive ends with an error after the
process-group timeout, which the data plane turns into executor_error).
"""
import os
import socket
import time
from datetime import timedelta

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(target, timeout=120, extra=()):
    ctx = mp.get_context("spawn")
    port = _free_port()
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, port, q, *extra)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + timeout
    while len(out) < 2 and time.time() < deadline:
        try:
            item = q.get(timeout=1)
            out[item["rank"]] = item
        except Exception:  # noqa: BLE001 - queue.Empty
            if all(p.exitcode is not None for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.terminate()
            p.join(timeout=10)
    return out


def _init(rank, port, seconds=60):
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", world_size=2, rank=rank,
                            timeout=timedelta(seconds=seconds))
    return dist


def _negotiation_worker(rank, port, q):
    try:
        dist = _init(rank, port)
        from lmpool_b200 import kv_transfer as kt

        # legacy swap_in negotiation, message for message (kv_transfer.py:438-450)
        if rank == 1:   # local (destination) side
            kt._send_block_list([5, 6, 7], dst=0)
            kt._send_block_list([1, 2, 3], dst=0)
            got = kt._recv_block_list(src=0)
        else:           # remote (source) side
            remote = kt._recv_block_list(src=1)
            specified = kt._recv_block_list(src=1)
            got = specified if specified else remote
            kt._send_block_list(got, dst=1)
        empty_ok = True
        if rank == 0:
            kt._send_block_list([], dst=1)
        else:
            empty_ok = kt._recv_block_list(src=0) == []
        q.put({"rank": rank, "got": got, "empty_ok": empty_ok})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put({"rank": rank, "error": repr(exc)})


def test_negotiation_messages_over_gloo():
    out = _run(_negotiation_worker)
    assert out[0]["got"] == [1, 2, 3] and out[1]["got"] == [1, 2, 3]
    assert out[0]["empty_ok"] and out[1]["empty_ok"]


def _swap_errors_worker(rank, port, q):
    import torch

    try:
        dist = _init(rank, port)
        from lmpool_b200 import kv_transfer as kt

        cache = torch.zeros(2, 1, 4, 2, 1, 8)
        errors = []

        def expect(fn, text):
            try:
                fn()
                errors.append(f"no error for {text}")
            except RuntimeError as exc:
                if text not in str(exc):
                    errors.append(f"{text!r} not in {exc!r}")

        kw = dict(kv_cache=cache, num_layers=1, block_size=2, num_kv_heads=1, head_dim=8)
        # destination of a planned transfer without reserved ids
        if rank == 1:
            expect(lambda: kt.swap_in(0, [0, 1], 1, negotiate_blocks=False, **kw),
                   "planned transfer requires local_target_blocks")
            expect(lambda: kt.swap_in(0, [0, 1], 1, local_target_blocks=[2], negotiate_blocks=False, **kw),
                   "mismatched block counts")
        dist.barrier()
        # both sides pass their checks but no pair was set up: refused before any GPU work
        expect(lambda: kt.swap_in(0, [0, 1], 1, local_target_blocks=[2, 3] if rank == 1 else None,
                                  negotiate_blocks=False, **kw), "prewarm_p2p_pairs has not run")
        dist.barrier()
        # legacy negotiated path: ids agreed over gloo, then the same refusal
        expect(lambda: kt.swap_in(0, [0, 1], 1, local_target_blocks=[3, 2] if rank == 1 else None,
                                  negotiate_blocks=True, **kw), "prewarm_p2p_pairs has not run")
        dist.barrier()
        # rank that is neither source nor destination of a self-transfer: no-op, ids echoed
        same = kt.swap_in(rank, [1, 2], rank, negotiate_blocks=False, **kw)
        if same != [1, 2]:
            errors.append(f"self transfer returned {same}")
        q.put({"rank": rank, "errors": errors})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put({"rank": rank, "errors": [repr(exc)]})


def test_swap_in_host_checks_on_both_ranks():
    out = _run(_swap_errors_worker)
    assert out[0]["errors"] == [] and out[1]["errors"] == [], out


def _record_worker(rank, port, q):
    try:
        dist = _init(rank, port)
        from lmpool_b200.endpoint import PeerRecord

        rec = PeerRecord(rank=rank, pid=os.getpid(), hostname="h", device=rank, mailbox_handle=bytes([rank]) * 64,
                         mailbox_offset=128 * rank, mailbox_ptr=1 << 40, mailbox_peers=2, mailbox_max_blocks=1536,
                         cache_handle=bytes([7]) * 64, cache_offset=0, cache_ptr=1 << 41,
                         cache_geometry={"kv_stride": 1, "layer_stride": 2, "block_stride": 3, "num_blocks": 4,
                                         "chunk_bytes": 5, "num_layers": 6, "dtype": "torch.bfloat16",
                                         "block_shape": (256, 8, 128)})
        recs = [None, None]
        dist.all_gather_object(recs, rec)
        ok = [r.rank for r in recs] == [0, 1] and recs[1 - rank].mailbox_handle == bytes([1 - rank]) * 64
        q.put({"rank": rank, "ok": ok})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put({"rank": rank, "ok": False, "error": repr(exc)})


def test_peer_records_exchange_over_gloo():
    out = _run(_record_worker)
    assert out[0]["ok"] and out[1]["ok"], out


def _dead_peer_worker(rank, port, q):
    try:
        dist = _init(rank, port, seconds=4)
        from lmpool_b200 import kv_transfer as kt

        if rank == 1:
            q.put({"rank": 1, "exited": True})
            q.close()
            q.join_thread()
            os._exit(0)   # leaves before the negotiation, between steps
        t0 = time.time()
        try:
            kt._recv_block_list(src=1)
            q.put({"rank": 0, "raised": False})
        except RuntimeError as exc:
            q.put({"rank": 0, "raised": True, "seconds": time.time() - t0, "msg": str(exc)[:200]})
    except Exception as exc:  # noqa: BLE001
        q.put({"rank": rank, "raised": True, "msg": repr(exc)})


def test_dead_peer_ends_in_an_error_not_a_hang():
    out = _run(_dead_peer_worker, timeout=90)
    assert out[1]["exited"]
    assert out[0]["raised"], out
