"""bench.py's host-side logic, on CPU: every name it uses resolves, the
benchmark-config-4 id sets are what the phase-B code assumes, and the
verification helpers catch a planted mistake (gloo ranks stand in for GPUs).
"""
import builtins
import dis
import os
import socket
import time
import types

import pytest
import torch
import torch.multiprocessing as mp

import bench


def _code_objects(code):
    yield code
    for const in code.co_consts:
        if isinstance(const, types.CodeType):
            yield from _code_objects(const)


def test_every_global_name_bench_uses_resolves():
    """A name deleted from the module but still used by a path (as the
    N>=4 phase-B helpers once were) fails here, without a GPU."""
    src = open(bench.__file__).read()
    missing = set()
    for code in _code_objects(compile(src, bench.__file__, "exec")):
        for ins in dis.get_instructions(code):
            if ins.opname in ("LOAD_GLOBAL", "LOAD_NAME") and not hasattr(bench, ins.argval) \
                    and not hasattr(builtins, ins.argval):
                missing.add(ins.argval)
    assert not missing, sorted(missing)


@pytest.mark.parametrize("world", [4, 8])
def test_phase_b_sets_are_disjoint_and_consistent(world):
    N, B = bench.PAIRS["N"], bench.PHASE_B_BLOCKS
    for r in range(world):
        incoming, outgoing = bench.all_partner_sets(N, world, r)
        assert sorted(incoming) == sorted(outgoing) == [x for x in range(world) if x != r]
        targets = [b for v in incoming.values() for b in v]
        assert len(targets) == len(set(targets)) == (world - 1) * B        # each block written once
        sources = {b for v in outgoing.values() for b in v}
        assert not sources & set(targets)                                   # never read and written at once
        assert all(len(v) == B and len(set(v)) == B for v in outgoing.values())
        assert all(0 <= b < N for b in list(sources) + targets)
    # what s sends to r has the length of what r reserves for s
    for s in range(world):
        for r in range(world):
            if s != r:
                assert len(bench.all_partner_sets(N, world, s)[1][r]) == len(bench.all_partner_sets(N, world, r)[0][s])


def test_both_arms_print_the_same_config():
    for world, g in ((1, bench.LOCAL), (2, bench.PAIRS), (8, bench.PAIRS)):
        a = bench.line_config(g, world)
        b = bench.line_config(dict(g), world)
        assert a == b and a["workload"] == g["workload"]


def test_fingerprints_see_any_change_and_nothing_else():
    cache = torch.randn(2, 3, 10, 4, 2, 8).to(torch.bfloat16)
    before = bench.block_fingerprints(cache, chunk=3)
    assert before.shape == (10,)
    cache[1, 2, 7, 3, 1, 5] = cache[1, 2, 7, 3, 1, 5] + 1
    cache[:, :, [2, 4]] = cache[:, :, [4, 2]]                         # swapped blocks
    after = bench.block_fingerprints(cache, chunk=3)
    assert (before != after).nonzero().flatten().tolist() == [2, 4, 7]
    assert bench.untouched_unchanged(before, after, [2, 4, 7]) == {"blocks_checked": 7, "blocks_changed": 0}
    assert bench.untouched_unchanged(before, after, [2, 4])["blocks_changed"] == 1


def test_local_verification_counts_mismatched_chunks():
    cache = torch.randn(2, 3, 10, 4, 2, 8).to(torch.bfloat16)
    cache[:, :, [5, 6]] = cache[:, :, [0, 1]]
    assert bench.verify_local(cache, [0, 1], [5, 6]) == {"chunks_checked": 12, "chunks_mismatched": 0}
    cache[0, 1, 6, 0, 0, 0] += 1
    assert bench.verify_local(cache, [0, 1], [5, 6])["chunks_mismatched"] == 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _verify_worker(rank, port, q, plant):
    import torch.distributed as dist

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        g = torch.Generator().manual_seed(rank)
        cache = torch.randn(2, 2, 12, 4, 2, 8, generator=g).to(torch.bfloat16)
        other = torch.randn(2, 2, 12, 4, 2, 8, generator=torch.Generator().manual_seed(1 - rank)).to(torch.bfloat16)
        src = {0: [3, 1, 3], 1: [0, 5, 9]}          # what each rank sends (a repeated id is legal)
        dst = {0: [7, 8, 2], 1: [4, 6, 10]}         # where each rank receives its partner's blocks
        peer = 1 - rank
        cache[:, :, dst[rank]] = other[:, :, src[peer]]   # what a correct transfer leaves behind
        if plant and rank == 1:
            cache[1, 1, 6, 2, 1, 3] += 1            # one wrong element in one chunk
        res = bench.verify_moves(cache, {peer: src[rank]}, {peer: dst[rank]}, dist)
        q.put({"rank": rank, "res": res})
        dist.destroy_process_group()
    except Exception as exc:  # noqa: BLE001
        q.put({"rank": rank, "error": repr(exc)})


@pytest.mark.parametrize("plant", [False, True])
def test_verify_moves_against_the_sent_bytes_over_two_ranks(plant):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_verify_worker, args=(r, port, q, plant)) for r in range(2)]
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
    assert len(out) == 2 and all("error" not in v for v in out.values()), out
    for r in (0, 1):
        assert out[r]["res"] == {"chunks_checked": 2 * 2 * 3 * 2, "chunks_mismatched": 1 if plant else 0}
